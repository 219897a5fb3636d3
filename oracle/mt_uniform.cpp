// mt_uniform.cpp — seeded input generator used by the reference's GTest files.
//
// TEST INFRASTRUCTURE ONLY (parity checker inputs; never linked into the product).
// tests/matrix_ops_test.cpp:20-26 and tests/attention_ops_test.cpp:17-32 of the
// reference build every tensor with a fresh std::mt19937(42) and
// std::uniform_real_distribution<float>(-1, 1).  Re-creating that stream here lets
// the parity tests feed the CUDA path exactly the inputs the reference tests use.
#include <cstddef>
#include <cstdint>
#include <random>

#include "fe_oracle.h"

extern "C" void fe_oracle_fill_uniform_mt19937(uint32_t seed, float lo, float hi, float *out,
                                               size_t count)
{
    std::mt19937 gen(seed);
    std::uniform_real_distribution<float> dist(lo, hi);
    for (size_t i = 0; i < count; ++i) out[i] = dist(gen);
}
