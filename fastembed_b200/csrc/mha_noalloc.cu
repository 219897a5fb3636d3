// mha_noalloc.cu — single-sequence FP32 multi-head attention that allocates nothing.
//
// fe_mha_f32 needs Q, K and V scratch and asks the caller for it.  Some callers cannot
// provide scratch on demand: a host whose device memory is owned by another
// framework's allocator (so a raw cudaMalloc would fight it or is forbidden), a
// latency-critical serving loop that must not call cudaMalloc / cudaFree because they
// can synchronise the device or fail part-way through a request, and code that runs
// after start-up in a process that forbids new allocations.  fe_mha_f32_noalloc
// serves them with a fixed scratch array that lives in the library image itself: it
// is created when the library is loaded onto a device and stays until the process
// exits.
//
// Limits and sharing:
//   * seq_len * dim must not exceed kNoAllocMaxElems (3 MiB of fp32 scratch in total:
//     Q, K and V of up to 262,144 elements each, e.g. 256 tokens at dim 1024 or 512
//     tokens at dim 512); larger sizes are rejected with FE_ERR_UNSUPPORTED.
//   * Every call on a device uses the same array.  Calls whose GPU work overlaps
//     (different streams, or host threads racing on one device) race on it and give
//     wrong results; order such calls on one stream.
//   * The scratch keeps the previous call's contents; nothing in it needs to start at
//     zero, because the three projections overwrite the Q, K and V they use before
//     anything reads them.
//   * The first call on each device looks up the array's device address (once per
//     device and CUDA context, with that device current); make that first call before
//     any CUDA stream capture on the device.
#include <cuda_runtime.h>

#include <mutex>

#include "fe_internal.h"

namespace {

constexpr int64_t kNoAllocMaxElems = 262144;  // per projection: Q, K and V each
constexpr int kMaxDevices = 64;

// The scratch: Q | K | V, each kNoAllocMaxElems floats, in device global memory.
static __device__ __align__(256) float g_mha_scratch[3 * kNoAllocMaxElems];

// Device address of g_mha_scratch per device, and the CUDA context it was looked up in.
// On the host the symbol name is only a handle for the runtime, not a device address,
// so it is never passed to a kernel.  After a cudaDeviceReset the library image is
// loaded again in the device's next context, possibly at another address, so the
// address is looked up again when the context changes.
std::mutex g_mu;
float *g_scratch_ptr[kMaxDevices] = {};
uint64_t g_scratch_ctx[kMaxDevices] = {};

fe_status scratch_for_current_device(float **out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fe::check_cuda(e, "fe_mha_f32_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fe::fail(FE_ERR_UNSUPPORTED, "fe_mha_f32_noalloc: device index too large");
    const uint64_t ctx = fe::current_context_id();
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_ptr[dev] || g_scratch_ctx[dev] != ctx) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_mha_scratch);
        if (e != cudaSuccess) return fe::check_cuda(e, "fe_mha_f32_noalloc: cudaGetSymbolAddress");
        g_scratch_ptr[dev] = static_cast<float *>(p);
        g_scratch_ctx[dev] = ctx;
    }
    *out = g_scratch_ptr[dev];
    return FE_OK;
}

}  // namespace

extern "C" fe_status fe_mha_f32_noalloc(const float *x, const float *wq, const float *wk, const float *wv,
                                        const float *bq, const float *bk, const float *bv, float *out,
                                        int64_t seq_len, int64_t dim, int64_t heads, fe_stream_t stream)
{
    if (heads <= 0 || dim <= 0 || seq_len < 0)
        return fe::fail(FE_ERR_INVALID_ARGUMENT, "fe_mha_f32_noalloc: bad shape");
    if (dim % heads != 0)
        return fe::fail(FE_ERR_INVALID_ARGUMENT, "Embedding dimension must be divisible by number of heads");
    if (seq_len == 0) return FE_OK;
    if (!x || !wq || !wk || !wv || !bq || !bk || !bv || !out)
        return fe::fail(FE_ERR_INVALID_ARGUMENT, "fe_mha_f32_noalloc: null pointer");
    if (seq_len > 0xffff || static_cast<size_t>(seq_len) * 4 > 200 * 1024)
        return fe::fail(FE_ERR_UNSUPPORTED, "fe_mha_f32_noalloc: sequence too long for the fp32 path");
    if (seq_len * dim > kNoAllocMaxElems)
        return fe::fail(FE_ERR_UNSUPPORTED,
                        "fe_mha_f32_noalloc: seq_len * dim exceeds the built-in scratch (262144 elements); "
                        "use fe_mha_f32 with a caller-provided workspace");
    float *scratch = nullptr;
    FE_TRY(scratch_for_current_device(&scratch));
    float *q = scratch;
    float *k = scratch + kNoAllocMaxElems;
    float *v = scratch + 2 * kNoAllocMaxElems;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    FE_TRY_CUDA(fe::launch_sgemm(x, wq, bq, q, seq_len, dim, dim, true, s));
    FE_TRY_CUDA(fe::launch_sgemm(x, wk, bk, k, seq_len, dim, dim, true, s));
    FE_TRY_CUDA(fe::launch_sgemm(x, wv, bv, v, seq_len, dim, dim, true, s));
    return fe::check_cuda(fe::launch_mha_core_f32(q, k, v, out, seq_len, dim, heads, s), "fe_mha_f32_noalloc");
}
