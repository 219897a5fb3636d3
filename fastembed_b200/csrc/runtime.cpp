// runtime.cpp — library plumbing: per-thread error text, the per-device status word,
// cached device properties and TMA descriptor encoding (cuTensorMapEncodeTiled,
// fetched through the runtime's driver entry-point query so the library needs no
// link-time dependency on libcuda).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <string>

#include "fe_internal.h"

namespace fe {

namespace {
thread_local std::string g_last_error;
constexpr int kMaxDevices = 64;
std::mutex g_mu;
int *g_status_words[kMaxDevices] = {};
uint64_t g_status_ctx[kMaxDevices] = {};  // context each status word was allocated in
int g_sm_count[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);
CtxGetCurrentFn g_ctx_current = nullptr;
CtxGetIdFn g_ctx_id = nullptr;
std::once_flag g_ctx_once;

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
}  // namespace

fe_status fail(fe_status s, const std::string &msg)
{
    g_last_error = msg;
    return s;
}

fe_status check_cuda(cudaError_t err, const char *what)
{
    if (err == cudaSuccess) return FE_OK;
    cudaGetLastError();  // clear a sticky launch error so the next call starts clean
    const fe_status s = err == cudaErrorMemoryAllocation ? FE_ERR_OUT_OF_MEMORY : FE_ERR_CUDA;
    return fail(s, std::string(what) + ": " + cudaGetErrorName(err) + " (" + cudaGetErrorString(err) + ")");
}

uint64_t current_context_id()
{
    std::call_once(g_ctx_once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_current = reinterpret_cast<CtxGetCurrentFn>(fn);
        fn = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_id = reinterpret_cast<CtxGetIdFn>(fn);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!g_ctx_current || !g_ctx_id || g_ctx_current(&ctx) != CUDA_SUCCESS)
        return 1;  // unknown: caches then behave as if the context never changes
    if (!ctx) {  // no context current on this thread yet: make the device's primary context current
        cudaFree(nullptr);
        if (g_ctx_current(&ctx) != CUDA_SUCCESS || !ctx) return 1;
    }
    if (g_ctx_id(ctx, &id) != CUDA_SUCCESS) return 1;
    return static_cast<uint64_t>(id) + 2;
}

int *device_status_word(int device)
{
    if (device < 0 || device >= kMaxDevices) return nullptr;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != device) cudaSetDevice(device);
    const uint64_t ctx = current_context_id();
    int *word = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_status_words[device] || g_status_ctx[device] != ctx) {
            // first use on this device, or the device was reset since: the word lives in the current context
            int *p = nullptr;
            g_status_words[device] = nullptr;
            if (cudaMalloc(&p, sizeof(int)) == cudaSuccess) {
                cudaMemset(p, 0, sizeof(int));
                cudaDeviceSynchronize();
                g_status_words[device] = p;
                g_status_ctx[device] = ctx;
            }
        }
        word = g_status_words[device];
    }
    if (prev != device) cudaSetDevice(prev);
    return word;
}

int *current_device_status_word()
{
    int dev = 0;
    cudaGetDevice(&dev);
    return device_status_word(dev);
}

int current_sm_count()
{
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) return 148;
    if (!g_sm_count[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_sm_count[dev] = n > 0 ? n : 148;
    }
    return g_sm_count[dev];
}

bool pdl_enabled()
{
    static const bool on = [] {
        const char *v = getenv("FE_PDL");
        return v && v[0] == '1';
    }();
    return on;
}

namespace {
fe_status load_encode()
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            return fail(FE_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
        g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    return FE_OK;
}
}  // namespace

fe_status make_tmap_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int elem_bytes,
                       uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows, uint32_t box_cols,
                       CUtensorMapSwizzle swizzle)
{
    FE_TRY(load_encode());
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
        return fail(FE_ERR_INVALID_ARGUMENT, "TMA operand base must be 16-byte aligned");
    if ((ld * elem_bytes) % 16 != 0)
        return fail(FE_ERR_INVALID_ARGUMENT, "TMA operand row stride must be a multiple of 16 bytes");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * static_cast<uint64_t>(elem_bytes)};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[160];
        std::snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d) for [%llu x %llu] box [%u x %u]",
                      static_cast<int>(r), static_cast<unsigned long long>(rows),
                      static_cast<unsigned long long>(cols), box_rows, box_cols);
        return fail(FE_ERR_CUDA, buf);
    }
    return FE_OK;
}

fe_status make_tmap_heads(CUtensorMap *map, const void *base, uint64_t heads, uint64_t rows, uint32_t box_rows)
{
    FE_TRY(load_encode());
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
        return fail(FE_ERR_INVALID_ARGUMENT, "TMA operand base must be 16-byte aligned");
    cuuint64_t dims[3] = {64, rows, heads};
    cuuint64_t strides[2] = {64 * 2, rows * 64 * 2};
    cuuint32_t box[3] = {64, box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(FE_ERR_CUDA, "cuTensorMapEncodeTiled failed for a head-major tensor");
    return FE_OK;
}

}  // namespace fe

extern "C" {

const char *fe_status_string(fe_status s)
{
    switch (s) {
        case FE_OK: return "ok";
        case FE_ERR_INVALID_ARGUMENT: return "invalid argument";
        case FE_ERR_CUDA: return "CUDA error";
        case FE_ERR_OUT_OF_MEMORY: return "out of device memory";
        case FE_ERR_UNSUPPORTED: return "unsupported";
        case FE_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
        case FE_ERR_IO: return "I/O error";
        case FE_ERR_NOT_FOUND: return "not found";
    }
    return "unknown status";
}

const char *fe_last_error_message(void) { return fe::g_last_error.c_str(); }

const char *fe_version(void) { return "fastembed_b200 0.1 (sm_100a)"; }

fe_status fe_set_wait_limit(int device, uint64_t limit_ns)
{
    if (limit_ns == 0) return fe::fail(FE_ERR_INVALID_ARGUMENT, "fe_set_wait_limit: limit_ns must be > 0");
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return fe::check_cuda(e, "fe_set_wait_limit");
    if (device < 0 || device >= count) return fe::fail(FE_ERR_INVALID_ARGUMENT, "bad device index");
    int prev = 0;
    cudaGetDevice(&prev);
    e = cudaSetDevice(device);
    if (e == cudaSuccess) e = fe::set_wait_limit_linear(limit_ns);
    if (e == cudaSuccess) e = fe::set_wait_limit_attention(limit_ns);
    if (e == cudaSuccess) e = fe::set_wait_limit_attention_wide(limit_ns);
    cudaSetDevice(prev);
    return fe::check_cuda(e, "fe_set_wait_limit");
}

fe_status fe_device_status(int device)
{
    int *w = fe::device_status_word(device);
    if (!w) return fe::fail(FE_ERR_INVALID_ARGUMENT, "bad device index");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    int v = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(w, 0, sizeof(int));
    cudaSetDevice(prev);
    if (e != cudaSuccess) return fe::check_cuda(e, "fe_device_status");
    if (v == fe::DEV_TIMEOUT) return fe::fail(FE_ERR_DEVICE_TIMEOUT, "a kernel's bounded wait ran out");
    if (v == fe::DEV_BAD_INPUT)
        return fe::fail(FE_ERR_INVALID_ARGUMENT, "a kernel met an out-of-range token id or position");
    return FE_OK;
}

}  // extern "C"
