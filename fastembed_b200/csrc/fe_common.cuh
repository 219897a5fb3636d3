// fe_common.cuh — device helpers shared by the sm_100a kernels: bf16 packing,
// warp reductions, bounded mbarrier waits, TMA loads/stores and the tcgen05
// (TMEM / UMMA) instruction wrappers, written as inline PTX.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fe_internal.h"

namespace fe {

// A bounded wait gives up after this many nanoseconds of %globaltimer; any wait
// that is correct finishes in microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
// Limits below this are checked at every poll instead of every 256th.
constexpr uint64_t kShortWaitNs = 1000000ull;

// The limit of the waits that guard work (a stage, an accumulator, a peer's row
// statistics), settable per device and per kernel file through fe_set_wait_limit: each
// .cu file that includes this header has its own copy, set by its own
// set_wait_limit_*() host function.  The drain waits that let a CTA's own copies and
// MMAs land before it exits (mbar_wait_drain) always use kWaitLimitNs.
static __constant__ uint64_t c_wait_limit_ns = kWaitLimitNs;

static inline cudaError_t set_wait_limit_this_file(uint64_t ns)
{
    return cudaMemcpyToSymbol(c_wait_limit_ns, &ns, sizeof(ns));
}

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi)
{
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t u)
{
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162 *>(&u);
    return __bfloat1622float2(v);
}

__device__ __forceinline__ void report(int *status, int code)
{
    if (status) atomicCAS(status, 0, code);
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking test of a phase (never suspends the thread): for polling several
// barriers in turn.
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t wait_limit_ns() { return c_wait_limit_ns; }

// Waits for the phase with the given parity to complete.  Returns false (and the
// caller must abandon its work) if the work-wait limit (wait_limit_ns) elapses first.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t limit = wait_limit_ns();
    const bool every = limit < kShortWaitNs;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (((i & 255u) == 0 || every) && globaltimer_ns() - t0 > limit) return false;
    }
}

// mbar_wait for the drain before a CTA exits: waits for copies and MMAs that this CTA
// started, which always complete, so it keeps the fixed kWaitLimitNs whatever the
// work-wait limit is.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t *bar, uint32_t parity)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// ------------------------------------------------ programmatic dependent launch
// A kernel launched by launch_k() may start (its CTAs become resident and run their
// set-up) while the previous kernel in its stream is still running.  grid_dep_wait()
// blocks until that kernel has completed and its memory is visible: every CTA calls it
// before its first access to a buffer that another kernel reads or writes, and before
// allocating TMEM.  grid_dep_launch() lets the next kernel start launching; a CTA calls
// it after its own TMEM allocation, so a successor waiting on the same SM never holds
// columns that this kernel still needs.  Both are no-ops for a plain launch.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launches a kernel that calls grid_dep_wait(), with programmatic stream serialisation
// when pdl_enabled().  Arguments are converted to the kernel's parameter types.
template <typename... KArgs, typename... Args>
__host__ cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args &&...args)
{
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<Args &&>(args)...);
}

// ----------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// 2-D tiled bulk tensor load into this CTA's shared memory, completing on `bar`.
// x is the innermost (contiguous) coordinate in elements.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x,
                                            int y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Prefetches a 2-D tile into L2 (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap *map, int x, int y)
{
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y)
                 : "memory");
}

// L2 eviction-priority policies for the cache-hinted TMA forms below.
__device__ __forceinline__ uint64_t l2_policy_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// tma_load_2d with an L2 cache-policy hint.
__device__ __forceinline__ void tma_load_2d_hint(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y,
                                                 uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
        : "memory");
}

// tma_store_2d with an L2 cache-policy hint.
__device__ __forceinline__ void tma_store_2d_hint(const CUtensorMap *map, const void *src, int x, int y,
                                                  uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
            map),
        "r"(smem_u32(src)), "r"(x), "r"(y), "l"(policy)
        : "memory");
}

// 3-D tiled bulk tensor load (x innermost), completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// 3-D tiled bulk tensor store from shared memory; elements outside the tensor are
// not written.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int x, int y, int z)
{
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
                 "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
                 : "memory");
}

// 2-D tiled bulk tensor store from shared memory; elements outside the tensor
// are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x, int y)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     map),
                 "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until at most N committed bulk groups are still reading shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read()
{
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_all()
{
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA / tensor core) reads of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// -------------------------------------------------------------------- tcgen05
// Allocates `ncols` TMEM columns (power of two, >= 32); whole warp executes.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem) (+)= A(smem desc) · B(smem desc)^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D(tmem) (+)= A(tmem) · B(smem desc)^T, kind::f16.  A is M=128 rows in TMEM lanes
// 0..127, two bf16 per 32-bit column along K.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// True in exactly one lane of a converged warp (elect.sync).  The MMA-issuing warps run
// their loop on all 32 lanes (the barrier waits and descriptor arithmetic are warp-uniform)
// and let the elected lane issue each tcgen05.mma / tcgen05.commit: issuing from a lone
// divergent lane measured about 20 % slower per instruction.
__device__ __forceinline__ bool elect_lane()
{
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
        "elect.sync rx|px, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, px;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// Arrives once on `bar` when every tcgen05.mma issued so far by this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// tcgen05.wait::ld that also names the registers of a pending tcgen05.ld as in/out
// operands, so that no use of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[32])
{
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// 32 lanes x 32 bit, 32 consecutive columns: thread i of the warp receives lane
// (lane base of taddr + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// 32 lanes x 32 bit, 16 consecutive columns: thread i of the warp writes lane
// (lane base of taddr + i), columns [col, col + 16).
__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------- grid-wide flags in global memory
__device__ __forceinline__ int ld_acquire_gpu(const int *p)
{
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int ld_relaxed_gpu(const int *p)
{
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ void red_release_gpu_add(int *p, int v)
{
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Shared-memory matrix descriptor for a K-major (or MN-major) operand laid out in
// 128-byte-swizzled atoms (8 rows x 128 B, 1024-byte aligned), as written by a TMA
// load with CU_TENSOR_MAP_SWIZZLE_128B.  Fields (sm_100 format): start address>>4
// [0,14), leading byte offset>>4 [16,30), stride byte offset>>4 [32,46),
// version 1 at [46,48), layout type 2 (128B swizzle) at [61,64).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes)
{
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
//   [4,6) D format (1 = f32), [7,10) A format (1 = bf16), [10,13) B format (1 = bf16),
//   bit 15 A major (0 = K), bit 16 B major (1 = MN), [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn_major, bool b_mn_major)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) |
           ((b_mn_major ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------- 2-CTA (cluster pair)
__device__ __forceinline__ uint32_t cluster_ctarank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address, in the shared::cluster window, of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(const void *p, uint32_t rank)
{
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
    return out;
}

// Arrive on an mbarrier given by its shared::cluster address (possibly the peer CTA's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t cluster_addr, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_addr),
                 "r"(bytes)
                 : "memory");
}

// 2-D TMA load into this CTA's shared memory whose completion is counted on the
// mbarrier at `bar_cluster_addr` (the pair leader's), for 2-CTA MMA operands.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, uint32_t bar_cluster_addr, int x,
                                                 int y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(bar_cluster_addr), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 2-CTA MMA issued by the pair leader: A rows 0..127 from this CTA's smem and 128..255
// from the peer's (same offset); B rows split the same way; D in both CTAs' TMEM.
__device__ __forceinline__ void umma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Commit of the pair's MMAs arriving on the barrier at the same offset in both CTAs.
__device__ __forceinline__ void umma_commit_pair_both(uint64_t *bar)
{
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(static_cast<uint16_t>(3))
        : "memory");
}

// tanh-form GELU (src/ops/cpu/cpu_matrix_ops.cpp:35-43) with the hardware tanh
// approximation; used where the result is rounded to bf16.
__device__ __forceinline__ float gelu_tanh_fast(float x)
{
    // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), arranged as
    // u = x (c0 + c1 x^2), h = x / 2, h + h tanh(u): four FP32 operations and one MUFU
    const float c0 = 0.7978845608028654f;              // sqrt(2/pi)
    const float c1 = 0.7978845608028654f * 0.044715f;  // sqrt(2/pi) * 0.044715
    const float u = x * fmaf(c1, x * x, c0);
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
    const float h = 0.5f * x;
    return fmaf(h, t, h);
}

// sin and cos of an angle: Cody-Waite reduction to [-pi, pi] with 2 pi split in two
// floats (the high part exact in the FMA, the low part the rounding error of the first),
// then the hardware sin / cos, accurate to about 1e-6 on that interval.  Angles here are
// position * inverse frequency, below 2^17, where the two-constant reduction is exact to
// float rounding.
__device__ __forceinline__ void sincos_reduced(float a, float &s, float &c)
{
    constexpr double kTwoPi = 6.283185307179586476925286766559;
    constexpr float kHi = static_cast<float>(kTwoPi);
    constexpr float kLo = static_cast<float>(kTwoPi - static_cast<double>(kHi));
    constexpr float kInv = static_cast<float>(1.0 / kTwoPi);
    const float k = rintf(a * kInv);
    float r = fmaf(-k, kHi, a);
    r = fmaf(-k, kLo, r);
    s = __sinf(r);
    c = __cosf(r);
}

// sin and cos of the rotary angle of (position, frequency index): inv_freq = theta^(-2 fi / HD),
// angle = position * inv_freq in fp32.  Measured: the reduced hardware form is faster at
// head_dim 128 (4 angles a lane), sincosf at 256 (8 angles a lane, 4 heads a token).
template <int HD>
__device__ __forceinline__ void rope_angle(int pos, int fi, float log2_theta, float &sn, float &cs)
{
    const float inv_freq = exp2f(-log2_theta * static_cast<float>(2 * fi) / static_cast<float>(HD));
    if constexpr (HD == 128) sincos_reduced(static_cast<float>(pos) * inv_freq, sn, cs);
    else sincosf(static_cast<float>(pos) * inv_freq, &sn, &cs);
}

// max(a, b, c) in one instruction (sm_100 three-input max)
__device__ __forceinline__ float max3f(float a, float b, float c)
{
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// (a, b) <- (xa * y + z, xb * y + z) as one packed f32x2 fma (each lane an IEEE fma)
__device__ __forceinline__ void fma_f32x2(float &a, float &b, float xa, float xb, float y, float z)
{
    unsigned long long x, yy, zz, d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(xa), "f"(xb));
    asm("mov.b64 %0, {%1, %1};" : "=l"(yy) : "f"(y));
    asm("mov.b64 %0, {%1, %1};" : "=l"(zz) : "f"(z));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(x), "l"(yy), "l"(zz));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(d));
}

// (a, b) <- (xa * ya + za, xb * yb + zb) as one packed f32x2 fma
__device__ __forceinline__ void fma_f32x2v(float &a, float &b, float xa, float xb, float ya, float yb, float za,
                                           float zb)
{
    unsigned long long x, y, z, d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(xa), "f"(xb));
    asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(ya), "f"(yb));
    asm("mov.b64 %0, {%1, %2};" : "=l"(z) : "f"(za), "f"(zb));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(x), "l"(y), "l"(z));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(d));
}

// a *= c, b *= d as one packed f32x2 multiply
__device__ __forceinline__ void mul_f32x2(float &a, float &b, float c, float d)
{
    unsigned long long x, y;
    asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a), "f"(b));
    asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(c), "f"(d));
    asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(x) : "l"(y));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(x));
}

// a += c, b += d as one packed f32x2 add (round to nearest, as the scalar adds)
__device__ __forceinline__ void add_f32x2(float &a, float &b, float c, float d)
{
    unsigned long long x, y;
    asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a), "f"(b));
    asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(c), "f"(d));
    asm("add.rn.f32x2 %0, %0, %1;" : "+l"(x) : "l"(y));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(x));
}

// silu(a) = a / (1 + e^-a) of two values: e^-a by ex2.approx, the division by
// rcp.approx (both MUFU), the FP32 arithmetic as packed f32x2 instructions.  Saturates
// correctly: e^-a = inf gives a * 0, e^-a = 0 gives a.
__device__ __forceinline__ void silu_fast2(float &a, float &b)
{
    float e0 = -1.4426950408889634f * a, e1 = -1.4426950408889634f * b;
    asm("ex2.approx.ftz.f32 %0, %0;" : "+f"(e0));
    asm("ex2.approx.ftz.f32 %0, %0;" : "+f"(e1));
    add_f32x2(e0, e1, 1.0f, 1.0f);
    asm("rcp.approx.ftz.f32 %0, %0;" : "+f"(e0));
    asm("rcp.approx.ftz.f32 %0, %0;" : "+f"(e1));
    mul_f32x2(a, b, e0, e1);
}

// gelu_tanh_fast of two values with the packed f32x2 FP32 instructions of sm_100 (the
// same operations per lane, so the results equal the scalar form's).
__device__ __forceinline__ void gelu_tanh_fast2(float &a, float &b)
{
    const float c0 = 0.7978845608028654f;
    const float c1 = 0.7978845608028654f * 0.044715f;
    unsigned long long x, k0, k1, kh, x2, p, u, h, t, o;
    asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a), "f"(b));
    asm("mov.b64 %0, {%1, %1};" : "=l"(k0) : "f"(c0));
    asm("mov.b64 %0, {%1, %1};" : "=l"(k1) : "f"(c1));
    asm("mov.b64 %0, {%1, %1};" : "=l"(kh) : "f"(0.5f));
    asm("mul.rn.f32x2 %0, %1, %1;" : "=l"(x2) : "l"(x));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(p) : "l"(k1), "l"(x2), "l"(k0));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(u) : "l"(x), "l"(p));
    float u0, u1, t0, t1;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(u0), "=f"(u1) : "l"(u));
    asm("tanh.approx.f32 %0, %1;" : "=f"(t0) : "f"(u0));
    asm("tanh.approx.f32 %0, %1;" : "=f"(t1) : "f"(u1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(t) : "f"(t0), "f"(t1));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(h) : "l"(kh), "l"(x));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(o) : "l"(h), "l"(t), "l"(h));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(o));
}

}  // namespace fe
