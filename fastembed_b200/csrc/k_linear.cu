// k_linear.cu — tcgen05 linear layer: y = epilogue(x · W^T), bf16 in, fp32 accumulate.
//
// Replaces the model's projection GEMMs and their host bias / activation / residual
// loops (src/sentence_transformers_impl.cpp:250-263 and :403-436; QKV at
// src/ops/cuda/cuda_attention_ops.cu:227-248).
//
// Design (one CTA per SM, persistent over 128 x BN output tiles, n fastest so the
// CTAs in flight share each 128-row block of x through L2):
//   warp 0      TMA producer: x tile [128 x 64] and W tile [BN x 64] per stage into
//               a STAGES-deep ring of 128B-swizzled shared-memory buffers.
//   warp 1      TMEM owner and MMA issuer: one thread issues tcgen05.mma
//               (M=128, N=BN, K=16) x 4 per stage into one of two TMEM accumulators,
//               tcgen05.commit frees the smem stage / publishes the accumulator.
//   warps 2-5   epilogue: each warp drains its 32 TMEM lanes (= 32 rows) with
//               tcgen05.ld, applies bias / activation / residual, writes a 32-row x
//               128-byte slab to swizzled shared memory and TMA-stores it; the other
//               accumulator is being filled meanwhile.
// Every mbarrier wait is bounded; on timeout the CTA records FE_ERR_DEVICE_TIMEOUT
// in the device status word, drains what it started and exits.
#include <cuda.h>
#include <cuda_bf16.h>

#include <cstdlib>

#include "fe_common.cuh"
#include "fe_internal.h"

namespace fe {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kEpiWarps = 4;
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer, mma, 4 epilogue warps
constexpr uint32_t kStageBufBytes = 32 * 128;  // one warp's 32-row x 128 B store slab

enum Epi : int { E_NONE = 0, E_BIAS = 1, E_GELU = 2, E_RELU = 3, E_SWISH = 4, E_RESID = 5 };

template <int BN>
struct Cfg {
    static constexpr int STAGES = BN == 256 ? 4 : 6;
    static constexpr uint32_t A_BYTES = BM * BK * 2;
    static constexpr uint32_t B_BYTES = BN * BK * 2;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr uint32_t TMEM_COLS = 2 * BN;
    static constexpr uint32_t RING_BYTES = STAGES * STAGE_BYTES;
    static constexpr uint32_t EPI_BYTES = kEpiWarps * 2 * kStageBufBytes;
    static constexpr uint32_t BAR_BYTES = 256;
    static constexpr uint32_t SMEM_BYTES = 1024 + RING_BYTES + EPI_BYTES + BAR_BYTES;
};

__device__ __forceinline__ float act(float x, int epi)
{
    if (epi == E_GELU) return gelu_tanh_fast(x);
    if (epi == E_RELU) return x > 0.f ? x : 0.f;
    if (epi == E_SWISH) return x / (1.0f + __expf(-x));
    return x;
}

// Drains one 128-row x BN accumulator from TMEM (this warp's 32 lanes = 32 rows):
// bias / activation / residual epilogue, then 32-row x 128-byte slabs staged in
// 128B-swizzled shared memory and written by TMA (rows >= M and columns >= N are
// clipped by the tensor map).  `row` is this thread's output row, `store_row` the
// warp's first row.
template <int BN, bool OUT_BF16>
__device__ __forceinline__ void drain_accumulator(uint32_t t_row, int row, int store_row, int n0, int M, int N,
                                                  const float *__restrict__ bias,
                                                  const float *__restrict__ residual, int epi,
                                                  const CUtensorMap *tm_y, uint8_t *bufs, int &pp, int lane)
{
    constexpr int CHUNK = OUT_BF16 ? 64 : 32;  // output columns per 128-byte slab
#pragma unroll 1
    for (int c = 0; c < BN; c += CHUNK) {
        float f[CHUNK];
#pragma unroll
        for (int h = 0; h < CHUNK / 32; ++h) {
            uint32_t v[32];
            tmem_ld_x32(t_row + c + h * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) f[h * 32 + j] = __uint_as_float(v[j]);
        }
        const int col0 = n0 + c;
        if (epi != E_NONE) {
            if (col0 + CHUNK <= N) {
#pragma unroll
                for (int j = 0; j < CHUNK; j += 4) {
                    const float4 bb = __ldg(reinterpret_cast<const float4 *>(bias + col0 + j));
                    f[j] += bb.x;
                    f[j + 1] += bb.y;
                    f[j + 2] += bb.z;
                    f[j + 3] += bb.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < CHUNK; ++j)
                    if (col0 + j < N) f[j] += __ldg(bias + col0 + j);
            }
        }
        if (epi == E_RESID) {
            if (row < M) {
                const float *rp = residual + static_cast<size_t>(row) * N + col0;
                if (col0 + CHUNK <= N) {
#pragma unroll
                    for (int j = 0; j < CHUNK; j += 4) {
                        const float4 rr = __ldg(reinterpret_cast<const float4 *>(rp + j));
                        f[j] += rr.x;
                        f[j + 1] += rr.y;
                        f[j + 2] += rr.z;
                        f[j + 3] += rr.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < CHUNK; ++j)
                        if (col0 + j < N) f[j] += rp[j];
                }
            }
        } else if (epi >= E_GELU) {
#pragma unroll
            for (int j = 0; j < CHUNK; ++j) f[j] = act(f[j], epi);
        }
        // Stage the warp's 32 x 128 B slab (128B-swizzled) and TMA-store it.
        uint8_t *buf = bufs + pp * kStageBufBytes;
        if (lane == 0) bulk_wait_read<1>();  // the store that last used `buf` has read it
        __syncwarp();
        uint8_t *rowp = buf + lane * 128;
#pragma unroll
        for (int c16 = 0; c16 < 8; ++c16) {
            uint4 w;
            if constexpr (OUT_BF16) {
                w.x = pack_bf16x2(f[c16 * 8 + 0], f[c16 * 8 + 1]);
                w.y = pack_bf16x2(f[c16 * 8 + 2], f[c16 * 8 + 3]);
                w.z = pack_bf16x2(f[c16 * 8 + 4], f[c16 * 8 + 5]);
                w.w = pack_bf16x2(f[c16 * 8 + 6], f[c16 * 8 + 7]);
            } else {
                w.x = __float_as_uint(f[c16 * 4 + 0]);
                w.y = __float_as_uint(f[c16 * 4 + 1]);
                w.z = __float_as_uint(f[c16 * 4 + 2]);
                w.w = __float_as_uint(f[c16 * 4 + 3]);
            }
            *reinterpret_cast<uint4 *>(rowp + ((c16 ^ (lane & 7)) << 4)) = w;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            tma_store_2d(tm_y, buf, col0, store_row);
            bulk_commit();
        }
        pp ^= 1;
    }
}

template <int BN, bool OUT_BF16>
__global__ void __launch_bounds__(kThreads, 1)
    linear_tcgen05(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_y, int M, int N, int K,
                   const float *__restrict__ bias, const float *__restrict__ residual, int epi,
                   int *status)
{
    using C = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = smem;
    uint8_t *epi_buf = smem + C::RING_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(epi_buf + C::EPI_BYTES);
    uint64_t *empty = full + C::STAGES;
    uint64_t *acc_full = empty + C::STAGES;  // [2]
    uint64_t *acc_empty = acc_full + 2;      // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int m_tiles = (M + BM - 1) / BM;
    const int n_tiles = (N + BN - 1) / BN;
    const int num_tiles = m_tiles * n_tiles;
    const int k_iters = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 32 * kEpiWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_w);
        tma_prefetch_desc(&tm_y);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0, armed_parity = 0;  // per-stage: armed at least once / parity of last arm
            for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
                const int m0 = (tile / n_tiles) * BM;
                const int n0 = (tile % n_tiles) * BN;
                for (int kb = 0; kb < k_iters; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1)) {
                        report(status, DEV_TIMEOUT);
                        *abort_flag = 1;
                        break;
                    }
                    uint8_t *a_dst = ring + stage * C::STAGE_BYTES;
                    uint8_t *b_dst = a_dst + C::A_BYTES;
                    mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                    tma_load_2d(a_dst, &tm_x, &full[stage], kb * BK, m0);
                    tma_load_2d(b_dst, &tm_w, &full[stage], kb * BK, n0);
                    armed |= 1u << stage;
                    armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Drain: every load this thread started must land before the CTA exits.
            for (int s = 0; s < C::STAGES; ++s)
                if (armed & (1u << s))
                    if (!mbar_wait(&full[s], (armed_parity >> s) & 1u)) report(status, DEV_TIMEOUT);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, false, false);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool issued = false;
            for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
                if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1)) {
                    report(status, DEV_TIMEOUT);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < k_iters; ++kb) {
                    if (!mbar_wait(&full[stage], phase)) {
                        report(status, DEV_TIMEOUT);
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(ring + stage * C::STAGE_BYTES);
                    const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        const uint64_t ad = sdesc_sw128(a_addr + k * 32, 16, 1024);
                        const uint64_t bd = sdesc_sw128(b_addr + k * 32, 16, 1024);
                        umma_f16_ss(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    issued = true;
                    umma_commit(&empty[stage]);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (*abort_flag) break;
                umma_commit(&acc_full[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            if (*abort_flag && issued) {
                // Let outstanding MMAs retire before TMEM is released.
                uint64_t *probe = &acc_full[acc];
                umma_commit(probe);
                if (!mbar_wait(probe, acc_phase)) report(status, DEV_TIMEOUT);
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        uint8_t *bufs = epi_buf + q * 2 * kStageBufBytes;
        int acc = 0;
        uint32_t acc_phase = 0;
        int pp = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            if (*abort_flag) break;
            if (!mbar_wait(&acc_full[acc], acc_phase)) {
                report(status, DEV_TIMEOUT);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int m0 = (tile / n_tiles) * BM;
            const int n0 = (tile % n_tiles) * BN;
            const int row = m0 + q * 32 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
            drain_accumulator<BN, OUT_BF16>(t_row, row, m0 + q * 32, n0, M, N, bias, residual, epi, &tm_y, bufs, pp,
                                            lane);
            tc_fence_before();
            mbar_arrive(&acc_empty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
        if (lane == 0) bulk_wait_all<0>();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// 2-CTA variant: a cluster pair computes a 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256).  Each CTA stages its own 128 rows of x and its
// own 128 rows of W per k-block (32 KB a stage instead of 48 KB for the same work per
// CTA), so each stage costs a third less L2 -> SM traffic and six stages fit.  The
// leader (cluster rank 0) issues the MMAs; both CTAs' TMA loads complete on the
// leader's stage barrier; commits are multicast to the barriers of both CTAs; each
// CTA's epilogue drains its own 128 accumulator rows and reports back to the leader.
constexpr int P_STAGES = 6;
constexpr int P_BN = 256;
constexpr uint32_t P_HALF_BYTES = 128 * BK * 2;        // 16 KB: 128 rows x 64 bf16
constexpr uint32_t P_STAGE_BYTES = 2 * P_HALF_BYTES;   // this CTA's x rows + W rows
constexpr uint32_t P_TMEM_COLS = 2 * P_BN;
constexpr uint32_t P_RING_BYTES = P_STAGES * P_STAGE_BYTES;
constexpr uint32_t P_EPI_BYTES = kEpiWarps * 2 * kStageBufBytes;
constexpr uint32_t P_SMEM_BYTES = 1024 + P_RING_BYTES + P_EPI_BYTES + 256;

template <bool OUT_BF16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    linear_tcgen05_pair(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_y, int M, int N, int K,
                        const float *__restrict__ bias, const float *__restrict__ residual, int epi, int *status)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = smem;
    uint8_t *epi_buf = smem + P_RING_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(epi_buf + P_EPI_BYTES);  // used in the leader
    uint64_t *empty = full + P_STAGES;                                     // both CTAs
    uint64_t *acc_full = empty + P_STAGES;                                 // both CTAs [2]
    uint64_t *acc_empty = acc_full + 2;                                    // used in the leader [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1;
    const int npairs = gridDim.x >> 1;
    const int m_tiles = (M + 255) / 256;
    const int n_tiles = (N + P_BN - 1) / P_BN;
    const int num_tiles = m_tiles * n_tiles;
    const int k_iters = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 2 * kEpiWarps);  // one arrival per epilogue warp of either CTA
        }
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_w);
        tma_prefetch_desc(&tm_y);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, P_TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs)
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0, armed_parity = 0;
            for (int tile = pair; tile < num_tiles && !*abort_flag; tile += npairs) {
                const int m0 = (tile / n_tiles) * 256;
                const int n0 = (tile % n_tiles) * P_BN;
                for (int kb = 0; kb < k_iters; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1)) {
                        report(status, DEV_TIMEOUT);
                        *abort_flag = 1;
                        break;
                    }
                    uint8_t *a_dst = ring + stage * P_STAGE_BYTES;
                    uint8_t *b_dst = a_dst + P_HALF_BYTES;
                    const uint32_t leader_full = map_to_rank(&full[stage], 0);
                    if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
                    tma_load_2d_pair(a_dst, &tm_x, leader_full, kb * BK, m0 + static_cast<int>(rank) * 128);
                    tma_load_2d_pair(b_dst, &tm_w, leader_full, kb * BK, n0 + static_cast<int>(rank) * 128);
                    armed |= 1u << stage;
                    armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // The leader's stage barriers count both CTAs' bytes: it drains the pair's loads.
            if (rank == 0)
                for (int s = 0; s < P_STAGES; ++s)
                    if (armed & (1u << s))
                        if (!mbar_wait(&full[s], (armed_parity >> s) & 1u)) report(status, DEV_TIMEOUT);
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---------------- MMA issuer (leader only)
            constexpr uint32_t idesc = idesc_bf16_f32(256, P_BN, false, false);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool issued = false;
            for (int tile = pair; tile < num_tiles && !*abort_flag; tile += npairs) {
                if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1)) {
                    report(status, DEV_TIMEOUT);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * P_BN;
                for (int kb = 0; kb < k_iters; ++kb) {
                    if (!mbar_wait(&full[stage], phase)) {
                        report(status, DEV_TIMEOUT);
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(ring + stage * P_STAGE_BYTES);
                    const uint64_t ad = sdesc_sw128(a_addr, 16, 1024);
                    const uint64_t bd = sdesc_sw128(a_addr + P_HALF_BYTES, 16, 1024);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)  // +32 bytes per K step inside the swizzle atom
                        umma_f16_ss_pair(d_tmem, ad + static_cast<uint64_t>(k * 2), bd + static_cast<uint64_t>(k * 2),
                                         idesc, (kb | k) != 0 ? 1u : 0u);
                    issued = true;
                    umma_commit_pair_both(&empty[stage]);
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (*abort_flag) break;
                umma_commit_pair_both(&acc_full[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            if (*abort_flag && issued) {
                uint64_t *probe = &acc_full[acc];
                umma_commit_pair_both(probe);
                if (!mbar_wait(probe, acc_phase)) report(status, DEV_TIMEOUT);
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5 of both CTAs)
        const int q = warp & 3;
        uint8_t *bufs = epi_buf + q * 2 * kStageBufBytes;
        const uint32_t leader_acc_empty[2] = {map_to_rank(&acc_empty[0], 0), map_to_rank(&acc_empty[1], 0)};
        int acc = 0;
        uint32_t acc_phase = 0;
        int pp = 0;
        for (int tile = pair; tile < num_tiles; tile += npairs) {
            if (*abort_flag) break;
            if (!mbar_wait(&acc_full[acc], acc_phase)) {
                report(status, DEV_TIMEOUT);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int m0 = (tile / n_tiles) * 256 + static_cast<int>(rank) * 128;
            const int n0 = (tile % n_tiles) * P_BN;
            const int row = m0 + q * 32 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * P_BN;
            drain_accumulator<P_BN, OUT_BF16>(t_row, row, m0 + q * 32, n0, M, N, bias, residual, epi, &tm_y, bufs, pp,
                                              lane);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(leader_acc_empty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
        if (lane == 0) bulk_wait_all<0>();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no CTA leaves while its peer may still signal it or read its smem
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, P_TMEM_COLS);
    }
}

template <bool OUT_BF16>
cudaError_t launch_pair(const CUtensorMap &tx, const CUtensorMap &tw, const CUtensorMap &ty, int M, int N, int K,
                        const float *bias, const float *residual, int epi, int *status, cudaStream_t s)
{
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(linear_tcgen05_pair<OUT_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             P_SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const int tiles = ((M + 255) / 256) * ((N + P_BN - 1) / P_BN);
    int pairs = current_sm_count() / 2;
    if (pairs > tiles) pairs = tiles;
    if (pairs < 1) pairs = 1;
    linear_tcgen05_pair<OUT_BF16><<<2 * pairs, kThreads, P_SMEM_BYTES, s>>>(tx, tw, ty, M, N, K, bias, residual, epi,
                                                                           status);
    return cudaGetLastError();
}

template <int BN, bool OUT_BF16>
cudaError_t launch(const CUtensorMap &tx, const CUtensorMap &tw, const CUtensorMap &ty, int M, int N,
                   int K, const float *bias, const float *residual, int epi, int *status,
                   cudaStream_t s)
{
    using C = Cfg<BN>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(linear_tcgen05<BN, OUT_BF16>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    int grid = current_sm_count();
    if (grid > tiles) grid = tiles;
    if (grid < 1) grid = 1;
    linear_tcgen05<BN, OUT_BF16><<<grid, kThreads, C::SMEM_BYTES, s>>>(tx, tw, ty, M, N, K, bias,
                                                                       residual, epi, status);
    return cudaGetLastError();
}

// The 2-CTA kernel is the default for large M; FE_LINEAR_PAIR=0 selects the 1-CTA
// kernel for every shape (both compute the same result; tests run both).
bool pair_mode_enabled()
{
    const char *v = getenv("FE_LINEAR_PAIR");
    return !(v && v[0] == '0');
}

}  // namespace

cudaError_t launch_linear_bf16(const void *x, const void *w, const float *bias,
                               const float *residual, void *y, int64_t m, int64_t n, int64_t k,
                               int epilogue, int y_dtype, cudaStream_t s, fe_status *st)
{
    *st = FE_OK;
    if (m == 0 || n == 0) return cudaSuccess;
    const int BN = (n % 256 == 0 || n > 1024) ? 256 : 128;
    // 256-row pair tiles once there are at least two of them per 256 columns
    const bool use_pair = pair_mode_enabled() && BN == 256 && m >= 512;
    const bool out_bf16 = y_dtype == FE_DTYPE_BF16;
    CUtensorMap tx, tw, ty;
    fe_status r = make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m, k, k, BM, BK);
    if (r == FE_OK) r = make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, n, k, k, BN, BK);
    if (r == FE_OK)
        r = out_bf16 ? make_tmap_2d(&ty, y, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m, n, n, 32, 64)
                     : make_tmap_2d(&ty, y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, m, n, n, 32, 32);
    if (r != FE_OK) {
        *st = r;
        return cudaSuccess;
    }
    int *status = current_device_status_word();
    const int M = static_cast<int>(m), N = static_cast<int>(n), K = static_cast<int>(k);
    if (BN == 256 && use_pair) {
        CUtensorMap tw2;  // each CTA of a pair stages 128 rows of W
        r = make_tmap_2d(&tw2, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, n, k, k, 128, BK);
        if (r != FE_OK) {
            *st = r;
            return cudaSuccess;
        }
        return out_bf16 ? launch_pair<true>(tx, tw2, ty, M, N, K, bias, residual, epilogue, status, s)
                        : launch_pair<false>(tx, tw2, ty, M, N, K, bias, residual, epilogue, status, s);
    }
    if (BN == 256)
        return out_bf16 ? launch<256, true>(tx, tw, ty, M, N, K, bias, residual, epilogue, status, s)
                        : launch<256, false>(tx, tw, ty, M, N, K, bias, residual, epilogue, status, s);
    return out_bf16 ? launch<128, true>(tx, tw, ty, M, N, K, bias, residual, epilogue, status, s)
                    : launch<128, false>(tx, tw, ty, M, N, K, bias, residual, epilogue, status, s);
}

}  // namespace fe
