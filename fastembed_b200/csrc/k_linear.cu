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
                    tma_store_2d(&tm_y, buf, col0, m0 + q * 32);
                    bulk_commit();
                }
                pp ^= 1;
            }
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

}  // namespace

cudaError_t launch_linear_bf16(const void *x, const void *w, const float *bias,
                               const float *residual, void *y, int64_t m, int64_t n, int64_t k,
                               int epilogue, int y_dtype, cudaStream_t s, fe_status *st)
{
    *st = FE_OK;
    if (m == 0 || n == 0) return cudaSuccess;
    const int BN = (n % 256 == 0 || n > 1024) ? 256 : 128;
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
    if (BN == 256)
        return out_bf16 ? launch<256, true>(tx, tw, ty, M, N, K, bias, residual, epilogue, status, s)
                        : launch<256, false>(tx, tw, ty, M, N, K, bias, residual, epilogue, status, s);
    return out_bf16 ? launch<128, true>(tx, tw, ty, M, N, K, bias, residual, epilogue, status, s)
                    : launch<128, false>(tx, tw, ty, M, N, K, bias, residual, epilogue, status, s);
}

}  // namespace fe
