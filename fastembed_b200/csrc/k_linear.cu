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
//   warp 1      TMEM owner and MMA issuer: the warp waits, one elected lane issues tcgen05.mma
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

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "fe_common.cuh"
#include "fe_internal.h"

namespace fe {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kEpiWarps = 4;
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer, mma, 4 epilogue warps
constexpr uint32_t kStageBufBytes = 32 * 128;  // one warp's 32-row x 128 B store slab
constexpr uint32_t kRopeTabBytes = 128 * 4;     // inverse RoPE frequencies of the q/k epilogue (head_dim / 2)

enum Epi : int {
    E_NONE = 0, E_BIAS = 1, E_GELU = 2, E_RELU = 3, E_SWISH = 4, E_RESID = 5, E_SWIGLU = 6, E_GEGLU = 7,
    E_QKROPE = 8  // per-head q/k RMSNorm + rotary embedding of a QKV projection (RopeParams)
};

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
    static constexpr uint32_t SMEM_BYTES = 1024 + RING_BYTES + EPI_BYTES + BAR_BYTES + kRopeTabBytes;
};

__device__ __forceinline__ float act(float x, int epi)
{
    if (epi == E_GELU) return gelu_tanh_fast(x);
    if (epi == E_RELU) return x > 0.f ? x : 0.f;
    if (epi == E_SWISH) return x / (1.0f + __expf(-x));
    return x;
}

// Per-head RMSNorm of the query and key heads followed by the rotate-half rotary embedding,
// applied to a QKV projection's accumulator before it is rounded to bf16 (E_QKROPE): the
// Qwen3 / Gemma3 q_norm / k_norm and RoPE, which otherwise run as a separate pass over the
// bf16 qkv buffer.  Columns [0, q_cols) are query heads, [q_cols, k_end) key heads, the
// rest value heads (stored as they are); every head-group boundary falls on a 256-column
// tile boundary, so a tile is all query, all key or all value.
//
// The same parameter block carries an optional deferred row scale (any epilogue): when
// row_ss is set, every accumulator row i is first multiplied by
//     s_i = 1 / sqrt(sum_p row_ss[i][p] * ss_inv_d + ss_eps),
// the RMSNorm factor of a pre-norm input whose per-column weight the producer already
// applied (x16 = bf16(h * w), row_ss = partial sums of h^2: linear_ln_tcgen05_pair's
// deferred form).  Null: no scaling.
struct RopeParams {
    const int32_t *pos;    // [M] position of each row's token in its sentence
    const float *qw, *kw;  // [hd] q_norm / k_norm weights
    int q_cols, k_end;
    int hd;                // 128 or 256
    int one_plus;          // Gemma3 weight form (1 + w)
    float eps, log2_theta;
    const float *row_ss;   // [M][ss_parts] partial sums of squares of the input rows, or null
    int ss_parts;
    float ss_inv_d, ss_eps;
};

// s_i of the deferred row scale (1 without one, and for rows past M)
__device__ __forceinline__ float deferred_row_scale(const RopeParams &rp, int row, int M)
{
    if (rp.row_ss == nullptr || row >= M) return 1.f;
    const float *p = rp.row_ss + static_cast<size_t>(row) * rp.ss_parts;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = i < rp.ss_parts ? __ldg(p + i) : 0.f;  // independent loads
    const float t = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    return 1.0f / sqrtf(t * rp.ss_inv_d + rp.ss_eps);
}

// The epilogue warps (threads 64 .. 64 + nthreads of the CTA) fill the CTA's table of
// inverse RoPE frequencies theta^(-2i / hd), i < hd / 2, then meet at named barrier 1.
__device__ __forceinline__ void fill_rope_table(float *inv_tab, const RopeParams &rp, int nthreads)
{
    const int et = static_cast<int>(threadIdx.x) - 64;
    for (int i = et; i < rp.hd / 2; i += nthreads)
        inv_tab[i] = exp2f(-rp.log2_theta * static_cast<float>(2 * i) / static_cast<float>(rp.hd));
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// One warp's 32 rows x BN columns of a query or key tile: for each head, pass 1 sums
// the squares of its HD accumulator columns (a thread owns a row, so no shuffles), pass 2
// reads each element with its rotation partner HD/2 columns away, normalises both, rotates
// them and stages them in the two 128-byte slabs (columns lo and lo + HD/2) that are
// TMA-stored together.  Leaves no store reading shared memory.
template <int BN, int HD>
__device__ __forceinline__ void drain_qk_rope(uint32_t t_row, int row, int store_row, int n0, int M,
                                              const RopeParams &rp, const float *inv_tab, const CUtensorMap *tm_y,
                                              uint8_t *bufs, int lane, float sc)
{
    static_assert(BN % HD == 0, "a tile holds whole heads");
    const float *wv = n0 < rp.q_cols ? rp.qw : rp.kw;
    const float wadd = rp.one_plus ? 1.f : 0.f;
    const float fpos = static_cast<float>(row < M ? __ldg(rp.pos + row) : 0);
    uint8_t *buf_lo = bufs, *buf_hi = bufs + kStageBufBytes;
#pragma unroll 1
    for (int h0 = 0; h0 < BN; h0 += HD) {
        float ss0 = 0.f, ss1 = 0.f;
#pragma unroll 1
        for (int c = 0; c < HD; c += 64) {  // two 32-column loads per wait
            uint32_t v[32], u[32];
            tmem_ld_x32(t_row + h0 + c, v);
            tmem_ld_x32(t_row + h0 + c + 32, u);
            tmem_wait_ld_regs(v);
            tmem_wait_ld_regs(u);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                ss0 = fmaf(__uint_as_float(v[j]), __uint_as_float(v[j]), ss0);
                ss1 = fmaf(__uint_as_float(u[j]), __uint_as_float(u[j]), ss1);
            }
        }
        const float ss = ss0 + ss1;
        // with a deferred row scale sc the head's values are sc * acc: norm factor of those, times sc
        const float r = sc * rsqrtf(sc * sc * ss / static_cast<float>(HD) + rp.eps);
#pragma unroll 1
        for (int sl = 0; sl < HD / 128; ++sl) {
            if (lane == 0) bulk_wait_read<0>();  // the slabs' previous stores have read shared memory
            __syncwarp();
            uint8_t *pa = buf_lo + lane * 128, *pb = buf_hi + lane * 128;
#pragma unroll 1
            for (int cc = 0; cc < 2; ++cc) {
                const int lo = 64 * sl + 32 * cc;  // head column of this chunk's first element
                uint32_t a[32], b[32];
                tmem_ld_x32(t_row + h0 + lo, a);
                tmem_ld_x32(t_row + h0 + lo + HD / 2, b);
                tmem_wait_ld_regs(a);
                tmem_wait_ld_regs(b);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    float sn, cs;
                    sincos_reduced(fpos * inv_tab[lo + j], sn, cs);
                    const float xa = __uint_as_float(a[j]) * r * (__ldg(wv + lo + j) + wadd);
                    const float xb = __uint_as_float(b[j]) * r * (__ldg(wv + lo + j + HD / 2) + wadd);
                    a[j] = __float_as_uint(xa * cs - xb * sn);
                    b[j] = __float_as_uint(xb * cs + xa * sn);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {  // 32 bf16 = 16-byte units 4 cc .. 4 cc + 3 of the slab row
                    const int c16 = 4 * cc + u;
                    uint4 wa, wb;
                    wa.x = pack_bf16x2(__uint_as_float(a[8 * u + 0]), __uint_as_float(a[8 * u + 1]));
                    wa.y = pack_bf16x2(__uint_as_float(a[8 * u + 2]), __uint_as_float(a[8 * u + 3]));
                    wa.z = pack_bf16x2(__uint_as_float(a[8 * u + 4]), __uint_as_float(a[8 * u + 5]));
                    wa.w = pack_bf16x2(__uint_as_float(a[8 * u + 6]), __uint_as_float(a[8 * u + 7]));
                    wb.x = pack_bf16x2(__uint_as_float(b[8 * u + 0]), __uint_as_float(b[8 * u + 1]));
                    wb.y = pack_bf16x2(__uint_as_float(b[8 * u + 2]), __uint_as_float(b[8 * u + 3]));
                    wb.z = pack_bf16x2(__uint_as_float(b[8 * u + 4]), __uint_as_float(b[8 * u + 5]));
                    wb.w = pack_bf16x2(__uint_as_float(b[8 * u + 6]), __uint_as_float(b[8 * u + 7]));
                    *reinterpret_cast<uint4 *>(pa + ((c16 ^ (lane & 7)) << 4)) = wa;
                    *reinterpret_cast<uint4 *>(pb + ((c16 ^ (lane & 7)) << 4)) = wb;
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(tm_y, buf_lo, n0 + h0 + 64 * sl, store_row);
                tma_store_2d(tm_y, buf_hi, n0 + h0 + 64 * sl + HD / 2, store_row);
                bulk_commit();
            }
        }
    }
    if (lane == 0) bulk_wait_read<0>();  // the caller's double-buffering assumes no store of these slabs pending
    __syncwarp();
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
                                                  const CUtensorMap *tm_y, uint8_t *bufs, int &pp, int lane,
                                                  const RopeParams &rp, const float *inv_tab, float sc)
{
    if constexpr (OUT_BF16) {
        if (epi == E_QKROPE) {
            // a warp drains whole heads: 128-column warps (the 8-warp pair kernel) take head_dim 128
            // only, and the launcher gives them no other
            if constexpr (BN >= 256) {
                if (n0 < rp.k_end) {
                    if (rp.hd == 128) drain_qk_rope<BN, 128>(t_row, row, store_row, n0, M, rp, inv_tab, tm_y, bufs, lane, sc);
                    else drain_qk_rope<BN, 256>(t_row, row, store_row, n0, M, rp, inv_tab, tm_y, bufs, lane, sc);
                    return;
                }
            } else if constexpr (BN == 128) {
                if (n0 < rp.k_end && rp.hd == 128) {
                    drain_qk_rope<BN, 128>(t_row, row, store_row, n0, M, rp, inv_tab, tm_y, bufs, lane, sc);
                    return;
                }
            }
            epi = E_NONE;  // value heads: stored as they are
        }
        if (epi == E_SWIGLU || epi == E_GEGLU) {
            // Gated MLP: W rows interleave 32 gate and 32 up rows, so each 64-column block of
            // the accumulator gives 32 outputs act(gate) * up; 128 accumulator columns fill one
            // 64-column bf16 slab of y, which has N / 2 columns.
#pragma unroll 1
            for (int c = 0; c < BN; c += 128) {
                float o[64];
#pragma unroll
                for (int hb = 0; hb < 2; ++hb) {
                    uint32_t g[32], u[32];
                    tmem_ld_x32(t_row + c + 64 * hb, g);
                    tmem_ld_x32(t_row + c + 64 * hb + 32, u);
                    tmem_wait_ld_regs(g);
                    tmem_wait_ld_regs(u);
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        float a0 = __uint_as_float(g[j]), a1 = __uint_as_float(g[j + 1]);
                        float b0 = __uint_as_float(u[j]), b1 = __uint_as_float(u[j + 1]);
                        if (rp.row_ss != nullptr) {  // warp-uniform: no cost without a row scale
                            mul_f32x2(a0, a1, sc, sc);
                            mul_f32x2(b0, b1, sc, sc);
                        }
                        if (epi == E_SWIGLU) silu_fast2(a0, a1);
                        else gelu_tanh_fast2(a0, a1);
                        mul_f32x2(a0, a1, b0, b1);
                        o[32 * hb + j] = a0;
                        o[32 * hb + j + 1] = a1;
                    }
                }
                uint8_t *buf = bufs + pp * kStageBufBytes;
                if (lane == 0) bulk_wait_read<1>();
                __syncwarp();
                uint8_t *rowp = buf + lane * 128;
#pragma unroll
                for (int c16 = 0; c16 < 8; ++c16) {
                    uint4 w;
                    w.x = pack_bf16x2(o[c16 * 8 + 0], o[c16 * 8 + 1]);
                    w.y = pack_bf16x2(o[c16 * 8 + 2], o[c16 * 8 + 3]);
                    w.z = pack_bf16x2(o[c16 * 8 + 4], o[c16 * 8 + 5]);
                    w.w = pack_bf16x2(o[c16 * 8 + 6], o[c16 * 8 + 7]);
                    *reinterpret_cast<uint4 *>(rowp + ((c16 ^ (lane & 7)) << 4)) = w;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(tm_y, buf, (n0 + c) / 2, store_row);
                    bulk_commit();
                }
                pp ^= 1;
            }
            return;
        }
    }
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
        if (rp.row_ss != nullptr) {  // warp-uniform: no cost without a row scale
#pragma unroll
            for (int j = 0; j < CHUNK; ++j) f[j] *= sc;
        }
        const int col0 = n0 + c;
        if (epi != E_NONE) {
            if (col0 + CHUNK <= N) {
#pragma unroll
                for (int j = 0; j < CHUNK; j += 4) {
                    const float4 bb = __ldg(reinterpret_cast<const float4 *>(bias + col0 + j));
                    add_f32x2(f[j], f[j + 1], bb.x, bb.y);
                    add_f32x2(f[j + 2], f[j + 3], bb.z, bb.w);
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
                        add_f32x2(f[j], f[j + 1], rr.x, rr.y);
                        add_f32x2(f[j + 2], f[j + 3], rr.z, rr.w);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < CHUNK; ++j)
                        if (col0 + j < N) f[j] += rp[j];
                }
            }
        } else if (epi == E_GELU) {
#pragma unroll
            for (int j = 0; j < CHUNK; j += 2) gelu_tanh_fast2(f[j], f[j + 1]);
        } else if (epi == E_SWISH) {
#pragma unroll
            for (int j = 0; j < CHUNK; j += 2) silu_fast2(f[j], f[j + 1]);
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
                   int *status, const RopeParams rp)
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
    float *inv_tab = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(full) + C::BAR_BYTES);

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
    grid_dep_wait();
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    grid_dep_launch();
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
                    if (!mbar_wait_drain(&full[s], (armed_parity >> s) & 1u)) report(status, DEV_TIMEOUT);
        }
    } else if (warp == 1) {
        {
            const bool leader = elect_lane();  // the whole warp waits; this lane issues
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
                        if (leader) umma_f16_ss(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    issued = true;
                    if (leader) umma_commit(&empty[stage]);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (*abort_flag) break;
                if (leader) umma_commit(&acc_full[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            if (*abort_flag && issued) {
                // Let outstanding MMAs retire before TMEM is released.
                uint64_t *probe = &acc_full[acc];
                if (leader) umma_commit(probe);
                if (!mbar_wait_drain(probe, acc_phase)) report(status, DEV_TIMEOUT);
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        if (epi == E_QKROPE) fill_rope_table(inv_tab, rp, 32 * kEpiWarps);
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        uint8_t *bufs = epi_buf + q * 2 * kStageBufBytes;
        int acc = 0;
        uint32_t acc_phase = 0;
        int pp = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            if (*abort_flag) break;
            const int m0 = (tile / n_tiles) * BM;
            const int n0 = (tile % n_tiles) * BN;
            const int row = m0 + q * 32 + lane;
            // the row's deferred RMSNorm factor: its loads overlap the wait for the accumulator
            const float sc = deferred_row_scale(rp, row, M);
            if (!mbar_wait(&acc_full[acc], acc_phase)) {
                report(status, DEV_TIMEOUT);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
            drain_accumulator<BN, OUT_BF16>(t_row, row, m0 + q * 32, n0, M, N, bias, residual, epi, &tm_y, bufs, pp,
                                            lane, rp, inv_tab, sc);
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
// Pair p owns tiles p, p + npairs, ...; tile t covers rows (t / n_tiles) * 256 and
// columns (t % n_tiles) * 256.
constexpr int P_BN = 256;
constexpr uint32_t P_HALF_BYTES = 128 * BK * 2;        // 16 KB: 128 rows x 64 bf16
constexpr uint32_t P_STAGE_BYTES = 2 * P_HALF_BYTES;   // this CTA's x rows + W rows
constexpr uint32_t P_TMEM_COLS = 2 * P_BN;

// Pair-kernel configuration: ring stages and epilogue warps (4, or 8 = two per TMEM
// lane quarter, each draining 128 of the 256 accumulator columns).
template <int STAGES, int EPI_WARPS>
struct PairCfg {
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int COLS = P_BN / (EPI_WARPS / 4);
    static constexpr uint32_t RING = STAGES * P_STAGE_BYTES;
    static constexpr uint32_t EPI = EPI_WARPS * 2 * kStageBufBytes;
    static constexpr uint32_t SMEM = 1024 + RING + EPI + 256 + kRopeTabBytes;
    static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "epilogue warps");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

// TMA producer of a pair (lane 0 of warp 0 in both CTAs).
template <int STAGES>
__device__ __forceinline__ void pair_producer(uint8_t *ring, uint64_t *full, uint64_t *empty, const CUtensorMap *tm_x,
                                              const CUtensorMap *tm_w, uint32_t rank, int pair, int npairs,
                                              int num_tiles, int n_tiles, int k_iters, volatile int *abort_flag,
                                              int *status)
{
    int stage = 0;
    uint32_t phase = 0;
    uint32_t armed = 0, armed_parity = 0;  // per stage: armed at least once / parity of the last arm
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
            tma_load_2d_pair(a_dst, tm_x, leader_full, kb * BK, m0 + static_cast<int>(rank) * 128);
            tma_load_2d_pair(b_dst, tm_w, leader_full, kb * BK, n0 + static_cast<int>(rank) * 128);
            armed |= 1u << stage;
            armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
            if (++stage == STAGES) {
                stage = 0;
                phase ^= 1;
            }
        }
    }
    // The leader's stage barriers count both CTAs' bytes: it drains the pair's loads.
    if (rank == 0)
        for (int s = 0; s < STAGES; ++s)
            if (armed & (1u << s))
                if (!mbar_wait_drain(&full[s], (armed_parity >> s) & 1u)) report(status, DEV_TIMEOUT);
}

// MMA issuer of a pair (warp 1 of the leader; its elected lane issues): 256 x 256 x 64 per stage
// into one of two TMEM accumulators.
template <int STAGES>
__device__ __forceinline__ void pair_mma(uint8_t *ring, uint64_t *full, uint64_t *empty, uint64_t *acc_full,
                                         uint64_t *acc_empty, uint32_t tmem_base, int pair, int npairs, int num_tiles,
                                         int k_iters, volatile int *abort_flag, int *status, bool leader)
{
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
                if (leader) umma_f16_ss_pair(d_tmem, ad + static_cast<uint64_t>(k * 2), bd + static_cast<uint64_t>(k * 2), idesc,
                                 (kb | k) != 0 ? 1u : 0u);
            issued = true;
            if (leader) umma_commit_pair_both(&empty[stage]);
            if (++stage == STAGES) {
                stage = 0;
                phase ^= 1;
            }
        }
        if (*abort_flag) break;
        if (leader) umma_commit_pair_both(&acc_full[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
    }
    if (*abort_flag && issued) {
        // Let outstanding MMAs retire before TMEM is released.
        uint64_t *probe = &acc_full[acc];
        if (leader) umma_commit_pair_both(probe);
        if (!mbar_wait_drain(probe, acc_phase)) report(status, DEV_TIMEOUT);
    }
}

template <bool OUT_BF16, int P_STAGES, int EPI_WARPS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairCfg<P_STAGES, EPI_WARPS>::THREADS, 1)
    linear_tcgen05_pair(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_y, int M, int N, int K,
                        const float *__restrict__ bias, const float *__restrict__ residual, int epi, int *status,
                        const RopeParams rp)
{
    using Cfg = PairCfg<P_STAGES, EPI_WARPS>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = smem;
    uint8_t *epi_buf = smem + Cfg::RING;
    uint64_t *full = reinterpret_cast<uint64_t *>(epi_buf + Cfg::EPI);  // used in the leader
    uint64_t *empty = full + P_STAGES;                                  // both CTAs
    uint64_t *acc_full = empty + P_STAGES;                              // both CTAs [2]
    uint64_t *acc_empty = acc_full + 2;                                    // used in the leader [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    float *inv_tab = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(full) + 256);

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
            mbar_init(&acc_empty[b], 2 * EPI_WARPS);  // one arrival per epilogue warp of either CTA
        }
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_w);
        tma_prefetch_desc(&tm_y);
    }
    grid_dep_wait();
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, P_TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
    tc_fence_after();
    grid_dep_launch();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0)
            pair_producer<P_STAGES>(ring, full, empty, &tm_x, &tm_w, rank, pair, npairs, num_tiles, n_tiles, k_iters,
                                    abort_flag, status);
    } else if (warp == 1) {
        if (rank == 0)  // the whole warp: waits on every lane, MMAs from the elected one
            pair_mma<P_STAGES>(ring, full, empty, acc_full, acc_empty, tmem_base, pair, npairs, num_tiles, k_iters,
                               abort_flag, status, elect_lane());
    } else {
        // ---------------- epilogue (warps 2.. of both CTAs): warp w drains TMEM lanes
        // 32 * (w % 4) (the lane-quarter rule), columns [h * COLS, (h + 1) * COLS), h = (w - 2) / 4
        constexpr int COLS = Cfg::COLS;
        if (epi == E_QKROPE) fill_rope_table(inv_tab, rp, 32 * EPI_WARPS);
        const int q = warp & 3;
        const int h = (warp - 2) >> 2;
        uint8_t *bufs = epi_buf + (warp - 2) * 2 * kStageBufBytes;
        const uint32_t leader_acc_empty[2] = {map_to_rank(&acc_empty[0], 0), map_to_rank(&acc_empty[1], 0)};
        int acc = 0;
        uint32_t acc_phase = 0;
        int pp = 0;
        for (int tile = pair; tile < num_tiles; tile += npairs) {
            if (*abort_flag) break;
            const int m0 = (tile / n_tiles) * 256 + static_cast<int>(rank) * 128;
            const int n0 = (tile % n_tiles) * P_BN + h * COLS;
            const int row = m0 + q * 32 + lane;
            // the row's deferred RMSNorm factor: its loads overlap the wait for the accumulator
            const float sc = deferred_row_scale(rp, row, M);
            if (!mbar_wait(&acc_full[acc], acc_phase)) {
                report(status, DEV_TIMEOUT);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * P_BN + h * COLS;
            drain_accumulator<COLS, OUT_BF16>(t_row, row, m0 + q * 32, n0, M, N, bias, residual, epi, &tm_y, bufs, pp,
                                              lane, rp, inv_tab, sc);
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

// ---------------------------------------------------------------------------
// Linear + residual + LayerNorm in one kernel:
//     h32 <- LayerNorm((x W^T + bias) + h32) * gamma + beta,   h16 <- bf16(h32)
// the out-projection / FFN-down step of a post-LN encoder layer (reference:
// src/sentence_transformers_impl.cpp:250-263 and :403-436, LayerNorm statistics as in
// src/ops/cpu/cpu_matrix_ops.cpp:64-92).  The mainloop is the pair kernel's.  A row of
// N = 256 * n_tiles columns spans n_tiles tiles, which run on different pairs at the
// same time, so LayerNorm statistics are exchanged through global memory:
//   pass 1   each epilogue warp forms x = (acc + bias) + residual for its 32 rows (the
//            residual arrives by TMA), writes x back into its TMEM accumulator and
//            computes each row's (mean, M2) over its columns: exact two-pass per
//            32-column chunk, chunks (all the same size) combined exactly;
//   exchange each row's partial goes to stats[row][part] as two 64-bit words holding the
//            value and the launch's epoch, so a reader that sees the epoch sees the value
//            (single-copy atomic 64-bit accesses): no counter, no fence.  The warp polls
//            its rows' other parts (bounded wait) and combines them in part order, so the
//            result does not depend on arrival order;
//   pass 2   x is read back from TMEM, normalised and TMA-stored as fp32 (in place over the
//            residual) and bf16.
// The waiting needs every pair of the launch resident at once and every row group's
// tiles in the same round: the launcher sizes the grid from the occupancy of this
// kernel, as a multiple of n_tiles, and orders launches of this kernel on a device one
// after another.
//
// Configurations: ring stages, epilogue warps (4 or 8; 8 = two per TMEM lane quarter,
// splitting the 256 columns) and 4 KB fp32 slabs per epilogue warp (plus one 2 KB bf16
// slab); shared memory is the binding limit.  The launcher uses this kernel for
// K >= 2048 only.  Every tile's accumulator stays in TMEM from the end of its mainloop
// until its row statistics have crossed between pairs (a few microseconds of L2 round
// trips), and with two accumulators the next-but-one mainloop waits for that.  A K = 4096
// mainloop (~25 us a tile) hides it; a K = 1024 one (~7 us) does not: measured on the
// bge-large out-projection, 102-138 us fused against 51 + 59 us for the pair kernel and
// the LayerNorm kernel, which the launcher uses there instead.
constexpr uint32_t L_BAR_BYTES = 512;
template <int STAGES, int EPI_WARPS, int SLABS>
struct LnCfg {
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int COLS = P_BN / (EPI_WARPS / 4);  // accumulator columns per epilogue warp
    static constexpr int CH = COLS / 32;                 // 32-column chunks per warp
    static constexpr uint32_t WARP_BYTES = SLABS * 4096 + 2048;
    static constexpr uint32_t RING = STAGES * P_STAGE_BYTES;
    static constexpr uint32_t EPI = EPI_WARPS * WARP_BYTES;
    static constexpr uint32_t VEC = 3 * P_BN * 4;  // bias, gamma, beta of the pair's 256 columns
    static constexpr uint32_t SMEM = 1024 + RING + EPI + VEC + L_BAR_BYTES;
    static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "epilogue warps");
    static_assert(SLABS == 1 || SLABS == 2, "fp32 slabs");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

struct LnParams {
    const float *bias;
    const float *gamma;
    const float *beta;
    unsigned long long *stats;  // [M][nparts][2]: (mean, M2) of each row over each warp's columns,
                                // each word = float bits << 32 | epoch
    unsigned epoch;             // nonzero, unique per launch on this workspace
    float eps;
    int nparts;                 // statistics partials per row = N / COLS
    int rms;                    // 0: LayerNorm, h32 <- the normalised rows (post-norm);
                                // 1: RMSNorm, h32 <- x itself, h16 <- x / rms(x) * gamma (pre-norm);
                                // 2: deferred RMSNorm, h32 <- x, h16 <- x * gamma, and the row's sum of
                                //    x^2 over each part into ((float *) stats)[row * nparts + part]:
                                //    the consumer applies 1 / rms(x) (no exchange, one pass)
};

__device__ __forceinline__ void st_relaxed_u64(unsigned long long *p, unsigned long long v)
{
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long tag(float v, unsigned epoch)
{
    return (static_cast<unsigned long long>(__float_as_uint(v)) << 32) | epoch;
}

// DEFER: the deferred RMSNorm form (LnParams::rms == 2), its own instantiation so that the
// LayerNorm / RMSNorm forms keep their code unchanged.
template <int STAGES, int EPI_WARPS, int SLABS, bool DEFER>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(LnCfg<STAGES, EPI_WARPS, SLABS>::THREADS, 1)
    linear_ln_tcgen05_pair(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                           const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ CUtensorMap tm_h16,
                           int M, int N, int K, LnParams p, int write16, int *status)
{
    using C = LnCfg<STAGES, EPI_WARPS, SLABS>;
    constexpr int COLS = C::COLS, CH = C::CH;
    // The epilogue's FP32 arithmetic as packed f32x2 instructions: measured 2-4 % faster
    // where the epilogue bounds the kernel (the 5-stage / 2-slab form below K = 4096) and
    // 2 % slower at K = 4096, where the mainloop does.
    constexpr bool PACKED = SLABS == 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = smem;
    uint8_t *epi_buf = smem + C::RING;
    float *vec = reinterpret_cast<float *>(epi_buf + C::EPI);  // [3][256]
    uint64_t *full = reinterpret_cast<uint64_t *>(epi_buf + C::EPI + C::VEC);
    uint64_t *empty = full + STAGES;
    uint64_t *acc_full = empty + STAGES;  // [2]
    uint64_t *acc_empty = acc_full + 2;   // [2]
    uint64_t *res_bar = acc_empty + 2;    // [EPI_WARPS][SLABS]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(res_bar + SLABS * EPI_WARPS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    static_assert((2 * STAGES + 4 + SLABS * EPI_WARPS) * 8 + 8 <= L_BAR_BYTES, "barrier space");

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1;
    const int npairs = gridDim.x >> 1;  // a multiple of n_tiles: every tile of this pair has the same columns
    const int m_tiles = (M + 255) / 256;
    const int n_tiles = N / P_BN;
    const int num_tiles = m_tiles * n_tiles;
    const int k_iters = (K + BK - 1) / BK;
    const int n0 = (pair % n_tiles) * P_BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 2 * EPI_WARPS);
        }
        for (int b = 0; b < SLABS * EPI_WARPS; ++b) mbar_init(&res_bar[b], 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_w);
        tma_prefetch_desc(&tm_h);
        if (write16) tma_prefetch_desc(&tm_h16);
    }
    grid_dep_wait();
    for (int i = threadIdx.x; i < 3 * P_BN; i += blockDim.x) {
        const float *src = i < P_BN ? p.bias : (i < 2 * P_BN ? p.gamma : p.beta);
        vec[i] = src[n0 + (i % P_BN)];
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, P_TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    grid_dep_launch();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0)
            pair_producer<STAGES>(ring, full, empty, &tm_x, &tm_w, rank, pair, npairs, num_tiles, n_tiles, k_iters,
                                  abort_flag, status);
    } else if (warp == 1) {
        if (rank == 0)  // the whole warp: waits on every lane, MMAs from the elected one
            pair_mma<STAGES>(ring, full, empty, acc_full, acc_empty, tmem_base, pair, npairs, num_tiles, k_iters,
                             abort_flag, status, elect_lane());
    } else {
        // ---------------- epilogue: warp w drains TMEM lanes 32 * (w % 4) (the lane-quarter
        // rule), accumulator columns [h * COLS, (h + 1) * COLS), h = (w - 2) / 4.
        // Staging per warp: SLABS 4 KB fp32 slabs (residual in pass 1, output in pass 2)
        // and one 2 KB bf16 output slab.
        const int ew = warp - 2;
        const int q = warp & 3;
        const int h = ew >> 2;
        const int c0 = n0 + h * COLS;  // first column of this warp
        uint8_t *wb = epi_buf + ew * C::WARP_BYTES;
        uint8_t *hs = wb + SLABS * 4096;
        uint64_t *rbar = res_bar + SLABS * ew;
        const float *vb = vec + h * COLS, *vg = vec + P_BN + h * COLS, *ve = vec + 2 * P_BN + h * COLS;
        const int part = c0 / COLS;
        const uint32_t leader_acc_empty[2] = {map_to_rank(&acc_empty[0], 0), map_to_rank(&acc_empty[1], 0)};
        uint32_t rpar = 0;      // bit b: parity of the next completion of rbar[b]
        uint32_t inflight = 0;  // bit b: a residual load into slab b has not been waited for
        int acc = 0;
        uint32_t acc_phase = 0;
        const float inv_n = 1.0f / static_cast<float>(N);
        auto warp_row0 = [&](int t) { return (t / n_tiles) * 256 + static_cast<int>(rank) * 128 + q * 32; };
        // The residual is read once and the outputs written once: evict-first in L2, so that
        // they do not displace the x row blocks the other column tiles of a row group read.
        const uint64_t stream_policy = l2_policy_evict_first();
        auto load_res = [&](int b, int col, int row) {  // lane 0
            mbar_arrive_expect_tx(&rbar[b], 4096);
            tma_load_2d_hint(wb + b * 4096, &tm_h, &rbar[b], col, row, stream_policy);
        };
        if (lane < CH && pair < num_tiles) tma_prefetch_l2_2d(&tm_h, c0 + 32 * lane, warp_row0(pair));
        for (int tile = pair; tile < num_tiles; tile += npairs) {
            if (*abort_flag) break;
            const int row0 = warp_row0(tile);
            const int row = row0 + lane;
            // (no L2 prefetch of the next tile's residual: issued a whole round ahead, the
            // lines were evicted before use and the residual crossed HBM twice)
            if (lane == 0) {
                bulk_wait_read<0>();  // the previous tile's stores have read every slab
                load_res(0, c0, row0);
            }
            inflight = 1;
            __syncwarp();
            if (!mbar_wait(&acc_full[acc], acc_phase)) {
                report(status, DEV_TIMEOUT);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * P_BN + h * COLS;

            if constexpr (DEFER) {
                // ---- deferred RMSNorm, one pass per 32-column chunk: x = (acc + bias) + residual,
                // its squares summed, x TMA-stored as fp32 from the residual's own slab and
                // bf16(x * gamma) from the bf16 slab.  Bulk groups per chunk c: F(c), then B(c).
                float ss4[4] = {0.f, 0.f, 0.f, 0.f};
                bool ok = true;
                uint32_t v[2][32];
                tmem_ld_x32(t_row, v[0]);
#pragma unroll
                for (int c = 0; c < CH; ++c) {
                    const int b = c % SLABS;
                    uint32_t(&cur)[32] = v[c & 1];
                    tmem_wait_ld_regs(cur);
                    if (c + 1 < CH) {
                        tmem_ld_x32(t_row + (c + 1) * 32, v[(c + 1) & 1]);
                        if (SLABS == 2) {  // the other slab held chunk c - 1's output: F(c - 1) has read it
                            if (lane == 0) {
                                if (c >= 1) bulk_wait_read<1>();
                                load_res((c + 1) % SLABS, c0 + 32 * (c + 1), row0);
                            }
                            inflight |= 1u << ((c + 1) % SLABS);
                        }
                    }
                    if (!mbar_wait(&rbar[b], (rpar >> b) & 1u)) {
                        ok = false;
                        break;
                    }
                    rpar ^= 1u << b;
                    inflight &= ~(1u << b);
                    uint8_t *fs = wb + b * 4096;
                    const uint8_t *rs = fs + lane * 128;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint4 r = *reinterpret_cast<const uint4 *>(rs + ((j ^ (lane & 7)) << 4));
                        const float4 bb = *reinterpret_cast<const float4 *>(vb + c * 32 + 4 * j);
                        float x0 = __uint_as_float(cur[4 * j + 0]), x1 = __uint_as_float(cur[4 * j + 1]);
                        float x2 = __uint_as_float(cur[4 * j + 2]), x3 = __uint_as_float(cur[4 * j + 3]);
                        add_f32x2(x0, x1, bb.x, bb.y);
                        add_f32x2(x2, x3, bb.z, bb.w);
                        add_f32x2(x0, x1, __uint_as_float(r.x), __uint_as_float(r.y));
                        add_f32x2(x2, x3, __uint_as_float(r.z), __uint_as_float(r.w));
                        fma_f32x2v(ss4[0], ss4[1], x0, x1, x0, x1, ss4[0], ss4[1]);
                        fma_f32x2v(ss4[2], ss4[3], x2, x3, x2, x3, ss4[2], ss4[3]);
                        cur[4 * j + 0] = __float_as_uint(x0);
                        cur[4 * j + 1] = __float_as_uint(x1);
                        cur[4 * j + 2] = __float_as_uint(x2);
                        cur[4 * j + 3] = __float_as_uint(x3);
                    }
                    __syncwarp();  // every lane has read the residual: the slab takes the fp32 output
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        *reinterpret_cast<uint4 *>(fs + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                            make_uint4(cur[4 * j + 0], cur[4 * j + 1], cur[4 * j + 2], cur[4 * j + 3]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d_hint(&tm_h, fs, c0 + c * 32, row0, stream_policy);
                        bulk_commit();
                    }
                    if (write16) {
                        if (lane == 0) bulk_wait_read<1>();  // B(c - 1) has read the bf16 slab
                        __syncwarp();
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float4 g0 = *reinterpret_cast<const float4 *>(vg + c * 32 + 8 * j);
                            const float4 g1 = *reinterpret_cast<const float4 *>(vg + c * 32 + 8 * j + 4);
                            const uint32_t *xv = cur + 8 * j;
                            *reinterpret_cast<uint4 *>(hs + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = make_uint4(
                                pack_bf16x2(__uint_as_float(xv[0]) * g0.x, __uint_as_float(xv[1]) * g0.y),
                                pack_bf16x2(__uint_as_float(xv[2]) * g0.z, __uint_as_float(xv[3]) * g0.w),
                                pack_bf16x2(__uint_as_float(xv[4]) * g1.x, __uint_as_float(xv[5]) * g1.y),
                                pack_bf16x2(__uint_as_float(xv[6]) * g1.z, __uint_as_float(xv[7]) * g1.w));  // 64B swizzle
                        }
                        fence_proxy_async_smem();
                        __syncwarp();
                    }
                    if (lane == 0) {  // an empty group keeps the F / B alternation when bf16 is not written
                        if (write16) tma_store_2d_hint(&tm_h16, hs, c0 + c * 32, row0, stream_policy);
                        bulk_commit();
                    }
                    if (SLABS == 1 && c + 1 < CH) {  // the only slab held chunk c's output: F(c) has read it
                        if (lane == 0) {
                            bulk_wait_read<1>();
                            load_res(0, c0 + 32 * (c + 1), row0);
                        }
                        inflight |= 1u;
                    }
                }
                tmem_wait_ld();
                if (!ok) {
                    report(status, DEV_TIMEOUT);
                    *abort_flag = 1;
                    break;
                }
                if (row < M)
                    reinterpret_cast<float *>(p.stats)[static_cast<size_t>(row) * p.nparts + part] =
                        (ss4[0] + ss4[1]) + (ss4[2] + ss4[3]);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(leader_acc_empty[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
                continue;
            }

            // ---- pass 1: x = (acc + bias) + residual back into TMEM; per-chunk mean / M2
            float cm[CH], cq_sum = 0.f;
            bool ok = true;
            uint32_t v[2][32];
            tmem_ld_x32(t_row, v[0]);
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const int b = c % SLABS;
                uint32_t(&cur)[32] = v[c & 1];
                tmem_wait_ld_regs(cur);
                if (c + 1 < CH) {
                    if (c >= 1) tmem_wait_st();  // v[(c + 1) & 1] was the source of the previous store
                    tmem_ld_x32(t_row + (c + 1) * 32, v[(c + 1) & 1]);
                    if (SLABS == 2) {  // the other slab was consumed by chunk c - 1
                        if (lane == 0) load_res((c + 1) % SLABS, c0 + 32 * (c + 1), row0);
                        inflight |= 1u << ((c + 1) % SLABS);
                    }
                }
                if (!mbar_wait(&rbar[b], (rpar >> b) & 1u)) {
                    ok = false;
                    break;
                }
                rpar ^= 1u << b;
                inflight &= ~(1u << b);
                const uint8_t *rs = wb + b * 4096 + lane * 128;
                float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint4 r = *reinterpret_cast<const uint4 *>(rs + ((j ^ (lane & 7)) << 4));
                    const float4 bb = *reinterpret_cast<const float4 *>(vb + c * 32 + 4 * j);
                    // x = (acc + bias) + residual and the running sums
                    float x0 = __uint_as_float(cur[4 * j + 0]), x1 = __uint_as_float(cur[4 * j + 1]);
                    float x2 = __uint_as_float(cur[4 * j + 2]), x3 = __uint_as_float(cur[4 * j + 3]);
                    if constexpr (PACKED) {
                        add_f32x2(x0, x1, bb.x, bb.y);
                        add_f32x2(x2, x3, bb.z, bb.w);
                        add_f32x2(x0, x1, __uint_as_float(r.x), __uint_as_float(r.y));
                        add_f32x2(x2, x3, __uint_as_float(r.z), __uint_as_float(r.w));
                        add_f32x2(s4[0], s4[1], x0, x1);
                        add_f32x2(s4[2], s4[3], x2, x3);
                    } else {
                        x0 = (x0 + bb.x) + __uint_as_float(r.x);
                        x1 = (x1 + bb.y) + __uint_as_float(r.y);
                        x2 = (x2 + bb.z) + __uint_as_float(r.z);
                        x3 = (x3 + bb.w) + __uint_as_float(r.w);
                        s4[0] += x0;
                        s4[1] += x1;
                        s4[2] += x2;
                        s4[3] += x3;
                    }
                    cur[4 * j + 0] = __float_as_uint(x0);
                    cur[4 * j + 1] = __float_as_uint(x1);
                    cur[4 * j + 2] = __float_as_uint(x2);
                    cur[4 * j + 3] = __float_as_uint(x3);
                }
                __syncwarp();  // every lane has read slab b
                if (SLABS == 1 && c + 1 < CH) {
                    if (lane == 0) load_res(0, c0 + 32 * (c + 1), row0);
                    inflight |= 1u;
                }
                cm[c] = ((s4[0] + s4[1]) + (s4[2] + s4[3])) * (1.0f / 32.0f);
                float q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    float d0 = __uint_as_float(cur[j]), d1 = __uint_as_float(cur[j + 1]);
                    if constexpr (PACKED) {
                        add_f32x2(d0, d1, -cm[c], -cm[c]);
                        fma_f32x2v(q4[j & 3], q4[(j & 3) + 1], d0, d1, d0, d1, q4[j & 3], q4[(j & 3) + 1]);
                    } else {
                        d0 -= cm[c];
                        d1 -= cm[c];
                        q4[j & 3] += d0 * d0;
                        q4[(j & 3) + 1] += d1 * d1;
                    }
                }
                cq_sum += (q4[0] + q4[1]) + (q4[2] + q4[3]);
                tmem_st_x32(t_row + c * 32, cur);
            }
            tmem_wait_ld();
            tmem_wait_st();
            if (!ok) {
                report(status, DEV_TIMEOUT);
                *abort_flag = 1;
                break;
            }
            // this warp's (mean, M2) over its COLS columns: equal-size chunks combined exactly
            float mean = 0.f;
#pragma unroll
            for (int c = 0; c < CH; ++c) mean += cm[c];
            mean *= 1.0f / CH;
            float m2 = 0.f;
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const float d = cm[c] - mean;
                m2 += d * d;
            }
            m2 = cq_sum + 32.0f * m2;

            // ---- publish, then collect the row's other parts (data and epoch in one
            // 64-bit word each: no fences, no counters)
            unsigned long long *sp = p.stats + (static_cast<size_t>(row) * p.nparts) * 2;
            if (row < M) {
                st_relaxed_u64(sp + 2 * part, tag(mean, p.epoch));
                st_relaxed_u64(sp + 2 * part + 1, tag(m2, p.epoch));
            }
            // The parts' means are accumulated about the first one (shifted sums), so that
            // no per-part value has to stay live: gm = K + S1 / P,
            // M2 = sum(M2_i) + COLS * (S2 - S1^2 / P).
            constexpr int kMaxParts = 2048 / COLS;  // rows of up to 2048 columns
            float pk = 0.f, ps1 = 0.f, ps2 = 0.f, pq_sum = 0.f;
            bool ready = row >= M;
            const uint64_t t0 = globaltimer_ns();
            for (uint32_t it = 0;; ++it) {
                if (!ready) {
                    const unsigned long long a0 = ld_relaxed_u64(sp);
                    bool all = static_cast<unsigned>(a0) == p.epoch;
                    const float k0 = __uint_as_float(static_cast<unsigned>(a0 >> 32));
                    float s1 = 0.f, s2 = 0.f, qs = 0.f;
#pragma unroll
                    for (int i = 0; i < kMaxParts; ++i)
                        if (i < p.nparts) {
                            const unsigned long long a = i == 0 ? a0 : ld_relaxed_u64(sp + 2 * i);
                            const unsigned long long bq = ld_relaxed_u64(sp + 2 * i + 1);
                            all = all && static_cast<unsigned>(a) == p.epoch && static_cast<unsigned>(bq) == p.epoch;
                            const float d = __uint_as_float(static_cast<unsigned>(a >> 32)) - k0;
                            s1 += d;
                            s2 += d * d;
                            qs += __uint_as_float(static_cast<unsigned>(bq >> 32));
                        }
                    ready = all;
                    pk = k0;
                    ps1 = s1;
                    ps2 = s2;
                    pq_sum = qs;
                }
                if (__all_sync(0xffffffffu, ready)) break;
                const bool stop = (it & 15u) == 15u && (*abort_flag || globaltimer_ns() - t0 > wait_limit_ns());
                if (__any_sync(0xffffffffu, stop)) {  // the same decision in every lane
                    ok = false;
                    break;
                }
            }
            if (!ok) {
                report(status, DEV_TIMEOUT);
                *abort_flag = 1;
                break;
            }
            float gm = 0.f, gq = 0.f;
            if (row < M) {
                const float inv_p = 1.0f / static_cast<float>(p.nparts);
                gm = pk + ps1 * inv_p;
                gq = pq_sum + static_cast<float>(COLS) * fmaxf(ps2 - ps1 * ps1 * inv_p, 0.f);
            }
            // LayerNorm: 1 / sqrt(var + eps); RMSNorm: 1 / sqrt(mean(x^2) + eps), mean(x^2) = var + mean^2
            const float inv_sd = 1.0f / sqrtf(gq * inv_n + (p.rms ? gm * gm : 0.f) + p.eps);

            // ---- pass 2: normalise from TMEM, TMA-store fp32 and bf16.  Bulk groups per
            // chunk c: F(c) (fp32 slab c % SLABS), then B(c) (the bf16 slab).
            tmem_ld_x32(t_row, v[0]);
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const int b = c % SLABS;
                uint32_t(&cur)[32] = v[c & 1];
                tmem_wait_ld_regs(cur);
                if (c + 1 < CH) tmem_ld_x32(t_row + (c + 1) * 32, v[(c + 1) & 1]);
                float o[32];
                const float sub = p.rms ? 0.f : gm;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 g = *reinterpret_cast<const float4 *>(vg + c * 32 + 4 * j);
                    float4 e = *reinterpret_cast<const float4 *>(ve + c * 32 + 4 * j);
                    if (p.rms) e = make_float4(0.f, 0.f, 0.f, 0.f);
                    // o = ((x - sub) * inv_sd) * g + e
                    float t0 = __uint_as_float(cur[4 * j + 0]), t1 = __uint_as_float(cur[4 * j + 1]);
                    float t2 = __uint_as_float(cur[4 * j + 2]), t3 = __uint_as_float(cur[4 * j + 3]);
                    if constexpr (PACKED) {
                        add_f32x2(t0, t1, -sub, -sub);
                        add_f32x2(t2, t3, -sub, -sub);
                        mul_f32x2(t0, t1, inv_sd, inv_sd);
                        mul_f32x2(t2, t3, inv_sd, inv_sd);
                        fma_f32x2v(o[4 * j + 0], o[4 * j + 1], t0, t1, g.x, g.y, e.x, e.y);
                        fma_f32x2v(o[4 * j + 2], o[4 * j + 3], t2, t3, g.z, g.w, e.z, e.w);
                    } else {
                        o[4 * j + 0] = (t0 - sub) * inv_sd * g.x + e.x;
                        o[4 * j + 1] = (t1 - sub) * inv_sd * g.y + e.y;
                        o[4 * j + 2] = (t2 - sub) * inv_sd * g.z + e.z;
                        o[4 * j + 3] = (t3 - sub) * inv_sd * g.w + e.w;
                    }
                }
                // F(c - SLABS) has read slab b: at most 2 * SLABS - 1 newer groups pending
                if (lane == 0) bulk_wait_read<2 * SLABS - 1>();
                __syncwarp();
                uint8_t *fs = wb + b * 4096;
#pragma unroll
                for (int j = 0; j < 8; ++j)  // 128B swizzle; pre-norm keeps x itself in the fp32 stream
                    *reinterpret_cast<uint4 *>(fs + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                        p.rms ? make_uint4(cur[4 * j + 0], cur[4 * j + 1], cur[4 * j + 2], cur[4 * j + 3])
                              : make_uint4(__float_as_uint(o[4 * j + 0]), __float_as_uint(o[4 * j + 1]),
                                           __float_as_uint(o[4 * j + 2]), __float_as_uint(o[4 * j + 3]));
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d_hint(&tm_h, fs, c0 + c * 32, row0, stream_policy);
                    bulk_commit();
                }
                if (write16) {
                    if (lane == 0) bulk_wait_read<1>();  // B(c - 1) has read the bf16 slab
                    __syncwarp();
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        *reinterpret_cast<uint4 *>(hs + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
                            make_uint4(pack_bf16x2(o[8 * j + 0], o[8 * j + 1]), pack_bf16x2(o[8 * j + 2], o[8 * j + 3]),
                                       pack_bf16x2(o[8 * j + 4], o[8 * j + 5]),
                                       pack_bf16x2(o[8 * j + 6], o[8 * j + 7]));  // 64B swizzle
                    fence_proxy_async_smem();
                    __syncwarp();
                }
                if (lane == 0) {  // an empty group keeps the F / B alternation when bf16 is not written
                    if (write16) tma_store_2d_hint(&tm_h16, hs, c0 + c * 32, row0, stream_policy);
                    bulk_commit();
                }
            }
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(leader_acc_empty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
        // Residual loads still in flight (abandoned tiles) must land before the CTA exits.
        if (lane == 0) {
            for (int b = 0; b < SLABS; ++b)
                if (inflight & (1u << b))
                    if (!mbar_wait_drain(&rbar[b], (rpar >> b) & 1u)) report(status, DEV_TIMEOUT);
            bulk_wait_all<0>();
        }
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, P_TMEM_COLS);
    }
}

// Ring stages x epilogue warps of the pair kernel, by epilogue.  With bias only (or none), 6 x 4:
// on the bge-large projections (K = 1024) 5 x 8 measured 2-3 % slower, the deeper ring mattering
// more.  The GELU and gated (SwiGLU / GeGLU) drains cost more arithmetic per element, and with
// 5 x 8 (two warps per TMEM lane quarter, 128 columns each) FFN1 + GELU went 163.7 -> 158.6 us
// and the N = 3072 GELU shape 128.8 -> 123.2 us.  The q/k norm + RoPE drain needs a whole head
// per warp: head_dim 128 takes the 8-warp form (Qwen3 QKV 472.6 -> 468.4 us), head_dim 256
// stays on four warps.
template <bool OUT_BF16, int STAGES, int EPI_WARPS>
cudaError_t launch_pair_cfg(const CUtensorMap &tx, const CUtensorMap &tw, const CUtensorMap &ty, int M, int N, int K,
                            const float *bias, const float *residual, int epi, int *status, cudaStream_t s,
                            const RopeParams &rp)
{
    using Cfg = PairCfg<STAGES, EPI_WARPS>;
    auto kern = linear_tcgen05_pair<OUT_BF16, STAGES, EPI_WARPS>;
    static uint64_t configured[64] = {};  // context the attribute was set in
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t ctx = current_context_id();
    if (dev < 64 && configured[dev] != ctx) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
        if (e != cudaSuccess) return e;
        configured[dev] = ctx;
    }
    const int tiles = ((M + 255) / 256) * ((N + P_BN - 1) / P_BN);
    int pairs = current_sm_count() / 2;
    if (pairs > tiles) pairs = tiles;
    if (pairs < 1) pairs = 1;
    return launch_k(kern, dim3(2 * pairs), dim3(Cfg::THREADS), Cfg::SMEM, s, tx, tw, ty, M, N, K, bias, residual,
                    epi, status, rp);
}

template <bool OUT_BF16>
cudaError_t launch_pair(const CUtensorMap &tx, const CUtensorMap &tw, const CUtensorMap &ty, int M, int N, int K,
                        const float *bias, const float *residual, int epi, int *status, cudaStream_t s,
                        const RopeParams &rp)
{
    if (epi == E_GELU || epi == E_SWIGLU || epi == E_GEGLU || (epi == E_QKROPE && rp.hd == 128))
        return launch_pair_cfg<OUT_BF16, 5, 8>(tx, tw, ty, M, N, K, bias, residual, epi, status, s, rp);
    return launch_pair_cfg<OUT_BF16, 6, 4>(tx, tw, ty, M, N, K, bias, residual, epi, status, s, rp);
}

// Pairs of linear_ln_tcgen05_pair<Cfg> that can be resident at once on the current
// device (0 if unknown).
template <class Cfg, int STAGES, int EPI_WARPS, int SLABS, bool DEFER>
int ln_resident_pairs()
{
    static int cached[64] = {};
    static uint64_t cached_ctx[64] = {};  // context the attribute was set in
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t ctx = current_context_id();
    if (dev < 64 && cached[dev] > 0 && cached_ctx[dev] == ctx) return cached[dev];
    auto kern = linear_ln_tcgen05_pair<STAGES, EPI_WARPS, SLABS, DEFER>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) != cudaSuccess) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (dev < 64) {
        cached[dev] = clusters;
        cached_ctx[dev] = ctx;
    }
    return clusters;
}

template <int BN, bool OUT_BF16>
cudaError_t launch(const CUtensorMap &tx, const CUtensorMap &tw, const CUtensorMap &ty, int M, int N,
                   int K, const float *bias, const float *residual, int epi, int *status,
                   cudaStream_t s, const RopeParams &rp)
{
    using C = Cfg<BN>;
    static uint64_t configured[64] = {};  // context the attribute was set in
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t ctx = current_context_id();
    if (dev < 64 && configured[dev] != ctx) {
        cudaError_t e = cudaFuncSetAttribute(linear_tcgen05<BN, OUT_BF16>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured[dev] = ctx;
    }
    const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    int grid = current_sm_count();
    if (grid > tiles) grid = tiles;
    if (grid < 1) grid = 1;
    return launch_k(linear_tcgen05<BN, OUT_BF16>, dim3(grid), dim3(kThreads), C::SMEM_BYTES, s, tx, tw, ty, M, N, K,
                    bias, residual, epi, status, rp);
}

// The 2-CTA kernel is the default for large M; FE_LINEAR_PAIR=0 selects the 1-CTA
// kernel for every shape (both compute the same result; tests run both).
bool pair_mode_enabled()
{
    const char *v = getenv("FE_LINEAR_PAIR");
    return !(v && v[0] == '0');
}

// FE_LINEAR_NORM_FUSE=0 takes the two-launch form of linear + residual + norm for every
// shape (same result; used to compare the two forms on a workload).
bool norm_fuse_enabled()
{
    const char *v = getenv("FE_LINEAR_NORM_FUSE");
    return !(v && v[0] == '0');
}

}  // namespace

namespace {
cudaError_t launch_linear_any(const void *x, const void *w, const float *bias, const float *residual, void *y,
                              int64_t m, int64_t n, int64_t k, int epilogue, int y_dtype, cudaStream_t s, fe_status *st,
                              const RopeParams &rp)
{
    *st = FE_OK;
    if (m == 0 || n == 0) return cudaSuccess;
    const int BN = (n % 256 == 0 || n > 1024) ? 256 : 128;
    // 256-row pair tiles once there are at least two of them per 256 columns
    const bool use_pair = pair_mode_enabled() && BN == 256 && m >= 512;
    const bool out_bf16 = y_dtype == FE_DTYPE_BF16;
    const bool glu = epilogue == E_SWIGLU || epilogue == E_GEGLU;
    const int64_t ny = glu ? n / 2 : n;  // y columns
    CUtensorMap tx, tw, ty;
    fe_status r = make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m, k, k, BM, BK);
    if (r == FE_OK) r = make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, n, k, k, BN, BK);
    if (r == FE_OK)
        r = out_bf16 ? make_tmap_2d(&ty, y, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m, ny, ny, 32, 64)
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
        return out_bf16 ? launch_pair<true>(tx, tw2, ty, M, N, K, bias, residual, epilogue, status, s, rp)
                        : launch_pair<false>(tx, tw2, ty, M, N, K, bias, residual, epilogue, status, s, rp);
    }
    if (BN == 256)
        return out_bf16 ? launch<256, true>(tx, tw, ty, M, N, K, bias, residual, epilogue, status, s, rp)
                        : launch<256, false>(tx, tw, ty, M, N, K, bias, residual, epilogue, status, s, rp);
    return out_bf16 ? launch<128, true>(tx, tw, ty, M, N, K, bias, residual, epilogue, status, s, rp)
                    : launch<128, false>(tx, tw, ty, M, N, K, bias, residual, epilogue, status, s, rp);
}
}  // namespace

cudaError_t launch_linear_bf16(const void *x, const void *w, const float *bias, const float *residual, void *y,
                               int64_t m, int64_t n, int64_t k, int epilogue, int y_dtype, cudaStream_t s, fe_status *st,
                               const float *row_ss, int ss_parts, float ss_eps)
{
    RopeParams rp{};
    rp.row_ss = row_ss;
    rp.ss_parts = ss_parts;
    rp.ss_inv_d = 1.0f / static_cast<float>(k);
    rp.ss_eps = ss_eps;
    return launch_linear_any(x, w, bias, residual, y, m, n, k, epilogue, y_dtype, s, st, rp);
}

cudaError_t launch_linear_qk_norm_rope(const void *x, const void *w, void *y, int64_t m, int64_t k, int q_heads,
                                       int kv_heads, int head_dim, const float *q_w, const float *k_w,
                                       const int32_t *pos, bool one_plus, float eps, float theta, cudaStream_t s,
                                       fe_status *st, const float *row_ss, int ss_parts)
{
    RopeParams rp{};
    rp.row_ss = row_ss;
    rp.ss_parts = ss_parts;
    rp.ss_inv_d = 1.0f / static_cast<float>(k);
    rp.ss_eps = eps;
    rp.pos = pos;
    rp.qw = q_w;
    rp.kw = k_w;
    rp.q_cols = q_heads * head_dim;
    rp.k_end = (q_heads + kv_heads) * head_dim;
    rp.hd = head_dim;
    rp.one_plus = one_plus ? 1 : 0;
    rp.eps = eps;
    rp.log2_theta = log2f(theta);
    const int64_t n = static_cast<int64_t>(q_heads + 2 * kv_heads) * head_dim;
    return launch_linear_any(x, w, nullptr, nullptr, y, m, n, k, E_QKROPE, FE_DTYPE_BF16, s, st, rp);
}

}  // namespace fe

namespace fe {
namespace {

constexpr int kMaxLnParts = 8;  // rows of up to 2048 columns

size_t round_up_256(size_t v) { return (v + 255) & ~size_t(255); }

// Launches of linear_ln_tcgen05_pair on one device run one after another, whatever
// their streams: a launch waits for the previous one's completion event.  Two such
// launches running at once could each hold SMs that the other's waiting pairs need.
std::mutex g_ln_mu;
cudaEvent_t g_ln_last[64] = {};
cudaStream_t g_ln_last_stream[64] = {};  // stream of that launch: no wait needed on the same stream
uint64_t g_ln_last_ctx[64] = {};          // context the event was created in
// Next epoch of each statistics workspace (keyed by its address); 0 is never used, so
// a zero-filled workspace holds no valid partial.
std::unordered_map<const void *, unsigned> g_ln_epoch;

}  // namespace

// Workspace layout: [stats: two 64-bit words per row and 128-column part]
// [fp32 [m, n] scratch of the unfused form].
size_t linear_layernorm_stats_bytes(int64_t m, int64_t n)
{
    return round_up_256(static_cast<size_t>(m) * static_cast<size_t>((n + 127) / 128) * 16);
}

size_t linear_layernorm_workspace_bytes(int64_t m, int64_t n)
{
    return linear_layernorm_stats_bytes(m, n) + static_cast<size_t>(m) * static_cast<size_t>(n) * 4;
}

void linear_layernorm_split_workspace(void *ws, int64_t m, int64_t n, void **stats, float **y)
{
    *stats = ws;
    *y = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + linear_layernorm_stats_bytes(m, n));
}

namespace {
using LnKernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, int, int, int,
                          LnParams, int, int *);
struct LnVariant {
    int (*resident)();
    int cols, threads;
    uint32_t smem;
    LnKernel kern;
};
template <int S, int E, int L, bool DEFER = false>
LnVariant ln_variant()
{
    using Cf = LnCfg<S, E, L>;
    return {&ln_resident_pairs<Cf, S, E, L, DEFER>, Cf::COLS, Cf::THREADS, Cf::SMEM,
            &linear_ln_tcgen05_pair<S, E, L, DEFER>};
}
// Ring depth against residual double-buffering (shared memory holds one or the other):
// measured per launch at n = 1024 on one B200,
//   k = 4096, m = 26508 (LayerNorm):  6 stages / 1 slab 216 us, 5 stages / 2 slabs 221 us;
//   k = 3072, m = 71550 (RMSNorm):    468 us and 427 us;  k = 2048: 378 us and 344 us.
// Eight epilogue warps were slower in every case (252-545 us).
LnVariant pick_ln_variant(int64_t k, bool defer = false)
{
    if (defer) return k >= 4096 ? ln_variant<6, 4, 1, true>() : ln_variant<5, 4, 2, true>();
    return k >= 4096 ? ln_variant<6, 4, 1>() : ln_variant<5, 4, 2>();
}
}  // namespace

namespace {
// ---------------------------------------------------------------------------
// Linear + residual + LayerNorm for rows of up to 1024 columns, one cluster per row block:
//     h32 <- LayerNorm((x W^T + bias) + h32) * gamma + beta,   h16 <- bf16(h32)
// the out-projection step of a post-LN encoder layer (reference:
// src/sentence_transformers_impl.cpp:250-266).  A cluster of R = N / 256 CTAs (one per SM)
// owns a 128-row block; CTA r computes columns [256 r, 256 r + 256) with 1-CTA tcgen05
// MMAs into one of two 256-column TMEM accumulators, so one row block's epilogue overlaps
// the next one's mainloop.  Each epilogue thread owns a row: it forms x = acc + bias +
// residual in TMEM with per-32-column exact two-pass statistics, sends its (mean, M2)
// over 256 columns to every CTA of the cluster through distributed shared memory
// (st.shared::cluster + a remote mbarrier arrive, release / acquire at cluster scope),
// combines the R parts in rank order (so every CTA and every run gets the same bits),
// then normalises from TMEM and TMA-stores fp32 and bf16.  Unlike the pair kernel's
// global-memory exchange, the statistics never leave the GPC, and the cluster is
// co-scheduled by the hardware, so no grid-residency assumption is made.
constexpr int LC_STAGES = 3;
constexpr int LC_BN = 256;
constexpr int LC_MAX_R = 4;                       // rows of up to 1024 columns
constexpr uint32_t LC_STAGE = BM * BK * 2 + LC_BN * BK * 2;  // x tile + W tile, 48 KB
constexpr uint32_t LC_FSLAB = 32 * 32 * 4;        // one warp's fp32 32 x 32 slab: residual in, output out
constexpr uint32_t LC_BSLAB = 32 * 32 * 2;        // its bf16 32 x 32 output slab
constexpr int LC_RSLABS = 3;                      // fp32 slabs per warp (residual chunks in flight)
constexpr uint32_t LC_WARP = LC_RSLABS * LC_FSLAB + 2 * LC_BSLAB;
constexpr uint32_t LC_EPI = kEpiWarps * LC_WARP;
constexpr uint32_t LC_STATS = 2 * LC_MAX_R * BM * 8;                 // [tile parity][rank][row] (mean, M2)
constexpr uint32_t LC_VEC = 3 * LC_BN * 4;                           // bias, gamma, beta of this CTA's columns
constexpr uint32_t LC_BAR = 256;
constexpr uint32_t LC_SMEM = 1024 + LC_STAGES * LC_STAGE + LC_EPI + LC_STATS + LC_VEC + LC_BAR;
static_assert(LC_SMEM <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait with cluster-scope acquire: the peers' distributed-shared-memory writes
// made before their release arrives are visible after it.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity)
{
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t limit = wait_limit_ns();
    const bool every = limit < kShortWaitNs;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if (((i & 255u) == 0 || every) && globaltimer_ns() - t0 > limit) return false;
    }
}

// Asynchronous store of (a, b) into the shared memory of a CTA of the cluster (shared::cluster
// address `addr`); its 8 bytes count as completed transaction bytes on that CTA's mbarrier at
// `bar` (shared::cluster address), so the receiver's phase completes once every expected byte
// has landed, with no fence on the sending side.
__device__ __forceinline__ void st_async_v2(uint32_t addr, float a, float b, uint32_t bar)
{
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(addr),
                 "f"(a), "f"(b), "r"(bar)
                 : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    linear_ln_cluster(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                      const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ CUtensorMap tm_h16, int M,
                      int N, int K, const float *__restrict__ bias, const float *__restrict__ gamma,
                      const float *__restrict__ beta, float *h32, float eps, int write16, int *status)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = smem;
    uint8_t *epi_buf = ring + LC_STAGES * LC_STAGE;      // per warp: 2 x (fp32 slab, bf16 slab)
    float2 *stats = reinterpret_cast<float2 *>(epi_buf + LC_EPI);  // [2][LC_MAX_R][BM]
    float *vb = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(stats) + LC_STATS);
    float *vg = vb + LC_BN, *ve = vg + LC_BN;
    uint64_t *full = reinterpret_cast<uint64_t *>(ve + LC_BN);
    uint64_t *empty = full + LC_STAGES;
    uint64_t *acc_full = empty + LC_STAGES;  // [2]
    uint64_t *acc_empty = acc_full + 2;      // [2]
    uint64_t *stat_bar = acc_empty + 2;      // [2] by row-block parity: the cluster's statistics landed
    uint64_t *rbar_all = stat_bar + 2;       // [kEpiWarps][LC_RSLABS] residual slab landed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(rbar_all + kEpiWarps * LC_RSLABS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int R = N / LC_BN;                         // CTAs per cluster (the cluster dimension)
    const uint32_t rank = cluster_ctarank();
    const int cluster = static_cast<int>(blockIdx.x) / R;
    const int nclusters = static_cast<int>(gridDim.x) / R;
    const int m_tiles = (M + BM - 1) / BM;
    const int k_iters = (K + BK - 1) / BK;
    const int n0 = static_cast<int>(rank) * LC_BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < LC_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 32 * kEpiWarps);
            mbar_init(&stat_bar[b], 1);  // armed by this CTA with the bytes the cluster sends it
        }
        for (int i = 0; i < kEpiWarps * LC_RSLABS; ++i) mbar_init(&rbar_all[i], 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_w);
        tma_prefetch_desc(&tm_h);
        tma_prefetch_desc(&tm_h16);
    }
    grid_dep_wait();
    for (int i = threadIdx.x; i < LC_BN; i += blockDim.x) {
        vb[i] = bias[n0 + i];
        vg[i] = gamma[n0 + i];
        ve[i] = beta[n0 + i];
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * LC_BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // every CTA's barriers exist before any remote arrive
    tc_fence_after();
    grid_dep_launch();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer: x rows of the row block, W rows n0 .. n0 + 255
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0, armed_parity = 0;
            for (int t = cluster; t < m_tiles && !*abort_flag; t += nclusters) {
                const int m0 = t * BM;
                for (int kb = 0; kb < k_iters; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1)) {
                        report(status, DEV_TIMEOUT);
                        *abort_flag = 1;
                        break;
                    }
                    uint8_t *a_dst = ring + stage * LC_STAGE;
                    uint8_t *b_dst = a_dst + BM * BK * 2;
                    mbar_arrive_expect_tx(&full[stage], LC_STAGE);
                    tma_load_2d(a_dst, &tm_x, &full[stage], kb * BK, m0);
                    tma_load_2d(b_dst, &tm_w, &full[stage], kb * BK, n0);
                    armed |= 1u << stage;
                    armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == LC_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            for (int s = 0; s < LC_STAGES; ++s)
                if (armed & (1u << s))
                    if (!mbar_wait_drain(&full[s], (armed_parity >> s) & 1u)) report(status, DEV_TIMEOUT);
        }
    } else if (warp == 1) {
        {
            const bool leader = elect_lane();  // the whole warp waits; this lane issues
            // ---------------- MMA issuer: 128 x 256 per row block, accumulators alternate
            constexpr uint32_t idesc = idesc_bf16_f32(BM, LC_BN, false, false);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool issued = false;
            for (int t = cluster; t < m_tiles && !*abort_flag; t += nclusters) {
                if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1)) {
                    report(status, DEV_TIMEOUT);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * LC_BN;
                for (int kb = 0; kb < k_iters; ++kb) {
                    if (!mbar_wait(&full[stage], phase)) {
                        report(status, DEV_TIMEOUT);
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(ring + stage * LC_STAGE);
                    const uint32_t b_addr = a_addr + BM * BK * 2;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        if (leader) umma_f16_ss(d_tmem, sdesc_sw128(a_addr + k * 32, 16, 1024), sdesc_sw128(b_addr + k * 32, 16, 1024),
                                    idesc, (kb | k) != 0 ? 1u : 0u);
                    issued = true;
                    if (leader) umma_commit(&empty[stage]);
                    if (++stage == LC_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (*abort_flag) break;
                if (leader) umma_commit(&acc_full[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            if (*abort_flag && issued) {
                uint64_t *probe = &acc_full[acc];
                if (leader) umma_commit(probe);
                if (!mbar_wait_drain(probe, acc_phase)) report(status, DEV_TIMEOUT);
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5): thread = row of the row block
        const int q = warp & 3;  // TMEM lane quarter
        const int wi = warp - 2;
        uint8_t *wbuf = epi_buf + wi * LC_WARP;  // LC_RSLABS fp32 slabs, then 2 bf16 slabs
        uint64_t *rbar = rbar_all + wi * LC_RSLABS;
        uint32_t rpar = 0, inflight = 0;          // per slab: parity to wait for / a load in flight
        const float inv_n = 1.0f / static_cast<float>(N);
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t it = 0;  // row blocks done by this CTA
        // residual chunk c (32 rows x 32 columns of h32) into slab `sl`, by TMA
        auto load_res = [&](int sl, int c, int row0) {
            mbar_arrive_expect_tx(&rbar[sl], LC_FSLAB);
            tma_load_2d(wbuf + sl * LC_FSLAB, &tm_h, &rbar[sl], n0 + 32 * c, row0);
        };
        for (int t = cluster; t < m_tiles; t += nclusters, ++it) {
            if (*abort_flag) break;
            const int row0 = t * BM + q * 32;
            const int p = static_cast<int>(it & 1);
            constexpr int CH = LC_BN / 32;
            // this row block's statistics: R parts x 128 rows x 8 bytes from the cluster (the
            // barrier's previous phase of this parity, two row blocks ago, has completed)
            if (threadIdx.x == 64) mbar_arrive_expect_tx(&stat_bar[p], static_cast<uint32_t>(R) * BM * 8);
            // the previous row block's stores have read every slab; then the first residual chunks
            if (lane == 0) {
                bulk_wait_read<0>();
                for (int c = 0; c < LC_RSLABS; ++c) load_res(c, c, row0);
            }
            inflight = (1u << LC_RSLABS) - 1;
            __syncwarp();
            if (!mbar_wait(&acc_full[acc], acc_phase)) {
                report(status, DEV_TIMEOUT);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * LC_BN;

            // ---- pass 1: x = (acc + bias) + residual back into TMEM; per-chunk mean and M2
            float cm[CH], cq_sum = 0.f;
            bool ok = true;
            uint32_t vv[2][32];  // TMEM chunks: the next one loads while this one is worked on
            tmem_ld_x32(t_row, vv[0]);
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const int sl = c % LC_RSLABS;
                uint32_t(&v)[32] = vv[c & 1];
                tmem_wait_ld_regs(v);
                if (c + 1 < CH) {
                    if (c >= 1) tmem_wait_st();  // vv[(c + 1) & 1] was the source of chunk c - 1's store
                    tmem_ld_x32(t_row + (c + 1) * 32, vv[(c + 1) & 1]);
                }
                if (!mbar_wait(&rbar[sl], (rpar >> sl) & 1u)) {
                    ok = false;
                    break;
                }
                rpar ^= 1u << sl;
                inflight &= ~(1u << sl);
                const uint8_t *rs = wbuf + sl * LC_FSLAB + lane * 128;
                float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint4 r = *reinterpret_cast<const uint4 *>(rs + ((j ^ (lane & 7)) << 4));
                    const float4 bb = *reinterpret_cast<const float4 *>(vb + c * 32 + 4 * j);
                    float x0 = __uint_as_float(v[4 * j + 0]), x1 = __uint_as_float(v[4 * j + 1]);
                    float x2 = __uint_as_float(v[4 * j + 2]), x3 = __uint_as_float(v[4 * j + 3]);
                    add_f32x2(x0, x1, bb.x, bb.y);
                    add_f32x2(x2, x3, bb.z, bb.w);
                    add_f32x2(x0, x1, __uint_as_float(r.x), __uint_as_float(r.y));
                    add_f32x2(x2, x3, __uint_as_float(r.z), __uint_as_float(r.w));
                    add_f32x2(s4[0], s4[1], x0, x1);
                    add_f32x2(s4[2], s4[3], x2, x3);
                    v[4 * j + 0] = __float_as_uint(x0);
                    v[4 * j + 1] = __float_as_uint(x1);
                    v[4 * j + 2] = __float_as_uint(x2);
                    v[4 * j + 3] = __float_as_uint(x3);
                }
                __syncwarp();  // every lane has read the slab: it takes chunk c + LC_RSLABS
                if (c + LC_RSLABS < CH) {
                    if (lane == 0) load_res(sl, c + LC_RSLABS, row0);
                    inflight |= 1u << sl;
                }
                cm[c] = ((s4[0] + s4[1]) + (s4[2] + s4[3])) * (1.0f / 32.0f);
                float q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    float d0 = __uint_as_float(v[j]), d1 = __uint_as_float(v[j + 1]);
                    add_f32x2(d0, d1, -cm[c], -cm[c]);
                    fma_f32x2v(q4[j & 3], q4[(j & 3) + 1], d0, d1, d0, d1, q4[j & 3], q4[(j & 3) + 1]);
                }
                cq_sum += (q4[0] + q4[1]) + (q4[2] + q4[3]);
                tmem_st_x32(t_row + c * 32, v);
            }
            tmem_wait_ld();
            tmem_wait_st();
            if (!ok) {
                report(status, DEV_TIMEOUT);
                *abort_flag = 1;
                break;
            }
            // (mean, M2) of this row over the CTA's 256 columns: equal-size chunks combined exactly
            float mean = 0.f;
#pragma unroll
            for (int c = 0; c < CH; ++c) mean += cm[c];
            mean *= 1.0f / CH;
            float m2 = 0.f;
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const float d = cm[c] - mean;
                m2 += d * d;
            }
            m2 = cq_sum + 32.0f * m2;

            // ---- exchange: this part to every CTA of the cluster, then the row's R parts
            float2 *slot = stats + (p * LC_MAX_R + static_cast<int>(rank)) * BM + q * 32 + lane;
            for (int k = 0; k < R; ++k)
                st_async_v2(map_to_rank(slot, static_cast<uint32_t>(k)), mean, m2,
                            map_to_rank(&stat_bar[p], static_cast<uint32_t>(k)));
            if (!mbar_wait_cluster(&stat_bar[p], (it >> 1) & 1)) {
                report(status, DEV_TIMEOUT);
                *abort_flag = 1;
                break;
            }
            float gm = 0.f;
            float2 part[LC_MAX_R];
#pragma unroll
            for (int k = 0; k < LC_MAX_R; ++k)
                if (k < R) {
                    part[k] = stats[(p * LC_MAX_R + k) * BM + q * 32 + lane];
                    gm += part[k].x;
                }
            gm /= static_cast<float>(R);
            float gq = 0.f, gd = 0.f;
#pragma unroll
            for (int k = 0; k < LC_MAX_R; ++k)
                if (k < R) {
                    const float d = part[k].x - gm;
                    gq += part[k].y;
                    gd += d * d;
                }
            gq += static_cast<float>(LC_BN) * gd;
            const float inv_sd = 1.0f / sqrtf(gq * inv_n + eps);

            // ---- pass 2: normalise from TMEM; per 32-column chunk an fp32 slab (128B swizzle)
            // and a bf16 slab (64B swizzle), TMA-stored as one bulk group, double-buffered
            tmem_ld_x32(t_row, vv[0]);
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                uint32_t(&v)[32] = vv[c & 1];
                tmem_wait_ld_regs(v);
                if (c + 1 < CH) tmem_ld_x32(t_row + (c + 1) * 32, vv[(c + 1) & 1]);
                float o[32];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 g = *reinterpret_cast<const float4 *>(vg + c * 32 + 4 * j);
                    const float4 e = *reinterpret_cast<const float4 *>(ve + c * 32 + 4 * j);
                    float t0 = __uint_as_float(v[4 * j + 0]), t1 = __uint_as_float(v[4 * j + 1]);
                    float t2 = __uint_as_float(v[4 * j + 2]), t3 = __uint_as_float(v[4 * j + 3]);
                    add_f32x2(t0, t1, -gm, -gm);
                    add_f32x2(t2, t3, -gm, -gm);
                    mul_f32x2(t0, t1, inv_sd, inv_sd);
                    mul_f32x2(t2, t3, inv_sd, inv_sd);
                    fma_f32x2v(o[4 * j + 0], o[4 * j + 1], t0, t1, g.x, g.y, e.x, e.y);
                    fma_f32x2v(o[4 * j + 2], o[4 * j + 3], t2, t3, g.z, g.w, e.z, e.w);
                }
                uint8_t *fs = wbuf + (c % LC_RSLABS) * LC_FSLAB;
                uint8_t *bs = wbuf + LC_RSLABS * LC_FSLAB + (c & 1) * LC_BSLAB;
                if (lane == 0) bulk_wait_read<1>();  // the groups of chunks up to c - 2 have read their slabs
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    *reinterpret_cast<uint4 *>(fs + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                        make_uint4(__float_as_uint(o[4 * j + 0]), __float_as_uint(o[4 * j + 1]),
                                   __float_as_uint(o[4 * j + 2]), __float_as_uint(o[4 * j + 3]));
                if (write16) {
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        *reinterpret_cast<uint4 *>(bs + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
                            make_uint4(pack_bf16x2(o[8 * j + 0], o[8 * j + 1]), pack_bf16x2(o[8 * j + 2], o[8 * j + 3]),
                                       pack_bf16x2(o[8 * j + 4], o[8 * j + 5]), pack_bf16x2(o[8 * j + 6], o[8 * j + 7]));
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tm_h, fs, n0 + c * 32, row0);
                    if (write16) tma_store_2d(&tm_h16, bs, n0 + c * 32, row0);
                    bulk_commit();
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
        // residual loads still in flight (an abandoned row block) land before the CTA exits
        if (lane == 0) {
            for (int sl = 0; sl < LC_RSLABS; ++sl)
                if (inflight & (1u << sl))
                    if (!mbar_wait_drain(&rbar[sl], (rpar >> sl) & 1u)) report(status, DEV_TIMEOUT);
            bulk_wait_all<0>();
        }
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no CTA leaves while a peer may still write its shared memory or arrive on it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * LC_BN);
    }
}

// FE_LN_CLUSTER: 0 = never use linear_ln_cluster; "all" = also where the pair kernel would
// fuse (K >= 2048, for comparison); otherwise (default) for the shapes the pair kernel leaves
// to two launches.
int ln_cluster_mode()
{
    const char *v = getenv("FE_LN_CLUSTER");
    if (v && v[0] == '0') return 0;
    if (v && v[0] == 'a') return 2;
    return 1;
}

// Clusters of linear_ln_cluster with R CTAs that can be resident at once (0 if unknown).
int ln_cluster_resident(int R)
{
    static int cached[64][LC_MAX_R + 1] = {};
    static uint64_t cached_ctx[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t ctx = current_context_id();
    if (dev < 64 && cached_ctx[dev] == ctx && cached[dev][R] > 0) return cached[dev][R];
    if (cudaFuncSetAttribute(linear_ln_cluster, cudaFuncAttributeMaxDynamicSharedMemorySize, LC_SMEM) != cudaSuccess)
        return 0;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = R;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(R, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = LC_SMEM;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, linear_ln_cluster, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (dev < 64) {
        if (cached_ctx[dev] != ctx) {
            for (int r = 0; r <= LC_MAX_R; ++r) cached[dev][r] = 0;
            cached_ctx[dev] = ctx;
        }
        cached[dev][R] = clusters;
    }
    return clusters;
}

cudaError_t launch_ln_cluster(const void *x, const void *w, const float *bias, const float *gamma, const float *beta,
                              float *h32, void *h16, int64_t m, int64_t n, int64_t k, float eps, cudaStream_t s,
                              fe_status *st)
{
    const int R = static_cast<int>(n / LC_BN);
    CUtensorMap tx, tw, th, th16;
    fe_status r = make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m, k, k, BM, BK);
    if (r == FE_OK) r = make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, n, k, k, LC_BN, BK);
    if (r == FE_OK) r = make_tmap_2d(&th, h32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, m, n, n, 32, 32);
    if (r == FE_OK)
        r = h16 ? make_tmap_2d(&th16, h16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m, n, n, 32, 32,
                               CU_TENSOR_MAP_SWIZZLE_64B)
                : make_tmap_2d(&th16, h32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, m, n, n, 32, 32);  // not used
    if (r != FE_OK) {
        *st = r;
        return cudaSuccess;
    }
    const int resident = ln_cluster_resident(R);
    if (resident < 1) {
        *st = fail(FE_ERR_UNSUPPORTED, "linear+LayerNorm: no cluster of this size fits on the device");
        return cudaSuccess;
    }
    const int m_tiles = static_cast<int>((m + BM - 1) / BM);
    int nclusters = std::min(resident, current_sm_count() / R);
    if (nclusters > m_tiles) nclusters = m_tiles;
    if (nclusters < 1) nclusters = 1;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = R;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(R * nclusters, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = LC_SMEM;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const int M = static_cast<int>(m), N = static_cast<int>(n), K = static_cast<int>(k);
    return cudaLaunchKernelEx(&cfg, linear_ln_cluster, tx, tw, th, th16, M, N, K, bias, gamma, beta ? beta : gamma, h32,
                              eps, h16 ? 1 : 0, current_device_status_word());
}

}  // namespace

bool ln_cluster_applies(int64_t n, int64_t k, bool rms, bool pair_fused)
{
    const int mode = ln_cluster_mode();
    if (rms || mode == 0 || n % LC_BN != 0 || n / LC_BN < 2 || n / LC_BN > LC_MAX_R || k % BK != 0) return false;
    return mode == 2 || !pair_fused;
}

cudaError_t launch_linear_layernorm(const void *x, const void *w, const float *bias, const float *gamma,
                                    const float *beta, float *h32, void *h16, int64_t m, int64_t n, int64_t k,
                                    float eps, void *stats, float *y_fallback, cudaStream_t s, fe_status *st, bool rms)
{
    *st = FE_OK;
    if (m == 0 || n == 0) return cudaSuccess;
    const int n_tiles = static_cast<int>(n / P_BN);
    // fused only where the mainloop hides the statistics exchange (see linear_ln_tcgen05_pair)
    bool fused = k >= 2048 && pair_mode_enabled() && norm_fuse_enabled() && n % P_BN == 0 && n_tiles <= kMaxLnParts && stats;
    int pairs = 0;
    const LnVariant var = pick_ln_variant(k);
    if (fused) {
        const int tiles = static_cast<int>((m + 255) / 256) * n_tiles;
        pairs = std::min(var.resident(), current_sm_count() / 2);
        pairs = pairs / n_tiles * n_tiles;  // each row group's tiles in the same round
        if (pairs > tiles) pairs = tiles;
        fused = pairs >= n_tiles;
    }
    if (ln_cluster_applies(n, k, rms, fused)) return launch_ln_cluster(x, w, bias, gamma, beta, h32, h16, m, n, k, eps, s, st);
    if (!fused && rms) {
        // Unfused pre-norm form: x = x W^T + b + h32 in place, then RMSNorm into h16.
        cudaError_t e = launch_linear_bf16(x, w, bias, h32, h32, m, n, k, FE_EPI_BIAS_RESIDUAL, FE_DTYPE_F32, s, st);
        if (e != cudaSuccess || *st != FE_OK || !h16) return e;
        return launch_rms_norm_rows(h32, gamma, false, eps, m, static_cast<int>(n), nullptr, h16, s);
    }
    if (!fused) {
        // Unfused form of the same step: linear with bias into fp32, then residual + LayerNorm.
        if (!y_fallback) {
            *st = fail(FE_ERR_INVALID_ARGUMENT, "linear+LayerNorm: no fp32 scratch for this shape");
            return cudaSuccess;
        }
        cudaError_t e = launch_linear_bf16(x, w, bias, nullptr, y_fallback, m, n, k, FE_EPI_BIAS, FE_DTYPE_F32, s, st);
        if (e != cudaSuccess || *st != FE_OK) return e;
        return launch_layernorm_dual(y_fallback, h32, gamma, beta, h32, h16, m, static_cast<int>(n), eps, s);
    }
    CUtensorMap tx, tw, th, th16;
    fe_status r = make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m, k, k, BM, BK);
    if (r == FE_OK) r = make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, n, k, k, 128, BK);
    if (r == FE_OK) r = make_tmap_2d(&th, h32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, m, n, n, 32, 32);
    if (r == FE_OK)
        r = h16 ? make_tmap_2d(&th16, h16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m, n, n, 32, 32,
                               CU_TENSOR_MAP_SWIZZLE_64B)
                : make_tmap_2d(&th16, h32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, m, n, n, 32, 32);  // not used
    if (r != FE_OK) {
        *st = r;
        return cudaSuccess;
    }
    LnParams p;
    p.bias = bias;
    p.gamma = gamma;
    p.beta = beta ? beta : gamma;  // read into shared memory; unused by the RMSNorm form
    p.stats = static_cast<unsigned long long *>(stats);
    p.eps = eps;
    p.nparts = static_cast<int>(n / var.cols);
    p.rms = rms ? 1 : 0;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(s, &cap);
    const bool order = cap == cudaStreamCaptureStatusNone && dev < 64;
    const uint64_t ctx = current_context_id();
    std::lock_guard<std::mutex> lock(g_ln_mu);
    if (order && g_ln_last[dev] && g_ln_last_ctx[dev] != ctx) {
        // the device was reset since the event was made: it and its stream are gone
        g_ln_last[dev] = nullptr;
        g_ln_last_stream[dev] = nullptr;
    }
    unsigned &ep = g_ln_epoch[stats];
    if (++ep == 0) ep = 1;
    p.epoch = ep;
    if (order && g_ln_last[dev] && g_ln_last_stream[dev] != s) {
        cudaError_t e = cudaStreamWaitEvent(s, g_ln_last[dev], 0);
        if (e != cudaSuccess) return e;
    }
    const int M = static_cast<int>(m), N = static_cast<int>(n), K = static_cast<int>(k);
    const int w16 = h16 != nullptr;
    int *status = current_device_status_word();
    cudaError_t e = launch_k(var.kern, dim3(2 * pairs), dim3(var.threads), var.smem, s, tx, tw, th, th16, M, N, K, p,
                             w16, status);
    if (e != cudaSuccess) return e;
    if (order) {
        if (!g_ln_last[dev]) {
            e = cudaEventCreateWithFlags(&g_ln_last[dev], cudaEventDisableTiming);
            if (e != cudaSuccess) return e;
            g_ln_last_ctx[dev] = ctx;
        }
        e = cudaEventRecord(g_ln_last[dev], s);
        g_ln_last_stream[dev] = s;
    }
    return e;
}

}  // namespace fe

namespace fe {

int linear_rms_deferred_parts(int64_t n) { return static_cast<int>(n / LnCfg<5, 4, 2>::COLS); }

cudaError_t launch_linear_rms_deferred(const void *x, const void *w, const float *bias, const float *gamma, float *h32,
                                       void *h16, float *row_ss, int64_t m, int64_t n, int64_t k, cudaStream_t s,
                                       fe_status *st)
{
    *st = FE_OK;
    if (m == 0 || n == 0) return cudaSuccess;
    const int n_tiles = static_cast<int>(n / P_BN);
    if (n % P_BN != 0 || n_tiles > kMaxLnParts) {
        *st = fail(FE_ERR_UNSUPPORTED, "linear + deferred RMSNorm: n must be a multiple of 256, at most 2048");
        return cudaSuccess;
    }
    const LnVariant var = pick_ln_variant(k, true);
    static_assert(LnCfg<5, 4, 2>::COLS == LnCfg<6, 4, 1>::COLS, "one partial count for both variants");
    const int tiles = static_cast<int>((m + 255) / 256) * n_tiles;
    // no pair waits for another in this form; the grid is still a multiple of n_tiles, so
    // that every tile of a pair has the same columns
    int pairs = std::min(var.resident(), current_sm_count() / 2);
    pairs = pairs / n_tiles * n_tiles;
    if (pairs > tiles) pairs = tiles;
    if (pairs < n_tiles) {
        *st = fail(FE_ERR_UNSUPPORTED, "linear + deferred RMSNorm: too few resident CTA pairs");
        return cudaSuccess;
    }
    CUtensorMap tx, tw, th, th16;
    fe_status r = make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m, k, k, BM, BK);
    if (r == FE_OK) r = make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, n, k, k, 128, BK);
    if (r == FE_OK) r = make_tmap_2d(&th, h32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, m, n, n, 32, 32);
    if (r == FE_OK)
        r = h16 ? make_tmap_2d(&th16, h16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m, n, n, 32, 32,
                               CU_TENSOR_MAP_SWIZZLE_64B)
                : make_tmap_2d(&th16, h32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, m, n, n, 32, 32);  // not used
    if (r != FE_OK) {
        *st = r;
        return cudaSuccess;
    }
    LnParams p;
    p.bias = bias;
    p.gamma = gamma;
    p.beta = gamma;  // read into shared memory, unused
    p.stats = reinterpret_cast<unsigned long long *>(row_ss);
    p.epoch = 1;
    p.eps = 0.f;
    p.nparts = static_cast<int>(n / var.cols);
    p.rms = 2;
    const int M = static_cast<int>(m), N = static_cast<int>(n), K = static_cast<int>(k);
    return launch_k(var.kern, dim3(2 * pairs), dim3(var.threads), var.smem, s, tx, tw, th, th16, M, N, K, p,
                    h16 != nullptr ? 1 : 0, current_device_status_word());
}

cudaError_t set_wait_limit_linear(uint64_t ns) { return set_wait_limit_this_file(ns); }
}  // namespace fe
