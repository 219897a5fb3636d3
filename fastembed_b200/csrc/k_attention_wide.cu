// k_attention_wide.cu — variable-length attention on tcgen05 for head_dim 128 and 256,
// with grouped-query heads and an optional causal mask: the attention of the Qwen3
// (16 query / 8 key-value heads x 128, causal) and Gemma3 (3 / 1 x 256, bidirectional)
// encoders.  These shapes are not in the reference; the semantics are those of the
// model definitions (softmax(Q K^T * scale) V per sentence, key j of a query i kept
// when j < len and, causal, j <= i).
//
// One CTA per SM, persistent over units (sentence, 128-row query tile, query head);
// the key-value head of query head h is h / (q_heads / kv_heads).  TMEM (512 columns):
// two 128-column S slots, then one or two O accumulators of head_dim columns.
//   warp 0     TMA producer: the Q tile of a unit and the K and V tiles of each 128-key
//              item, each as head_dim / 64 boxes of 128 rows x 128 bytes (128B swizzle);
//              K and V advance independently (measured on the Qwen3-0.6B shape, 71,550
//              tokens, with an L2 prefetch since removed: 648 -> 557 us).
//   warp 1     MMA issuer: S = Q K^T (K = head_dim) into an S slot; for the previous item
//              O (+)= P V with P (bf16) read from TMEM and V an MN-major operand; the
//              first item of a unit overwrites O.  (Issuing each PV as soon as its P is
//              written, from a polled queue, measured 1 % slower.)
//   warps 2-5  softmax (thread = query row): masked online softmax over S, P written back
//              over S; when a row's reference max rises (by more than 2^8 in P), O is
//              rescaled in TMEM after the previous item's PV and before this one's; O / l
//              of a unit is stored as bf16 after the softmax of the next unit's first item.
// Waits are bounded; on timeout the CTA records FE_ERR_DEVICE_TIMEOUT and leaves.
#include <cuda.h>
#include <cuda_bf16.h>

#include "fe_common.cuh"
#include "fe_internal.h"

namespace fe {
namespace {

constexpr int TQ = 128;
constexpr int TK = 128;
constexpr int kThreadsW = 192;
constexpr int kMaxBatchW = 2048;
constexpr uint32_t BOX_BYTES = 128 * 128;  // 128 rows x 64 bf16
constexpr uint32_t WBAR_BYTES = 512;

template <int HD>
struct WCfg {
    static constexpr int BOXES = HD / 64;
    static constexpr uint32_t TILE = BOXES * BOX_BYTES;  // one Q, K or V tile
    static constexpr int QS = HD == 128 ? 2 : 1;         // Q slots
    static constexpr int KVS = HD == 128 ? 2 : 1;        // K / V slots
    static constexpr int OS = HD == 128 ? 2 : 1;         // O accumulators in TMEM
    static constexpr uint32_t SMEM = 1024 + QS * TILE + 2 * KVS * TILE + WBAR_BYTES + 4 * (kMaxBatchW + 1) + 64;
    static_assert(256 + OS * HD <= 512, "TMEM columns");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ float fast_exp2w(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int HD>
__global__ void __launch_bounds__(kThreadsW, 1)
    attn_wide_tcgen05(const __grid_constant__ CUtensorMap tm_qkv, const int32_t *__restrict__ cu_seqlens, int batch,
                      int q_heads, int kv_heads, int causal, float scale_log2, __nv_bfloat16 *__restrict__ out,
                      int *status)
{
    using C = WCfg<HD>;
    constexpr int QS = C::QS, KVS = C::KVS, OS = C::OS, BOXES = C::BOXES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem;
    uint8_t *sK = sQ + QS * C::TILE;
    uint8_t *sV = sK + KVS * C::TILE;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sV + KVS * C::TILE);
    uint64_t *q_full = bars;             // [QS]
    uint64_t *q_empty = q_full + QS;     // [QS]
    uint64_t *k_full = q_empty + QS;     // [KVS]
    uint64_t *k_empty = k_full + KVS;    // [KVS]
    uint64_t *v_full = k_empty + KVS;    // [KVS]
    uint64_t *v_empty = v_full + KVS;    // [KVS]
    uint64_t *s_full = v_empty + KVS;    // [2] S of a slot ready
    uint64_t *s_free = s_full + 2;       // [2] the PV reading P of a slot is done
    uint64_t *p_full = s_free + 2;       // [2] P of a slot written (and O corrected)
    uint64_t *pv_done = p_full + 2;      // [2] the PV of the item in a slot is done
    uint64_t *o_free = pv_done + 2;      // [OS] an O accumulator has been read out
    uint64_t *probe = o_free + OS;       // [1]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(probe + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *warp_tot = reinterpret_cast<int *>(tmem_slot + 2);
    int *upre = reinterpret_cast<int *>(reinterpret_cast<uint8_t *>(bars) + WBAR_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int group = q_heads / kv_heads;
    const int k_col0 = q_heads * HD, v_col0 = (q_heads + kv_heads) * HD;

    if (threadIdx.x == 0) {
        for (int i = 0; i < QS; ++i) {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], 1);
        }
        for (int i = 0; i < KVS; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 1);
            mbar_init(&p_full[i], 4);  // one arrival per softmax warp
            mbar_init(&pv_done[i], 1);
        }
        for (int i = 0; i < OS; ++i) mbar_init(&o_free[i], 4);
        mbar_init(probe, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tm_qkv);
    }
    grid_dep_wait();
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    // upre[s] = units of the sentences before s (ceil(len / 128) query tiles x q_heads each)
    {
        constexpr int nwarps = kThreadsW / 32;
        int carry = 0;
        for (int c0 = 0; c0 < batch; c0 += kThreadsW) {
            const int i = c0 + threadIdx.x;
            int v = 0;
            if (i < batch) v = ((cu_seqlens[i + 1] - cu_seqlens[i] + TQ - 1) / TQ) * q_heads;
            int x = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            if (lane == 31) warp_tot[warp] = x;
            __syncthreads();
            int off = carry, total = 0;
#pragma unroll
            for (int w2 = 0; w2 < nwarps; ++w2) {
                if (w2 < warp) off += warp_tot[w2];
                total += warp_tot[w2];
            }
            if (i < batch) upre[i + 1] = off + x;
            carry += total;
            __syncthreads();
        }
        if (threadIdx.x == 0) upre[0] = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    grid_dep_launch();
    const uint32_t tmem = *tmem_slot;
    const int total_units = upre[batch];

    struct U {
        int start, len, q0, head, n_kv;
    };
    // The k-th unit of this CTA (units blockIdx.x, + gridDim.x, ...).
    auto unit = [&](int g) -> U {
        int lo = 0, hi = batch - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (upre[mid] <= g) lo = mid;
            else hi = mid - 1;
        }
        const int rr = g - upre[lo];
        U w;
        w.start = cu_seqlens[lo];
        w.len = cu_seqlens[lo + 1] - w.start;
        w.head = rr % q_heads;
        const int t = rr / q_heads;
        w.q0 = t * TQ;
        const int nk = (w.len + TK - 1) / TK;
        w.n_kv = causal ? min(nk, t + 1) : nk;
        return w;
    };
    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (mbar_wait(bar, parity)) return true;
        report(status, DEV_TIMEOUT);
        *abort_flag = 1;
        return false;
    };

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer
            // K and V tiles are loaded by two cursors over the same item sequence, each
            // as soon as its own slot is released (a K slot when the S two items back is
            // done, a V slot when that item's PV is), so no K load queues behind a V slot.
            // A unit's Q tile is loaded when the K cursor enters the unit.  (Prefetching the
            // next unit's tiles into L2 then measured slower: 516 vs 502 us on the Qwen3
            // shape, 134 vs 122 us on the Gemma one.)
            bool ok = true;
            uint32_t qn = 0, kn = 0, vn = 0;
            uint32_t q_armed = 0, q_par = 0, k_armed = 0, k_par = 0, v_armed = 0, v_par = 0;
            struct Cur {
                int g, j;
                U w;
            };
            auto start_at = [&](Cur &c, int g) {
                c.g = g;
                c.j = 0;
                if (g < total_units) c.w = unit(g);
            };
            auto advance = [&](Cur &c) {
                if (++c.j == c.w.n_kv) start_at(c, c.g + static_cast<int>(gridDim.x));
            };
            Cur kc, vc;
            start_at(kc, blockIdx.x);
            start_at(vc, blockIdx.x);
            uint64_t t_last = globaltimer_ns();
            for (uint32_t i = 0; ok && !*abort_flag; ++i) {
                const bool k_more = kc.g < total_units, v_more = vc.g < total_units;
                if (!k_more && !v_more) break;
                bool progress = false;
                if (k_more) {
                    const int ks = kn % KVS;
                    const int qs = qn % QS;
                    bool can = mbar_test_wait(&k_empty[ks], ((kn / KVS) & 1) ^ 1);
                    if (can && kc.j == 0) can = mbar_test_wait(&q_empty[qs], ((qn / QS) & 1) ^ 1);
                    if (can) {
                        const U &w = kc.w;
                        if (kc.j == 0) {
                            mbar_arrive_expect_tx(&q_full[qs], C::TILE);
                            for (int b = 0; b < BOXES; ++b)
                                tma_load_2d(sQ + qs * C::TILE + b * BOX_BYTES, &tm_qkv, &q_full[qs],
                                            w.head * HD + 64 * b, w.start + w.q0);
                            q_armed |= 1u << qs;
                            q_par = (q_par & ~(1u << qs)) | (((qn / QS) & 1) << qs);
                            ++qn;
                        }
                        mbar_arrive_expect_tx(&k_full[ks], C::TILE);
                        for (int b = 0; b < BOXES; ++b)
                            tma_load_2d(sK + ks * C::TILE + b * BOX_BYTES, &tm_qkv, &k_full[ks],
                                        k_col0 + (w.head / group) * HD + 64 * b, w.start + kc.j * TK);
                        k_armed |= 1u << ks;
                        k_par = (k_par & ~(1u << ks)) | (((kn / KVS) & 1) << ks);
                        ++kn;
                        advance(kc);
                        progress = true;
                    }
                }
                if (v_more && vn < kn) {
                    const int vs = vn % KVS;
                    if (mbar_test_wait(&v_empty[vs], ((vn / KVS) & 1) ^ 1)) {
                        const U &w = vc.w;
                        mbar_arrive_expect_tx(&v_full[vs], C::TILE);
                        for (int b = 0; b < BOXES; ++b)
                            tma_load_2d(sV + vs * C::TILE + b * BOX_BYTES, &tm_qkv, &v_full[vs],
                                        v_col0 + (w.head / group) * HD + 64 * b, w.start + vc.j * TK);
                        v_armed |= 1u << vs;
                        v_par = (v_par & ~(1u << vs)) | (((vn / KVS) & 1) << vs);
                        ++vn;
                        advance(vc);
                        progress = true;
                    }
                }
                if (progress) {
                    t_last = globaltimer_ns();
                } else {
                    __nanosleep(32);
                    if (((i & 255u) == 255u || wait_limit_ns() < kShortWaitNs) && globaltimer_ns() - t_last > wait_limit_ns()) {
                        report(status, DEV_TIMEOUT);
                        *abort_flag = 1;
                        ok = false;
                    }
                }
            }
            // every load this thread started lands before the CTA exits
            for (int i = 0; i < QS; ++i)
                if ((q_armed >> i) & 1) (void)mbar_wait_drain(&q_full[i], (q_par >> i) & 1);
            for (int i = 0; i < KVS; ++i) {
                if ((k_armed >> i) & 1) (void)mbar_wait_drain(&k_full[i], (k_par >> i) & 1);
                if ((v_armed >> i) & 1) (void)mbar_wait_drain(&v_full[i], (v_par >> i) & 1);
            }
        }
    } else if (warp == 1) {
        {
            // ------------------------------------------------ MMA issuer (the whole warp waits; the
            // elected lane issues)
            const bool leader = elect_lane();
            constexpr uint32_t idesc_o = idesc_bf16_f32(TQ, HD, false, true);
            uint32_t qn = 0, kvn = 0, it = 0, un = 0;
            bool ok = true, issued = false, have_pend = false;
            uint32_t pend_it = 0, pend_ks = 0, pend_kvn = 0, pend_o = 0, pend_un = 0;
            int pend_valid = 0;
            bool pend_first = false;
            // O(o) (+)= P(slot) V for item `pit` (P from TMEM, V MN-major: 16 keys = 2048 bytes a step)
            auto issue_pv = [&]() -> bool {
                const uint32_t b = pend_it & 1;
                if (pend_first && !wait(&o_free[pend_o], ((pend_un / OS) & 1) ^ 1)) return false;
                if (!wait(&p_full[b], (pend_it >> 1) & 1)) return false;
                if (!wait(&v_full[pend_ks], (pend_kvn / KVS) & 1)) return false;
                tc_fence_after();
                const uint64_t v_desc = sdesc_sw128(smem_u32(sV + pend_ks * C::TILE), BOX_BYTES, 1024);
                const uint32_t o_tmem = tmem + 256 + pend_o * HD;
                const int nks = (pend_valid + 15) >> 4;
                for (int ks = 0; ks < nks; ++ks)
                    if (leader) umma_f16_ts(o_tmem, tmem + b * 128 + ks * 8, v_desc + static_cast<uint64_t>(ks * 128), idesc_o,
                                (pend_first && ks == 0) ? 0u : 1u);
                if (leader) umma_commit(&pv_done[b]);
                if (leader) umma_commit(&s_free[b]);
                if (leader) umma_commit(&v_empty[pend_ks]);
                return true;
            };
            for (int g = blockIdx.x; g < total_units && ok && !*abort_flag; g += gridDim.x) {
                const U w = unit(g);
                const int qs = qn % QS;
                if (!(ok = wait(&q_full[qs], (qn / QS) & 1))) break;
                for (int j = 0; j < w.n_kv; ++j) {
                    const uint32_t ks = kvn % KVS;
                    const uint32_t b = it & 1;
                    if (!(ok = wait(&k_full[ks], (kvn / KVS) & 1))) break;
                    if (!(ok = wait(&s_free[b], ((it >> 1) & 1) ^ 1))) break;
                    tc_fence_after();
                    const int valid = min(TK, w.len - j * TK);
                    const int n = min(TK, max(16, (valid + 15) & ~15));
                    const uint32_t idesc_s = idesc_bf16_f32(TQ, n, false, false);
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk) {  // 4 K steps per 128-byte swizzle atom, then the next box
                        const uint32_t off = (kk >> 2) * BOX_BYTES + (kk & 3) * 32;
                        if (leader) umma_f16_ss(tmem + b * 128, sdesc_sw128(smem_u32(sQ + qs * C::TILE) + off, 16, 1024),
                                    sdesc_sw128(smem_u32(sK + ks * C::TILE) + off, 16, 1024), idesc_s,
                                    kk != 0 ? 1u : 0u);
                    }
                    issued = true;
                    if (leader) umma_commit(&s_full[b]);
                    if (leader) umma_commit(&k_empty[ks]);
                    if (j == w.n_kv - 1 && leader) umma_commit(&q_empty[qs]);
                    if (have_pend && !(ok = issue_pv())) break;
                    have_pend = true;
                    pend_it = it;
                    pend_ks = ks;
                    pend_kvn = kvn;
                    pend_o = un % OS;
                    pend_un = un;
                    pend_valid = valid;
                    pend_first = j == 0;
                    ++it;
                    ++kvn;
                }
                ++qn;
                ++un;
            }
            if (ok && have_pend && !*abort_flag) ok = issue_pv();
            if (issued) {
                if (leader) umma_commit(probe);
                (void)mbar_wait_drain(probe, 0);
            }
        }
    } else {
        // ------------------------------------------------ softmax warps 2..5
        const int q = warp & 3;
        const int r = q * 32 + lane;  // query row within the tile == TMEM lane
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        uint32_t it = 0, un = 0;
        bool ok = true;
        // A unit's output step (wait for its last PV, O / l out, release the accumulator)
        // runs after the softmax of the next unit's first item, so the PV is not waited for.
        bool pe_have = false, pe_live = false, pe_row_ok = false;
        uint32_t pe_it = 0, pe_ocol = 0, pe_oslot = 0;
        float pe_l = 0.f;
        __nv_bfloat16 *pe_dst = nullptr;
        auto flush = [&]() -> bool {
            pe_have = false;
            if (!wait(&pv_done[pe_it & 1], (pe_it >> 1) & 1)) return false;
            tc_fence_after();
            if (pe_live) {
                const float inv = pe_l > 0.f ? 1.0f / pe_l : 0.f;
#pragma unroll 1
                for (int c = 0; c < HD; c += 32) {
                    uint32_t v[32];
                    tmem_ld_x32(tmem + lane_base + pe_ocol + c, v);
                    tmem_wait_ld_regs(v);
                    if (pe_row_ok) {
                        uint4 *d4 = reinterpret_cast<uint4 *>(pe_dst + c);
#pragma unroll
                        for (int x = 0; x < 4; ++x)
                            d4[x] = make_uint4(pack_bf16x2(__uint_as_float(v[8 * x + 0]) * inv, __uint_as_float(v[8 * x + 1]) * inv),
                                               pack_bf16x2(__uint_as_float(v[8 * x + 2]) * inv, __uint_as_float(v[8 * x + 3]) * inv),
                                               pack_bf16x2(__uint_as_float(v[8 * x + 4]) * inv, __uint_as_float(v[8 * x + 5]) * inv),
                                               pack_bf16x2(__uint_as_float(v[8 * x + 6]) * inv, __uint_as_float(v[8 * x + 7]) * inv));
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free[pe_oslot]);
            return true;
        };
        for (int g = blockIdx.x; g < total_units && ok; g += gridDim.x) {
            if (*abort_flag) break;
            const U w = unit(g);
            const uint32_t o_col = 256 + (un % OS) * HD;
            const bool warp_live = w.q0 + q * 32 < w.len;
            const int qi = w.q0 + r;  // this thread's query position in the sentence
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < w.n_kv; ++j) {
                const uint32_t b = it & 1;
                if (!(ok = wait(&s_full[b], (it >> 1) & 1))) break;
                tc_fence_after();
                const int valid = min(TK, w.len - j * TK);
                // keys kept for this row: c < lim (key position j * 128 + c)
                const int lim = causal ? min(valid, qi - j * TK + 1) : valid;
                const uint32_t tS = tmem + lane_base + b * 128;
                float alpha = 1.f, rs = 0.f, mx = m_run;
                if (warp_live) {
                    float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                    for (int c = 0; c < valid; c += 32) {
                        uint32_t v[32];
                        tmem_ld_x32(tS + c, v);
                        tmem_wait_ld_regs(v);
                        if (c + 32 <= lim) {  // no masked key in the chunk (all but the row's last)
#pragma unroll
                            for (int i = 0; i < 32; i += 2)
                                m4[(i >> 1) & 3] = max3f(m4[(i >> 1) & 3], __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (c + i < lim) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(v[i]));
                        }
                    }
                    const float tmax = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * scale_log2;
                    // Lazy reference max: P = exp2(s - m) with m raised only when a tile's max
                    // exceeds it by more than 8 (P <= 2^8 stays exact enough in fp32 sums and
                    // bf16 P), so O in TMEM is rescaled only then.  O and l share the scale.
                    if (m_run == -INFINITY || tmax > m_run + 8.0f) mx = fmaxf(m_run, tmax);
                    // a row with no kept key yet keeps m = -inf
                    alpha = mx == m_run ? 1.f : (m_run == -INFINITY ? 0.f : fast_exp2w(m_run - mx));
                    const float msub = mx == -INFINITY ? 0.f : mx;
                    float rs0 = 0.f, rs1 = 0.f;
                    for (int c = 0; c < valid; c += 32) {
                        uint32_t v[32];
                        tmem_ld_x32(tS + c, v);
                        tmem_wait_ld_regs(v);
                        uint32_t pk[16];
                        if (c + 32 <= lim) {
#pragma unroll
                            for (int i = 0; i < 16; ++i) {  // packed f32x2: scale and shift, then row sums
                                float p0, p1;
                                fma_f32x2(p0, p1, __uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]), scale_log2,
                                          -msub);
                                p0 = fast_exp2w(p0);
                                p1 = fast_exp2w(p1);
                                add_f32x2(rs0, rs1, p0, p1);
                                pk[i] = pack_bf16x2(p0, p1);
                            }
                        } else if (c >= lim) {  // every key of the chunk masked
#pragma unroll
                            for (int i = 0; i < 16; ++i) pk[i] = 0u;
                        } else {
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const float p0 =
                                    c + 2 * i < lim ? fast_exp2w(fmaf(__uint_as_float(v[2 * i]), scale_log2, -msub)) : 0.f;
                                const float p1 = c + 2 * i + 1 < lim
                                                     ? fast_exp2w(fmaf(__uint_as_float(v[2 * i + 1]), scale_log2, -msub))
                                                     : 0.f;
                                rs0 += p0;
                                rs1 += p1;
                                pk[i] = pack_bf16x2(p0, p1);
                            }
                        }
                        tmem_st_x16(tS + (c >> 1), pk);
                    }
                    rs = rs0 + rs1;
                    tmem_wait_st();
                }
                // O *= alpha before this item's PV accumulates (needs the previous PV done)
                if (j > 0 && warp_live && __any_sync(0xffffffffu, alpha != 1.f)) {
                    if (!(ok = wait(&pv_done[(it - 1) & 1], ((it - 1) >> 1) & 1))) break;
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < HD; c += 32) {
                        uint32_t v[32];
                        tmem_ld_x32(tmem + lane_base + o_col + c, v);
                        tmem_wait_ld_regs(v);
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
                        tmem_st_x32(tmem + lane_base + o_col + c, v);
                    }
                    tmem_wait_st();
                }
                l_run = l_run * alpha + rs;
                m_run = mx;
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[b]);
                ++it;
                if (j == 0 && pe_have && !(ok = flush())) break;
            }
            if (!ok) break;
            pe_have = true;
            pe_it = it - 1;
            pe_ocol = o_col;
            pe_oslot = un % OS;
            pe_live = warp_live;
            pe_row_ok = qi < w.len;
            pe_l = l_run;
            pe_dst = out + static_cast<size_t>(w.start + qi) * (q_heads * HD) + w.head * HD;
            ++un;
        }
        if (ok && pe_have && !*abort_flag) (void)flush();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// Head-pair kernel for head_dim 128 with an even number of query heads per key-value
// head (Qwen3: 16 / 8).  A unit is (sentence, 128-row query tile, key-value head, pair
// of its query heads).  The pair's two query heads run as two streams over the same key
// and value tiles, each with its own Q tile, S slot, O accumulator and softmax
// warpgroup; each K and V tile is loaded once for both.  TMEM: S of the first head in
// columns [0, 128), of the second in [128, 256), their O in [256, 384) and [384, 512).
//   warp 0     TMA producer: per stream a Q tile per unit; K and V tiles per item into
//              2-slot rings (a slot is reloaded when both streams are done with it).
//   warp 1     MMA issuer in a fixed order, PV0(n), S0(n + 1), PV1(n), S1(n + 1), with
//              blocking bounded waits (the whole warp waits, the elected lane issues):
//              S(n) of a stream needs its Q, K(n) and its previous PV complete (P of the
//              previous item sits in the S slot); PV(n) needs the stream's softmax of item
//              n, V(n) and, on a unit's first item, the stream's previous O read out.  An
//              issuer that polled both streams instead reacted 600-1,150 cycles late and
//              was slower than the one-stream kernel (553 vs 501 us on the Qwen3 shape);
//              with PV0, PV1 before S0, S1 it took 521 us; this order takes 463 us.
//   warps 2-5  softmax of the first head, warps 6-9 of the second (thread = query row);
//              after a unit's last item the warpgroup writes O / l and frees O.
// One head's softmax overlaps the other head's MMAs and softmax: two items are in
// flight per SM where the one-stream kernel has one.
namespace pairk {
constexpr int kWarps = 10;
constexpr int kThreads = 32 * kWarps;
constexpr int HDP = 128;
constexpr uint32_t TILE = 2 * BOX_BYTES;  // 128 rows x 128 bf16, two 64-column boxes
constexpr int KVS = 2;
constexpr uint32_t SMEM = 1024 + 2 * TILE + 2 * KVS * TILE + WBAR_BYTES + 4 * (kMaxBatchW + 1) + 64;
static_assert(SMEM <= 227 * 1024, "shared memory budget");
}  // namespace pairk

__global__ void __launch_bounds__(pairk::kThreads, 1)
    attn_pair_tcgen05(const __grid_constant__ CUtensorMap tm_qkv, const int32_t *__restrict__ cu_seqlens, int batch,
                      int q_heads, int kv_heads, int causal, float scale_log2, __nv_bfloat16 *__restrict__ out,
                      int *status)
{
    using namespace pairk;
    constexpr int HD = HDP;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem;               // [2 streams]
    uint8_t *sK = sQ + 2 * TILE;      // [KVS]
    uint8_t *sV = sK + KVS * TILE;    // [KVS]
    uint64_t *bars = reinterpret_cast<uint64_t *>(sV + KVS * TILE);
    uint64_t *q_full = bars;              // [2]
    uint64_t *q_empty = q_full + 2;       // [2]
    uint64_t *k_full = q_empty + 2;       // [KVS]
    uint64_t *k_empty = k_full + KVS;     // [KVS] one commit per stream's S
    uint64_t *v_full = k_empty + KVS;     // [KVS]
    uint64_t *v_empty = v_full + KVS;     // [KVS] one commit per stream's PV
    uint64_t *s_full = v_empty + KVS;     // [2]
    uint64_t *p_full = s_full + 2;        // [2] one arrival per softmax warp of the stream
    uint64_t *pv_done = p_full + 2;       // [2]
    uint64_t *o_free = pv_done + 2;       // [2] one arrival per softmax warp of the stream
    uint64_t *probe = o_free + 2;         // [1]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(probe + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *warp_tot = reinterpret_cast<int *>(tmem_slot + 2);
    int *upre = reinterpret_cast<int *>(reinterpret_cast<uint8_t *>(bars) + WBAR_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int group = q_heads / kv_heads;
    const int npairs = group / 2;
    const int k_col0 = q_heads * HD, v_col0 = (q_heads + kv_heads) * HD;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 4);
            mbar_init(&pv_done[i], 1);
            mbar_init(&o_free[i], 4);
        }
        for (int i = 0; i < KVS; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 2);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 2);
        }
        mbar_init(probe, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tm_qkv);
    }
    grid_dep_wait();
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    // upre[s] = units of the sentences before s (query tiles x key-value heads x head pairs)
    {
        int carry = 0;
        for (int c0 = 0; c0 < batch; c0 += kThreads) {
            const int i = c0 + threadIdx.x;
            int v = 0;
            if (i < batch) v = ((cu_seqlens[i + 1] - cu_seqlens[i] + TQ - 1) / TQ) * kv_heads * npairs;
            int x = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            if (lane == 31) warp_tot[warp] = x;
            __syncthreads();
            int off = carry, total = 0;
#pragma unroll
            for (int w2 = 0; w2 < kWarps; ++w2) {
                if (w2 < warp) off += warp_tot[w2];
                total += warp_tot[w2];
            }
            if (i < batch) upre[i + 1] = off + x;
            carry += total;
            __syncthreads();
        }
        if (threadIdx.x == 0) upre[0] = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    grid_dep_launch();
    const uint32_t tmem = *tmem_slot;
    const int total_units = upre[batch];

    struct U {
        int start, len, q0, kvh, qh0, n_kv;
    };
    auto unit = [&](int g) -> U {
        int lo = 0, hi = batch - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (upre[mid] <= g) lo = mid;
            else hi = mid - 1;
        }
        const int rr = g - upre[lo];
        const int per_tile = kv_heads * npairs;
        const int t = rr / per_tile;
        const int rem = rr - t * per_tile;
        U w;
        w.start = cu_seqlens[lo];
        w.len = cu_seqlens[lo + 1] - w.start;
        w.kvh = rem / npairs;
        w.qh0 = w.kvh * group + 2 * (rem - w.kvh * npairs);
        w.q0 = t * TQ;
        const int nk = (w.len + TK - 1) / TK;
        w.n_kv = causal ? min(nk, t + 1) : nk;
        return w;
    };
    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (mbar_wait(bar, parity)) return true;
        report(status, DEV_TIMEOUT);
        *abort_flag = 1;
        return false;
    };
    // a polled barrier, decided once for the whole warp (lane 0's view)
    auto ready = [&](uint64_t *bar, uint32_t parity) -> bool {
        const uint32_t r = mbar_test_wait(bar, parity) ? 1u : 0u;
        return __shfl_sync(0xffffffffu, r, 0) != 0;
    };

    if (warp == 0) {
        // ------------------------------------------------ TMA producer (whole warp polls)
        const bool leader = elect_lane();
        struct Cur {
            int g, j;
            U w;
        };
        auto start_at = [&](Cur &c, int g) {
            c.g = g;
            c.j = 0;
            if (g < total_units) c.w = unit(g);
        };
        auto advance = [&](Cur &c) {
            if (++c.j == c.w.n_kv) start_at(c, c.g + static_cast<int>(gridDim.x));
        };
        Cur kc, vc;
        start_at(kc, blockIdx.x);
        start_at(vc, blockIdx.x);
        int qg[2] = {static_cast<int>(blockIdx.x), static_cast<int>(blockIdx.x)};
        uint32_t qn[2] = {0, 0}, kn = 0, vn = 0;
        uint32_t q_armed = 0, k_armed = 0, k_par = 0, v_armed = 0, v_par = 0;
        bool ok = true;
        uint64_t t_last = __shfl_sync(0xffffffffu, globaltimer_ns(), 0);
        for (uint32_t i = 0; ok && !*abort_flag; ++i) {
            const bool k_more = kc.g < total_units, v_more = vc.g < total_units;
            if (!k_more && !v_more && qg[0] >= total_units && qg[1] >= total_units) break;
            bool progress = false;
            for (int s = 0; s < 2; ++s) {
                if (qg[s] >= total_units) continue;
                if (!ready(&q_empty[s], (qn[s] & 1) ^ 1)) continue;
                const U w = unit(qg[s]);
                if (leader) {
                    mbar_arrive_expect_tx(&q_full[s], TILE);
                    for (int b = 0; b < 2; ++b)
                        tma_load_2d(sQ + s * TILE + b * BOX_BYTES, &tm_qkv, &q_full[s], (w.qh0 + s) * HD + 64 * b,
                                    w.start + w.q0);
                }
                q_armed |= 1u << s;
                ++qn[s];
                qg[s] += gridDim.x;
                progress = true;
            }
            if (k_more) {
                const int ks = kn % KVS;
                if (ready(&k_empty[ks], ((kn / KVS) & 1) ^ 1)) {
                    if (leader) {
                        mbar_arrive_expect_tx(&k_full[ks], TILE);
                        for (int b = 0; b < 2; ++b)
                            tma_load_2d(sK + ks * TILE + b * BOX_BYTES, &tm_qkv, &k_full[ks],
                                        k_col0 + kc.w.kvh * HD + 64 * b, kc.w.start + kc.j * TK);
                    }
                    k_armed |= 1u << ks;
                    k_par = (k_par & ~(1u << ks)) | (((kn / KVS) & 1) << ks);
                    ++kn;
                    advance(kc);
                    progress = true;
                }
            }
            if (v_more && vn < kn) {
                const int vs = vn % KVS;
                if (ready(&v_empty[vs], ((vn / KVS) & 1) ^ 1)) {
                    if (leader) {
                        mbar_arrive_expect_tx(&v_full[vs], TILE);
                        for (int b = 0; b < 2; ++b)
                            tma_load_2d(sV + vs * TILE + b * BOX_BYTES, &tm_qkv, &v_full[vs],
                                        v_col0 + vc.w.kvh * HD + 64 * b, vc.w.start + vc.j * TK);
                    }
                    v_armed |= 1u << vs;
                    v_par = (v_par & ~(1u << vs)) | (((vn / KVS) & 1) << vs);
                    ++vn;
                    advance(vc);
                    progress = true;
                }
            }
            if (progress) {
                t_last = __shfl_sync(0xffffffffu, globaltimer_ns(), 0);
            } else {
                __nanosleep(32);
                const uint64_t now = __shfl_sync(0xffffffffu, globaltimer_ns(), 0);
                if (((i & 255u) == 255u || wait_limit_ns() < kShortWaitNs) && now - t_last > wait_limit_ns()) {
                    report(status, DEV_TIMEOUT);
                    *abort_flag = 1;
                    ok = false;
                }
            }
        }
        // every load this warp started lands before the CTA exits
        for (int s = 0; s < 2; ++s)
            if ((q_armed >> s) & 1) (void)mbar_wait_drain(&q_full[s], (qn[s] - 1) & 1);
        for (int i = 0; i < KVS; ++i) {
            if ((k_armed >> i) & 1) (void)mbar_wait_drain(&k_full[i], (k_par >> i) & 1);
            if ((v_armed >> i) & 1) (void)mbar_wait_drain(&v_full[i], (v_par >> i) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (blocking waits, fixed order)
        // Both streams walk the same units and items.  Per item n: PV0(n), S0(n + 1), PV1(n),
        // S1(n + 1): while one head's softmax runs, the other head's PV and next S are issued,
        // so the two streams settle half a step apart.  Every wait is a bounded blocking wait.
        const bool leader = elect_lane();
        constexpr uint32_t idesc_o = idesc_bf16_f32(TQ, HD, false, true);
        bool issued = false;
        auto issue_s = [&](int s, uint32_t nn, int jj, const U &ww, uint32_t uu) -> bool {
            const int slot = nn % KVS;
            if (!wait(&k_full[slot], (nn / KVS) & 1)) return false;
            if (jj == 0 && !wait(&q_full[s], uu & 1)) return false;
            if (nn > 0 && !wait(&pv_done[s], (nn - 1) & 1)) return false;  // P of item nn - 1 consumed
            tc_fence_after();
            const int valid = min(TK, ww.len - jj * TK);
            const int n16 = min(TK, max(16, (valid + 15) & ~15));
            const uint32_t idesc_s = idesc_bf16_f32(TQ, n16, false, false);
            const uint32_t qa = smem_u32(sQ + s * TILE), ka = smem_u32(sK + slot * TILE);
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {  // 4 K steps per 128-byte swizzle atom, then the next box
                const uint32_t off = (kk >> 2) * BOX_BYTES + (kk & 3) * 32;
                if (leader)
                    umma_f16_ss(tmem + s * 128, sdesc_sw128(qa + off, 16, 1024), sdesc_sw128(ka + off, 16, 1024),
                                idesc_s, kk != 0 ? 1u : 0u);
            }
            issued = true;
            if (leader) {
                umma_commit(&s_full[s]);
                umma_commit(&k_empty[slot]);
                if (jj == ww.n_kv - 1) umma_commit(&q_empty[s]);
            }
            return true;
        };
        auto issue_pv = [&](int s, uint32_t nn, int jj, const U &ww, uint32_t uu) -> bool {
            const int slot = nn % KVS;
            if (!wait(&p_full[s], nn & 1)) return false;
            if (!wait(&v_full[slot], (nn / KVS) & 1)) return false;
            if (jj == 0 && uu > 0 && !wait(&o_free[s], (uu - 1) & 1)) return false;
            tc_fence_after();
            const int valid = min(TK, ww.len - jj * TK);
            const uint64_t v_desc = sdesc_sw128(smem_u32(sV + slot * TILE), BOX_BYTES, 1024);
            const uint32_t o_tmem = tmem + 256 + s * HD;
            const int nks = (valid + 15) >> 4;
            for (int ks = 0; ks < nks; ++ks)
                if (leader)
                    umma_f16_ts(o_tmem, tmem + s * 128 + ks * 8, v_desc + static_cast<uint64_t>(ks * 128), idesc_o,
                                (jj == 0 && ks == 0) ? 0u : 1u);
            if (leader) {
                umma_commit(&pv_done[s]);
                umma_commit(&v_empty[slot]);
            }
            return true;
        };
        int g = blockIdx.x, j = 0;
        uint32_t n = 0, u = 0;
        U w;
        bool ok = g < total_units;
        if (ok) {
            w = unit(g);
            ok = issue_s(0, 0, 0, w, 0) && issue_s(1, 0, 0, w, 0);
        }
        while (ok && !*abort_flag) {
            int j2 = j + 1, g2 = g;
            uint32_t u2 = u;
            U w2 = w;
            if (j2 == w.n_kv) {
                j2 = 0;
                g2 += gridDim.x;
                ++u2;
                if (g2 < total_units) w2 = unit(g2);
            }
            const bool more = g2 < total_units;
            ok = issue_pv(0, n, j, w, u) && (!more || issue_s(0, n + 1, j2, w2, u2)) && issue_pv(1, n, j, w, u) &&
                 (!more || issue_s(1, n + 1, j2, w2, u2));
            if (!more) break;
            ++n;
            j = j2;
            g = g2;
            u = u2;
            w = w2;
        }
        if (issued) {
            if (leader) umma_commit(probe);
            (void)mbar_wait_drain(probe, 0);
        }
    } else {
        // ------------------------------------------------ softmax warpgroups (warps 2-5, 6-9)
        const int s = (warp - 2) >> 2;  // stream: the pair's first or second head
        const int q = warp & 3;         // TMEM lane quarter
        const int r = q * 32 + lane;    // query row within the tile == TMEM lane
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        const uint32_t tS = tmem + lane_base + s * 128;
        const uint32_t tO = tmem + lane_base + 256 + s * HD;
        uint32_t n = 0;
        bool ok = true;
        for (int g = blockIdx.x; g < total_units && ok; g += gridDim.x) {
            if (*abort_flag) break;
            const U w = unit(g);
            const bool warp_live = w.q0 + q * 32 < w.len;
            const int qi = w.q0 + r;  // this thread's query position in the sentence
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < w.n_kv; ++j) {
                if (!(ok = wait(&s_full[s], n & 1))) break;
                tc_fence_after();
                const int valid = min(TK, w.len - j * TK);
                // keys kept for this row: c < lim (key position j * 128 + c)
                const int lim = causal ? min(valid, qi - j * TK + 1) : valid;
                float alpha = 1.f, rs = 0.f, mx = m_run;
                if (warp_live) {
                    float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                    for (int c = 0; c < valid; c += 32) {
                        uint32_t v[32];
                        tmem_ld_x32(tS + c, v);
                        tmem_wait_ld_regs(v);
                        if (c + 32 <= lim) {  // no masked key in the chunk (all but the row's last)
#pragma unroll
                            for (int i = 0; i < 32; i += 2)
                                m4[(i >> 1) & 3] = max3f(m4[(i >> 1) & 3], __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (c + i < lim) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(v[i]));
                        }
                    }
                    const float tmax = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * scale_log2;
                    // lazy reference max, as in the one-stream kernel: raised only when a tile's max
                    // exceeds it by more than 8, so O is rescaled only then
                    if (m_run == -INFINITY || tmax > m_run + 8.0f) mx = fmaxf(m_run, tmax);
                    alpha = mx == m_run ? 1.f : (m_run == -INFINITY ? 0.f : fast_exp2w(m_run - mx));
                    const float msub = mx == -INFINITY ? 0.f : mx;
                    float rs0 = 0.f, rs1 = 0.f;
                    for (int c = 0; c < valid; c += 32) {
                        uint32_t v[32];
                        tmem_ld_x32(tS + c, v);
                        tmem_wait_ld_regs(v);
                        uint32_t pk[16];
                        if (c + 32 <= lim) {
#pragma unroll
                            for (int i = 0; i < 16; ++i) {  // packed f32x2: scale and shift, then row sums
                                float p0, p1;
                                fma_f32x2(p0, p1, __uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]), scale_log2,
                                          -msub);
                                p0 = fast_exp2w(p0);
                                p1 = fast_exp2w(p1);
                                add_f32x2(rs0, rs1, p0, p1);
                                pk[i] = pack_bf16x2(p0, p1);
                            }
                        } else if (c >= lim) {  // every key of the chunk masked
#pragma unroll
                            for (int i = 0; i < 16; ++i) pk[i] = 0u;
                        } else {
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const float p0 =
                                    c + 2 * i < lim ? fast_exp2w(fmaf(__uint_as_float(v[2 * i]), scale_log2, -msub)) : 0.f;
                                const float p1 = c + 2 * i + 1 < lim
                                                     ? fast_exp2w(fmaf(__uint_as_float(v[2 * i + 1]), scale_log2, -msub))
                                                     : 0.f;
                                rs0 += p0;
                                rs1 += p1;
                                pk[i] = pack_bf16x2(p0, p1);
                            }
                        }
                        tmem_st_x16(tS + (c >> 1), pk);
                    }
                    rs = rs0 + rs1;
                    tmem_wait_st();
                }
                // O *= alpha before this item's PV accumulates (needs the previous PV done)
                if (j > 0 && warp_live && __any_sync(0xffffffffu, alpha != 1.f)) {
                    if (!(ok = wait(&pv_done[s], (n - 1) & 1))) break;
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < HD; c += 32) {
                        uint32_t v[32];
                        tmem_ld_x32(tO + c, v);
                        tmem_wait_ld_regs(v);
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
                        tmem_st_x32(tO + c, v);
                    }
                    tmem_wait_st();
                }
                l_run = l_run * alpha + rs;
                m_run = mx;
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[s]);
                ++n;
            }
            if (!ok) break;
            // the unit's last PV, then O / l out and the accumulator released
            if (!(ok = wait(&pv_done[s], (n - 1) & 1))) break;
            tc_fence_after();
            if (warp_live) {
                const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
                const bool row_ok = qi < w.len;
                __nv_bfloat16 *dst = out + static_cast<size_t>(w.start + qi) * (q_heads * HD) + (w.qh0 + s) * HD;
#pragma unroll 1
                for (int c = 0; c < HD; c += 32) {
                    uint32_t v[32];
                    tmem_ld_x32(tO + c, v);
                    tmem_wait_ld_regs(v);
                    if (row_ok) {
                        uint4 *d4 = reinterpret_cast<uint4 *>(dst + c);
#pragma unroll
                        for (int x = 0; x < 4; ++x)
                            d4[x] = make_uint4(pack_bf16x2(__uint_as_float(v[8 * x + 0]) * inv, __uint_as_float(v[8 * x + 1]) * inv),
                                               pack_bf16x2(__uint_as_float(v[8 * x + 2]) * inv, __uint_as_float(v[8 * x + 3]) * inv),
                                               pack_bf16x2(__uint_as_float(v[8 * x + 4]) * inv, __uint_as_float(v[8 * x + 5]) * inv),
                                               pack_bf16x2(__uint_as_float(v[8 * x + 6]) * inv, __uint_as_float(v[8 * x + 7]) * inv));
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free[s]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

cudaError_t launch_pair(const CUtensorMap &tm, const int32_t *cu, int batch, int q_heads, int kv_heads, int causal,
                        float scale_log2, __nv_bfloat16 *out, int grid, cudaStream_t s)
{
    static uint64_t configured[64] = {};  // context the attribute was set in
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t ctx = current_context_id();
    if (dev < 64 && configured[dev] != ctx) {
        cudaError_t e = cudaFuncSetAttribute(attn_pair_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             pairk::SMEM);
        if (e != cudaSuccess) return e;
        configured[dev] = ctx;
    }
    return launch_k(attn_pair_tcgen05, dim3(grid), dim3(pairk::kThreads), pairk::SMEM, s, tm, cu, batch, q_heads,
                    kv_heads, causal, scale_log2, out, current_device_status_word());
}

// FE_ATTN_PAIR=0 keeps head_dim 128 GQA on the one-stream kernel (diagnostic).
bool pair_kernel_enabled()
{
    static const bool on = [] {
        const char *v = getenv("FE_ATTN_PAIR");
        return !(v && v[0] == '0');
    }();
    return on;
}

template <int HD>
cudaError_t launch_wide(const CUtensorMap &tm, const int32_t *cu, int batch, int q_heads, int kv_heads, int causal,
                        float scale_log2, __nv_bfloat16 *out, int grid, cudaStream_t s)
{
    static uint64_t configured[64] = {};  // context the attribute was set in
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t ctx = current_context_id();
    if (dev < 64 && configured[dev] != ctx) {
        cudaError_t e = cudaFuncSetAttribute(attn_wide_tcgen05<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             WCfg<HD>::SMEM);
        if (e != cudaSuccess) return e;
        configured[dev] = ctx;
    }
    return launch_k(attn_wide_tcgen05<HD>, dim3(grid), dim3(kThreadsW), WCfg<HD>::SMEM, s, tm, cu, batch, q_heads,
                    kv_heads, causal, scale_log2, out, current_device_status_word());
}

}  // namespace

cudaError_t launch_attention_wide(const void *qkv, const int32_t *cu_seqlens, int batch, int max_len, int q_heads,
                                  int kv_heads, int head_dim, bool causal, float scale, void *out,
                                  int64_t total_tokens, cudaStream_t s, fe_status *st)
{
    *st = FE_OK;
    if (batch == 0 || max_len == 0 || total_tokens == 0) return cudaSuccess;
    const int64_t width = static_cast<int64_t>(q_heads + 2 * kv_heads) * head_dim;
    CUtensorMap tm;
    fe_status r = make_tmap_2d(&tm, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, total_tokens, width, width, 128, 64);
    if (r != FE_OK) {
        *st = r;
        return cudaSuccess;
    }
    const float scale_log2 = scale * 1.4426950408889634f;
    const int sms = current_sm_count();
    for (int b0 = 0; b0 < batch; b0 += kMaxBatchW) {
        const int nb = batch - b0 < kMaxBatchW ? batch - b0 : kMaxBatchW;
        const int64_t units_bound = static_cast<int64_t>(nb) * ((max_len + TQ - 1) / TQ) * q_heads;
        const int grid = units_bound < sms ? static_cast<int>(units_bound) : sms;
        auto *o = static_cast<__nv_bfloat16 *>(out);
        if (head_dim == 128 && (q_heads / kv_heads) % 2 == 0 && pair_kernel_enabled()) {
            const int64_t pair_units = units_bound / 2;
            const int pgrid = pair_units < sms ? static_cast<int>(pair_units) : sms;
            cudaError_t e = launch_pair(tm, cu_seqlens + b0, nb, q_heads, kv_heads, causal ? 1 : 0, scale_log2, o, pgrid, s);
            if (e != cudaSuccess) return e;
            continue;
        }
        cudaError_t e = head_dim == 128
                            ? launch_wide<128>(tm, cu_seqlens + b0, nb, q_heads, kv_heads, causal ? 1 : 0, scale_log2,
                                               o, grid, s)
                            : launch_wide<256>(tm, cu_seqlens + b0, nb, q_heads, kv_heads, causal ? 1 : 0, scale_log2,
                                               o, grid, s);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace fe

namespace fe {
cudaError_t set_wait_limit_attention_wide(uint64_t ns) { return set_wait_limit_this_file(ns); }
}  // namespace fe
