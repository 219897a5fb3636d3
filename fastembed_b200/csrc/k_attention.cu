// k_attention.cu — variable-length bidirectional attention on tcgen05 (head_dim 64).
//
// Replaces the QK^T / softmax / PV stage of CUDAAttentionOps::multi_head_attention
// (src/ops/cuda/cuda_attention_ops.cu:264-313: permute, batched QK^T, scaled softmax,
// batched PV, unpermute) for a packed batch of unpadded sentences.  Its semantics are
// the CPU reference's per-sentence attention (src/ops/cpu/cpu_attention_ops.cpp:33-85):
// softmax(Q K^T / sqrt(hd)) V with keys limited to the sentence, i.e. a key-padding
// mask over a padded batch.
//
// Persistent and warp-specialised, two CTAs per SM, each an independent pipeline.  A
// work unit is (sentence, 128-row query tile, head); an item is one 128-key tile of a
// unit.  At start every CTA builds, in shared memory, the list of its units
// (blockIdx.x, +gridDim.x, ...) whose query tile starts inside the sentence.
//   warp 0     TMA producer: Q tile per unit and K/V tiles per item into 2-slot rings,
//              straight from the QKV buffer (no permute).  (An L2 prefetch of the tiles of
//              the units grabbed ahead measured 10-12 % slower and was removed.)
//   warp 1     TMEM owner + MMA issuer: S = Q K^T (M=128, N = keys rounded up to 16) into
//              one of two 128-column TMEM slots; for the previous item, O = P V with P
//              read from TMEM (A operand), V as an MN-major smem operand, O written into
//              the upper 64 columns of P's slot.
//   warps 2-5  softmax: thread = query row; reads its S row (tcgen05.ld), masks keys past
//              the sentence end, online max / sum, writes P (bf16) back over the first 64
//              columns (tcgen05.st) and the row's rescale factor and running sum into
//              shared memory.
//   warps 6-9  O fold: thread = query row; once an item's PV is done, reads its 64 O
//              columns from TMEM into fp32 registers (o = o * alpha + O), hands the slot
//              back to the MMA warp, and after a unit's last item stores O / l.
// A slot turns over as S -> softmax -> PV -> fold.  With the fold on warps of its own, the
// softmax warps go on to the other slot's S while this slot's PV and fold run, so neither
// the S latency nor the fold sits between two softmax passes (when the softmax warps also
// folded, each item cost the S latency + softmax + fold in a row).
// K and V tiles have separate full / empty barriers: a K slot is reloaded as soon as
// the S two items back is done with it, without waiting for that item's PV.
// Waits are bounded; on timeout the CTA records FE_ERR_DEVICE_TIMEOUT, drains what it
// started and exits.
#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>

#include "fe_common.cuh"
#include "fe_internal.h"

namespace fe {
namespace {

constexpr int HD = 64;
constexpr int TQ = 128;
constexpr int TK = 128;
constexpr int Q_SLOTS = 2;
constexpr int KV_SLOTS = 2;
constexpr int kLookahead = 2;                   // units grabbed ahead of the loads
constexpr int kRing = 8;                        // grabbed units in flight to the MMA, softmax and fold warps
constexpr int kMaxBatch = 2048;                 // sentences per launch (prefix table in shared memory)
constexpr int kCtasPerSm = 2;
constexpr int kSchedSlots = 64;                 // work counters, one per launch in flight
constexpr uint32_t Q_BYTES = TQ * HD * 2;       // 16 KB
constexpr uint32_t KV_BYTES = 2 * TK * HD * 2;  // K then V, 32 KB
constexpr uint32_t BAR_BYTES = 512;
constexpr uint32_t ROW_BYTES = 2 * 2 * TQ * 4;  // per slot and query row: rescale factor, running sum
constexpr uint32_t SMEM_BYTES =
    1024 + Q_SLOTS * Q_BYTES + KV_SLOTS * KV_BYTES + BAR_BYTES + 16 * kRing + ROW_BYTES + 4 * (kMaxBatch + 1) + 64;
constexpr uint32_t TMEM_COLS = 256;  // two slots: S [0,128) -> P [0,64) + O [64,128)
constexpr int kThreads = 320;

// 32 lanes x 32 bit, 8 consecutive columns: thread i of the warp receives lane
// (lane base of taddr + i), columns [col, col + 8).
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t (&r)[8])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

struct Unit {
    int start, len, q0, head, n_kv;
};

// Per-launch work counters: [2 * slot] = next unit to hand out, [2 * slot + 1] = CTAs
// finished; the last CTA of a launch sets both back to zero.
__device__ unsigned g_attn_sched[2 * kSchedSlots];

// A unit as passed through the ring: {first row of the sentence, sentence length (-1:
// no more units), (head << 8) | query tile}.
__device__ __forceinline__ Unit unit_of(const int4 e)
{
    Unit w;
    w.start = e.x;
    w.len = e.y;
    w.head = e.z >> 8;
    w.q0 = (e.z & 255) * TQ;
    w.n_kv = (w.len + TK - 1) / TK;
    return w;
}

__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    attn_varlen_tcgen05(const __grid_constant__ CUtensorMap tm_qkv, const int32_t *__restrict__ cu_seqlens,
                        int batch, int heads, unsigned *sched, __nv_bfloat16 *__restrict__ out, float scale_log2,
                        int total_tokens, int head_major, int *status)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem;
    uint8_t *sKV = sQ + Q_SLOTS * Q_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sKV + KV_SLOTS * KV_BYTES);
    uint64_t *q_full = bars;                  // [Q_SLOTS]
    uint64_t *q_empty = q_full + Q_SLOTS;     // [Q_SLOTS]
    uint64_t *k_full = q_empty + Q_SLOTS;     // [KV_SLOTS] K tile landed
    uint64_t *k_empty = k_full + KV_SLOTS;    // [KV_SLOTS] S MMAs done with the K tile
    uint64_t *v_full = k_empty + KV_SLOTS;    // [KV_SLOTS] V tile landed
    uint64_t *v_empty = v_full + KV_SLOTS;    // [KV_SLOTS] PV MMAs done with the V tile
    uint64_t *s_full = v_empty + KV_SLOTS;    // [2] S of a slot ready
    uint64_t *p_full = s_full + 2;            // [2] P of a slot written
    uint64_t *o_full = p_full + 2;            // [2] O of a slot ready
    uint64_t *slot_free = o_full + 2;         // [2] O of a slot consumed
    uint64_t *probe = slot_free + 2;          // [1]
    uint64_t *unit_full = probe + 1;          // [kRing] a grabbed unit is in the ring slot
    uint64_t *unit_empty = unit_full + kRing; // [kRing] the MMA, softmax and fold warps have read it
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(unit_empty + kRing);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *warp_tot = reinterpret_cast<int *>(tmem_slot + 2);  // [kThreads / 32]
    // ring entries are written before an mbarrier arrive and read after the matching wait
    int4 *ring = reinterpret_cast<int4 *>(reinterpret_cast<uint8_t *>(bars) + BAR_BYTES);
    // per slot and query row, written by the softmax warp before its p_full arrive and read
    // by the fold warp after waiting on the same p_full phase
    float *row_alpha = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(bars) + BAR_BYTES + 16 * kRing);  // [2][TQ]
    float *row_l = row_alpha + 2 * TQ;                                                                     // [2][TQ]
    int *upre = reinterpret_cast<int *>(reinterpret_cast<uint8_t *>(bars) + BAR_BYTES + 16 * kRing + ROW_BYTES);  // [batch + 1]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int dim = heads * HD;

    if (threadIdx.x == 0) {
        for (int i = 0; i < Q_SLOTS; ++i) {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], 1);
        }
        for (int i = 0; i < KV_SLOTS; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 4);     // one arrival per softmax warp
            mbar_init(&o_full[i], 1);
            mbar_init(&slot_free[i], 4);  // one arrival per fold warp
        }
        mbar_init(probe, 1);
        for (int i = 0; i < kRing; ++i) {
            mbar_init(&unit_full[i], 1);
            mbar_init(&unit_empty[i], 9);  // one arrival from the MMA warp, one per softmax and fold warp
        }
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tm_qkv);
    }
    grid_dep_wait();
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }

    // Units are handed out dynamically, in the order (sentence, query tile, head), from the
    // launch's work counter.  upre[s] = number of units of sentences before s (each has
    // ceil(len / 128) query tiles x heads units), so a unit index maps to its sentence by
    // binary search.
    {
        constexpr int nwarps = kThreads / 32;
        int carry = 0;
        for (int c0 = 0; c0 < batch; c0 += kThreads) {
            const int i = c0 + threadIdx.x;
            int v = 0;
            if (i < batch) v = ((cu_seqlens[i + 1] - cu_seqlens[i] + TQ - 1) / TQ) * heads;
            int x = v;  // inclusive warp scan
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
    const unsigned total_units = static_cast<unsigned>(upre[batch]);

    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (mbar_wait(bar, parity)) return true;
        report(status, DEV_TIMEOUT);
        *abort_flag = 1;
        return false;
    };
    // Tile `which` (0 = Q, 1 = K, 2 = V) of `head`, rows [row, row + 128): one 128-byte
    // row per token in the token-major layout, or a contiguous 16 KB block head-major.
    auto load_tile = [&](void *dst, uint64_t *bar, int which, int head, int row) {
        if (head_major) tma_load_3d(dst, &tm_qkv, bar, 0, row, which * heads + head);
        else tma_load_2d(dst, &tm_qkv, bar, which * dim + head * HD, row);
    };

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer + unit scheduler
            // Loads run in the order the MMA warp consumes them: a unit's Q, then per item its
            // K followed by the previous item's V (whose PV is issued after this item's S), so
            // neither the next K nor the next unit's Q waits behind a V slot.
            uint32_t qn = 0, kn = 0, vn = 0;
            uint32_t q_armed = 0, k_armed = 0, v_armed = 0, q_par = 0, k_par = 0, v_par = 0;
            bool ok = true;
            uint32_t grabbed = 0, loaded = 0;  // units pushed into the ring / whose tiles were loaded
            bool grab_done = false;
            // The next unit index is fetched one grab ahead, so the atomic's round trip
            // overlaps the loads instead of delaying the next unit's Q.
            unsigned ticket = atomicAdd(&sched[0], 1u);
            // Takes the ticketed unit of the launch (or, past the last one, the end marker),
            // pushes it into the ring.
            auto grab = [&]() -> bool {
                const unsigned g = ticket;
                int4 e = make_int4(0, -1, 0, 0);
                if (g < total_units) {
                    ticket = atomicAdd(&sched[0], 1u);
                    int lo = 0, hi = batch - 1;  // last sentence s with upre[s] <= g
                    while (lo < hi) {
                        const int mid = (lo + hi + 1) >> 1;
                        if (upre[mid] <= static_cast<int>(g)) lo = mid;
                        else hi = mid - 1;
                    }
                    const int rr = static_cast<int>(g) - upre[lo];
                    const int st = cu_seqlens[lo];
                    e = make_int4(st, cu_seqlens[lo + 1] - st, ((rr % heads) << 8) | (rr / heads), 0);
                }
                const int slot = grabbed % kRing;
                if (!wait(&unit_empty[slot], ((grabbed / kRing) & 1) ^ 1)) return false;
                ring[slot] = e;
                mbar_arrive(&unit_full[slot]);
                ++grabbed;
                if (e.y < 0) grab_done = true;
                return true;
            };
            // V of item vn (head, first key row) into the V half of its K/V slot
            auto load_v = [&](int head, int row) -> bool {
                const int vs = vn % KV_SLOTS;
                if (!wait(&v_empty[vs], ((vn / KV_SLOTS) & 1) ^ 1)) return false;
                mbar_arrive_expect_tx(&v_full[vs], KV_BYTES / 2);
                load_tile(sKV + vs * KV_BYTES + KV_BYTES / 2, &v_full[vs], 2, head, row);
                v_armed |= 1u << vs;
                v_par = (v_par & ~(1u << vs)) | (((vn / KV_SLOTS) & 1) << vs);
                ++vn;
                return true;
            };
            bool have_v = false;
            int v_head = 0, v_row = 0;
            while (ok && !*abort_flag) {
                while (ok && !grab_done && grabbed < loaded + kLookahead) ok = grab();
                if (!ok || loaded == grabbed) break;
                const int4 e = ring[loaded % kRing];
                ++loaded;
                if (e.y < 0) break;
                const Unit w = unit_of(e);
                const int qs = qn % Q_SLOTS;
                if (!(ok = wait(&q_empty[qs], ((qn / Q_SLOTS) & 1) ^ 1))) break;
                mbar_arrive_expect_tx(&q_full[qs], Q_BYTES);
                load_tile(sQ + qs * Q_BYTES, &q_full[qs], 0, w.head, w.start + w.q0);
                q_armed |= 1u << qs;
                q_par = (q_par & ~(1u << qs)) | (((qn / Q_SLOTS) & 1) << qs);
                ++qn;
                for (int j = 0; j < w.n_kv; ++j) {
                    // K as soon as the S of two items back is done with the slot
                    const int ks = kn % KV_SLOTS;
                    if (!(ok = wait(&k_empty[ks], ((kn / KV_SLOTS) & 1) ^ 1))) break;
                    mbar_arrive_expect_tx(&k_full[ks], KV_BYTES / 2);
                    load_tile(sKV + ks * KV_BYTES, &k_full[ks], 1, w.head, w.start + j * TK);
                    k_armed |= 1u << ks;
                    k_par = (k_par & ~(1u << ks)) | (((kn / KV_SLOTS) & 1) << ks);
                    ++kn;
                    // then the previous item's V, once the PV two items back is done with its slot
                    if (have_v && !(ok = load_v(v_head, v_row))) break;
                    have_v = true;
                    v_head = w.head;
                    v_row = w.start + j * TK;
                }
            }
            if (ok && have_v && !*abort_flag) (void)load_v(v_head, v_row);
            // every load this thread started lands before the CTA exits
            for (int i = 0; i < Q_SLOTS; ++i)
                if ((q_armed >> i) & 1) (void)mbar_wait_drain(&q_full[i], (q_par >> i) & 1);
            for (int i = 0; i < KV_SLOTS; ++i) {
                if ((k_armed >> i) & 1) (void)mbar_wait_drain(&k_full[i], (k_par >> i) & 1);
                if ((v_armed >> i) & 1) (void)mbar_wait_drain(&v_full[i], (v_par >> i) & 1);
            }
        }
    } else if (warp == 1) {
        {
            const bool leader = elect_lane();  // the whole warp waits; this lane issues
            // ------------------------------------------------ MMA issuer
            constexpr uint32_t idesc_o = idesc_bf16_f32(TQ, HD, false, true);
            uint32_t qn = 0, kvn = 0, it = 0;
            bool issued = false, ok = true, have_pend = false;
            uint32_t pend_it = 0, pend_ks = 0, pend_kvn = 0;
            int pend_valid = 0;
            // O(slot) = P(slot) V for item `pit` (P from TMEM, V MN-major from smem)
            auto issue_pv = [&](uint32_t pit, uint32_t pks, uint32_t pkvn, int pvalid) -> bool {
                const uint32_t b = pit & 1;
                if (!wait(&p_full[b], (pit >> 1) & 1)) return false;
                if (!wait(&v_full[pks], (pkvn / KV_SLOTS) & 1)) return false;
                tc_fence_after();
                const uint64_t v_desc = sdesc_sw128(smem_u32(sKV + pks * KV_BYTES + KV_BYTES / 2), TK * 128, 1024);
                const int nks = (pvalid + 15) >> 4;
                for (int ks = 0; ks < nks; ++ks)  // each K step advances 16 key rows = 2048 bytes
                    if (leader) umma_f16_ts(tmem + b * 128 + 64, tmem + b * 128 + ks * 8, v_desc + static_cast<uint64_t>(ks * 128),
                                idesc_o, ks != 0 ? 1u : 0u);
                if (leader) umma_commit(&o_full[b]);
                if (leader) umma_commit(&v_empty[pks]);
                return true;
            };
            for (uint32_t k = 0; ok && !*abort_flag; ++k) {
                const int slot = k % kRing;
                if (!(ok = wait(&unit_full[slot], (k / kRing) & 1))) break;
                const int4 e = ring[slot];
                __syncwarp();  // every lane has read the entry before the slot is handed back
                if (leader) mbar_arrive(&unit_empty[slot]);
                if (e.y < 0) break;
                const Unit w = unit_of(e);
                const int qs = qn % Q_SLOTS;
                if (!(ok = wait(&q_full[qs], (qn / Q_SLOTS) & 1))) break;
                const uint64_t q_desc = sdesc_sw128(smem_u32(sQ + qs * Q_BYTES), 16, 1024);
                for (int j = 0; j < w.n_kv; ++j) {
                    const uint32_t ks = kvn % KV_SLOTS;
                    const uint32_t b = it & 1;
                    if (!(ok = wait(&k_full[ks], (kvn / KV_SLOTS) & 1))) break;
                    if (!(ok = wait(&slot_free[b], ((it >> 1) & 1) ^ 1))) break;
                    tc_fence_after();
                    const int valid = min(TK, w.len - j * TK);
                    const int n = min(TK, max(16, (valid + 15) & ~15));
                    const uint32_t idesc_s = idesc_bf16_f32(TQ, n, false, false);
                    const uint64_t k_desc = sdesc_sw128(smem_u32(sKV + ks * KV_BYTES), 16, 1024);
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk)  // each K step advances 32 bytes inside the swizzle atom
                        if (leader) umma_f16_ss(tmem + b * 128, q_desc + static_cast<uint64_t>(kk * 2),
                                    k_desc + static_cast<uint64_t>(kk * 2), idesc_s, kk != 0 ? 1u : 0u);
                    issued = true;
                    if (leader) umma_commit(&s_full[b]);
                    if (leader) umma_commit(&k_empty[ks]);
                    if (j == w.n_kv - 1 && leader) umma_commit(&q_empty[qs]);
                    if (have_pend && !(ok = issue_pv(pend_it, pend_ks, pend_kvn, pend_valid))) break;
                    have_pend = true;
                    pend_it = it;
                    pend_ks = ks;
                    pend_kvn = kvn;
                    pend_valid = valid;
                    ++it;
                    ++kvn;
                }
                ++qn;
            }
            if (ok && have_pend && !*abort_flag) ok = issue_pv(pend_it, pend_ks, pend_kvn, pend_valid);
            if (issued) {
                // all MMAs issued by this thread retire before TMEM is released
                if (leader) umma_commit(probe);
                (void)mbar_wait_drain(probe, 0);
            }
        }
    } else if (warp < 6) {
        // ------------------------------------------------ softmax warps 2..5
        const int q = warp & 3;
        const int r = q * 32 + lane;  // query row within the tile == TMEM lane
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        uint32_t it = 0;
        bool ok = true;
        for (uint32_t k = 0; ok; ++k) {
            if (*abort_flag) break;
            const int slot = k % kRing;
            if (!(ok = wait(&unit_full[slot], (k / kRing) & 1))) break;
            const int4 e = ring[slot];
            __syncwarp();
            if (lane == 0) mbar_arrive(&unit_empty[slot]);
            if (e.y < 0) break;
            const Unit w = unit_of(e);
            float m_run = -INFINITY, l_run = 0.f;
            // A warp whose 32 query rows all lie past the sentence end does no softmax work:
            // its P and O rows are never read back (each O row depends only on its P row).
            const bool warp_live = w.q0 + q * 32 < w.len;
            for (int j = 0; j < w.n_kv; ++j) {
                const uint32_t b = it & 1;
                if (!(ok = wait(&s_full[b], (it >> 1) & 1))) break;
                tc_fence_after();
                const int valid = min(TK, w.len - j * TK);
                const uint32_t tS = tmem + lane_base + b * 128;
                float mx = m_run, alpha = 1.f, rs0 = 0.f, rs1 = 0.f;
                if (warp_live) {
                    // pass 1: row max of the raw scores (four independent chains)
                    float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                    for (int c = 0; c < valid; c += 32) {
                        uint32_t v[32];
                        tmem_ld_x32(tS + c, v);
                        tmem_wait_ld();
                        if (c + 32 <= valid) {
#pragma unroll
                            for (int i = 0; i < 32; i += 2)
                                m4[(i >> 1) & 3] = max3f(m4[(i >> 1) & 3], __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (c + i < valid) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(v[i]));
                        }
                    }
                    mx = fmaxf(m_run, fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * scale_log2);
                    alpha = fast_exp2(m_run - mx);  // 0 on a unit's first item
                    // pass 2: p = exp2(s * scale - max) in bf16, written back over S as P
                    for (int c = 0; c < valid; c += 32) {
                        uint32_t v[32];
                        tmem_ld_x32(tS + c, v);
                        tmem_wait_ld();
                        uint32_t pk[16];
                        if (c + 32 <= valid) {
#pragma unroll
                            for (int i = 0; i < 16; ++i) {  // packed f32x2: scale and shift, then row sums
                                float p0, p1;
                                fma_f32x2(p0, p1, __uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]), scale_log2,
                                          -mx);
                                p0 = fast_exp2(p0);
                                p1 = fast_exp2(p1);
                                add_f32x2(rs0, rs1, p0, p1);
                                pk[i] = pack_bf16x2(p0, p1);
                            }
                        } else {
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const float p0 = (c + 2 * i < valid) ? fast_exp2(fmaf(__uint_as_float(v[2 * i]), scale_log2, -mx)) : 0.f;
                                const float p1 = (c + 2 * i + 1 < valid) ? fast_exp2(fmaf(__uint_as_float(v[2 * i + 1]), scale_log2, -mx)) : 0.f;
                                rs0 += p0;
                                rs1 += p1;
                                pk[i] = pack_bf16x2(p0, p1);
                            }
                        }
                        tmem_st_x16(tS + (c >> 1), pk);  // P over the S columns already consumed
                    }
                    tmem_wait_st();
                }
                l_run = l_run * alpha + (rs0 + rs1);
                m_run = mx;
                row_alpha[b * TQ + r] = alpha;
                row_l[b * TQ + r] = l_run;
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[b]);
                ++it;
            }
        }
    } else {
        // ------------------------------------------------ O fold warps 6..9
        const int q = warp & 3;
        const int r = q * 32 + lane;  // query row within the tile == TMEM lane
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        float o[HD];
#pragma unroll
        for (int d = 0; d < HD; ++d) o[d] = 0.f;
        uint32_t it = 0;
        bool ok = true;
        for (uint32_t k = 0; ok; ++k) {
            if (*abort_flag) break;
            const int slot = k % kRing;
            if (!(ok = wait(&unit_full[slot], (k / kRing) & 1))) break;
            const int4 e = ring[slot];
            __syncwarp();
            if (lane == 0) mbar_arrive(&unit_empty[slot]);
            if (e.y < 0) break;
            const Unit w = unit_of(e);
            __nv_bfloat16 *dst = nullptr;
            if (w.q0 + r < w.len) {
                const size_t row = static_cast<size_t>(w.start + w.q0 + r);
                dst = head_major ? out + (static_cast<size_t>(w.head) * total_tokens + row) * HD
                                 : out + row * dim + w.head * HD;
            }
            const bool warp_live = w.q0 + q * 32 < w.len;  // the same rows the softmax warp skips
            for (int j = 0; j < w.n_kv; ++j) {
                const uint32_t b = it & 1;
                const uint32_t par = (it >> 1) & 1;
                if (!(ok = wait(&o_full[b], par))) break;
                if (warp_live) {
                    // p_full of this phase has completed (PV waited for it); waiting on it
                    // here orders the reads of the softmax warp's row values
                    if (!(ok = wait(&p_full[b], par))) break;
                    const float alpha = row_alpha[b * TQ + r];
                    const float inv = 1.0f / row_l[b * TQ + r];
                    const bool store = dst != nullptr && j == w.n_kv - 1;
                    tc_fence_after();
                    const uint32_t tO = tmem + lane_base + b * 128 + 64;
#pragma unroll
                    for (int c = 0; c < HD; c += 8) {  // 8 columns per load: o[64] stays in registers
                        uint32_t v[8];
                        tmem_ld_x8(tO + c, v);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 8; ++i) o[c + i] = o[c + i] * alpha + __uint_as_float(v[i]);
                        if (store) {  // O / l of the unit's last item, 8 columns at a time
                            uint4 wv;
                            wv.x = pack_bf16x2(o[c + 0] * inv, o[c + 1] * inv);
                            wv.y = pack_bf16x2(o[c + 2] * inv, o[c + 3] * inv);
                            wv.z = pack_bf16x2(o[c + 4] * inv, o[c + 5] * inv);
                            wv.w = pack_bf16x2(o[c + 6] * inv, o[c + 7] * inv);
                            *reinterpret_cast<uint4 *>(dst + c) = wv;
                        }
                    }
                    if (j == w.n_kv - 1) {
#pragma unroll
                        for (int d = 0; d < HD; ++d) o[d] = 0.f;
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&slot_free[b]);
                ++it;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
    // Every unit request of this CTA has been made; the launch's last CTA to get here
    // returns the work counter to zero for the next launch that uses this slot.
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&sched[1], 1u) == gridDim.x - 1) {
            atomicExch(&sched[0], 0u);
            atomicExch(&sched[1], 0u);
        }
    }
}

}  // namespace

cudaError_t launch_attention_varlen(const void *qkv, const int32_t *cu_seqlens, int batch, int max_len, int heads,
                                    int head_dim, void *out, int64_t total_tokens, bool head_major, cudaStream_t s,
                                    fe_status *st)
{
    *st = FE_OK;
    if (batch == 0 || max_len == 0 || total_tokens == 0) return cudaSuccess;
    const int dim = heads * head_dim;
    CUtensorMap tm;
    fe_status r = head_major ? make_tmap_heads(&tm, qkv, 3 * static_cast<uint64_t>(heads), total_tokens, 128)
                             : make_tmap_2d(&tm, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, total_tokens, 3 * (int64_t)dim,
                                            3 * (int64_t)dim, 128, HD);
    if (r != FE_OK) {
        *st = r;
        return cudaSuccess;
    }
    static uint64_t configured[64] = {};  // context the attribute was set in
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t ctx = current_context_id();
    if (dev < 64 && configured[dev] != ctx) {
        cudaError_t e = cudaFuncSetAttribute(attn_varlen_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured[dev] = ctx;
    }
    const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(head_dim));
    const int ctas = kCtasPerSm * current_sm_count();
    // Each launch takes the next of kSchedSlots work counters (launches in flight at once
    // on different streams use different counters); the counters live in this module.
    static std::mutex sched_mu;
    static unsigned *sched_base[64] = {};
    static uint64_t sched_ctx[64] = {};  // context the address was looked up in
    static unsigned next_slot[64] = {};
    if (dev >= 64) {
        *st = fail(FE_ERR_UNSUPPORTED, "attention: device index above 63");
        return cudaSuccess;
    }
    unsigned *sched_dev = nullptr;
    unsigned slot = 0;
    {
        std::lock_guard<std::mutex> lock(sched_mu);
        if (!sched_base[dev] || sched_ctx[dev] != ctx) {
            void *p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_attn_sched);
            if (e != cudaSuccess) return e;
            sched_base[dev] = static_cast<unsigned *>(p);
            sched_ctx[dev] = ctx;
        }
        sched_dev = sched_base[dev];
        slot = next_slot[dev];
        next_slot[dev] += static_cast<unsigned>((batch + kMaxBatch - 1) / kMaxBatch);
    }
    // Sentence offsets are absolute rows of qkv, so a long batch runs as chunks over the
    // same tensor map, each small enough for the per-CTA prefix table.
    for (int b0 = 0; b0 < batch; b0 += kMaxBatch) {
        const int nb = batch - b0 < kMaxBatch ? batch - b0 : kMaxBatch;
        const int64_t units_bound = static_cast<int64_t>(nb) * ((max_len + TQ - 1) / TQ) * heads;
        const int grid = units_bound < ctas ? static_cast<int>(units_bound) : ctas;
        unsigned *sched = sched_dev + 2 * (slot++ % kSchedSlots);
        cudaError_t e = launch_k(attn_varlen_tcgen05, dim3(grid), dim3(kThreads), SMEM_BYTES, s, tm, cu_seqlens + b0,
                                 nb, heads, sched, static_cast<__nv_bfloat16 *>(out), scale_log2,
                                 static_cast<int>(total_tokens), head_major ? 1 : 0, current_device_status_word());
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace fe

namespace fe {
cudaError_t set_wait_limit_attention(uint64_t ns) { return set_wait_limit_this_file(ns); }
}  // namespace fe
