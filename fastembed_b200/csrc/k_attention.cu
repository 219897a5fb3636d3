// k_attention.cu — variable-length bidirectional attention on tcgen05 (head_dim 64).
//
// Replaces the QK^T / softmax / PV stage of CUDAAttentionOps::multi_head_attention
// (src/ops/cuda/cuda_attention_ops.cu:264-313: permute, batched QK^T, scaled softmax,
// batched PV, unpermute) for a packed batch of unpadded sentences.  Its semantics are
// the CPU reference's per-sentence attention (src/ops/cpu/cpu_attention_ops.cpp:33-85):
// softmax(Q K^T / sqrt(hd)) V with keys limited to the sentence, which is exactly a
// key-padding mask over a padded batch.
//
// One CTA = (128-query tile, sentence, head); 4 warps, thread t owns query row t.
//   * TMA reads Q, K, V tiles [128 x 64] straight out of the packed QKV GEMM output
//     (column block h*64 of the Q / K / V thirds), so there is no permute pass.
//   * S = Q K^T (M=128, N=128, K=64) lands in TMEM; each thread reads its row with
//     tcgen05.ld, masks keys past the sentence end, runs the online-softmax update in
//     registers and writes P (bf16) into a 128B-swizzled shared-memory tile.
//   * O_j = P V_j (M=128, N=64, K=128, V as an MN-major operand) lands in TMEM; the
//     thread folds it into its fp32 accumulator with the running rescale factor.
// Waits are bounded (device status word on timeout).
#include <cuda.h>
#include <cuda_bf16.h>

#include "fe_common.cuh"
#include "fe_internal.h"

namespace fe {
namespace {

constexpr int HD = 64;
constexpr int TQ = 128;  // query rows per CTA
constexpr int TK = 128;  // keys per inner tile
constexpr uint32_t TILE_BYTES = 128 * HD * 2;  // 16 KB: [128 rows x 64] bf16
constexpr uint32_t P_BYTES = TQ * TK * 2;      // 32 KB
constexpr uint32_t SMEM_BYTES = 1024 + 3 * TILE_BYTES + P_BYTES + 128;
constexpr uint32_t TMEM_COLS = 256;  // S at [0,128), O at [128,192)

__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__global__ void __launch_bounds__(128)
    attn_varlen_tcgen05(const __grid_constant__ CUtensorMap tm_qkv, const int32_t *__restrict__ cu_seqlens,
                        int dim, __nv_bfloat16 *__restrict__ out, float scale_log2, int *status)
{
    const int seq = blockIdx.y;
    const int head = blockIdx.z;
    const int start = cu_seqlens[seq];
    const int len = cu_seqlens[seq + 1] - start;
    const int q0 = blockIdx.x * TQ;
    if (q0 >= len) return;  // whole CTA leaves before touching TMEM or barriers

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem;
    uint8_t *sK = sQ + TILE_BYTES;
    uint8_t *sV = sK + TILE_BYTES;
    uint8_t *sP = sV + TILE_BYTES;
    uint64_t *bar_ld = reinterpret_cast<uint64_t *>(sP + P_BYTES);
    uint64_t *bar_s = bar_ld + 1;
    uint64_t *bar_o = bar_ld + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar_ld + 3);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int n_kv = (len + TK - 1) / TK;
    const int qcol = head * HD, kcol = dim + head * HD, vcol = 2 * dim + head * HD;

    if (tid == 0) {
        mbar_init(bar_ld, 1);
        mbar_init(bar_s, 1);
        mbar_init(bar_o, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t t_lane = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tS = tmem + t_lane;
    const uint32_t tO = tmem + t_lane + 128;

    // Only thread 0 issues TMA loads and MMAs; `arms` counts the loads it armed on
    // bar_ld and `landed` those it has seen complete.
    int arms = 0, landed = 0;
    uint64_t *open_bar = nullptr;  // barrier of a committed MMA not yet seen complete
    uint32_t open_par = 0;
    if (tid == 0) {
        mbar_arrive_expect_tx(bar_ld, 3 * TILE_BYTES);
        tma_load_2d(sQ, &tm_qkv, bar_ld, qcol, start + q0);
        tma_load_2d(sK, &tm_qkv, bar_ld, kcol, start);
        tma_load_2d(sV, &tm_qkv, bar_ld, vcol, start);
        arms = 1;
    }

    constexpr uint32_t idesc_s = idesc_bf16_f32(TQ, TK, false, false);
    constexpr uint32_t idesc_o = idesc_bf16_f32(TQ, HD, false, true);
    float m_run = -INFINITY, l_run = 0.f;
    float o[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) o[d] = 0.f;
    bool aborted = false;

    for (int j = 0; j < n_kv; ++j) {
        const uint32_t par = j & 1;
        bool to = false;
        if (tid == 0) {
            to = !mbar_wait(bar_ld, par);
            if (!to) {
                landed = arms;
                tc_fence_after();
                const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK);
#pragma unroll
                for (int k = 0; k < HD / 16; ++k)
                    umma_f16_ss(tmem, sdesc_sw128(q_addr + k * 32, 16, 1024),
                                sdesc_sw128(k_addr + k * 32, 16, 1024), idesc_s, k != 0 ? 1u : 0u);
                umma_commit(bar_s);
                open_bar = bar_s;
                open_par = par;
            }
        }
        if (__syncthreads_or(to)) { aborted = true; break; }
        to = !mbar_wait(bar_s, par);
        if (__syncthreads_or(to)) { aborted = true; break; }
        open_bar = nullptr;
        tc_fence_after();
        const int valid = min(TK, len - j * TK);

        // pass 1: running max of the scaled scores of this row
        float mx = m_run;
#pragma unroll 1
        for (int c = 0; c < TK; c += 32) {
            uint32_t v[32];
            tmem_ld_x32(tS + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (c + i < valid) mx = fmaxf(mx, __uint_as_float(v[i]) * scale_log2);
        }
        const float alpha = fast_exp2(m_run - mx);  // exp2(-inf) = 0 on the first tile
        // pass 2: p = exp2(s*scale - max), row sum, P tile in bf16 (128B-swizzled, K-major)
        float rs = 0.f;
#pragma unroll 1
        for (int c = 0; c < TK; c += 32) {
            uint32_t v[32];
            tmem_ld_x32(tS + c, v);
            tmem_wait_ld();
            float p[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                p[i] = (c + i < valid) ? fast_exp2(__uint_as_float(v[i]) * scale_log2 - mx) : 0.f;
                rs += p[i];
            }
            // columns c..c+31 = atom (c/64), 16-byte chunks (c%64)/8 .. +3 of row tid
            uint8_t *row = sP + (c >> 6) * (TQ * 128) + tid * 128;
            const int chunk0 = (c & 63) >> 3;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                uint4 w;
                w.x = pack_bf16x2(p[u * 8 + 0], p[u * 8 + 1]);
                w.y = pack_bf16x2(p[u * 8 + 2], p[u * 8 + 3]);
                w.z = pack_bf16x2(p[u * 8 + 4], p[u * 8 + 5]);
                w.w = pack_bf16x2(p[u * 8 + 6], p[u * 8 + 7]);
                *reinterpret_cast<uint4 *>(row + (((chunk0 + u) ^ (tid & 7)) << 4)) = w;
            }
        }
        l_run = l_run * alpha + rs;
        m_run = mx;
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t p_addr = smem_u32(sP), v_addr = smem_u32(sV);
#pragma unroll
            for (int ks = 0; ks < TK / 16; ++ks) {
                const uint64_t ad = sdesc_sw128(p_addr + (ks >> 2) * (TQ * 128) + (ks & 3) * 32, 16, 1024);
                const uint64_t bd = sdesc_sw128(v_addr + ks * 16 * 128, TK * 128, 1024);
                umma_f16_ss(tmem + 128, ad, bd, idesc_o, ks != 0 ? 1u : 0u);
            }
            umma_commit(bar_o);
            open_bar = bar_o;
            open_par = par;
        }
        to = !mbar_wait(bar_o, par);
        if (__syncthreads_or(to)) { aborted = true; break; }
        open_bar = nullptr;
        tc_fence_after();
        // K/V buffers are free once PV has completed: fetch the next key tile.
        if (tid == 0 && j + 1 < n_kv) {
            mbar_arrive_expect_tx(bar_ld, 2 * TILE_BYTES);
            tma_load_2d(sK, &tm_qkv, bar_ld, kcol, start + (j + 1) * TK);
            tma_load_2d(sV, &tm_qkv, bar_ld, vcol, start + (j + 1) * TK);
            ++arms;
        }
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
            uint32_t v[32];
            tmem_ld_x32(tO + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[c + i] = o[c + i] * alpha + __uint_as_float(v[i]);
        }
    }

    if (aborted) {
        if (tid == 0) {
            report(status, DEV_TIMEOUT);
            // Loads and MMAs this CTA started must finish before smem / TMEM are released.
            if (arms > landed && !mbar_wait(bar_ld, (arms - 1) & 1)) report(status, DEV_TIMEOUT);
            if (open_bar && !mbar_wait(open_bar, open_par)) report(status, DEV_TIMEOUT);
        }
    } else if (q0 + tid < len) {
        const float inv = 1.0f / l_run;
        uint4 *dst = reinterpret_cast<uint4 *>(out + static_cast<size_t>(start + q0 + tid) * dim + qcol);
#pragma unroll
        for (int u = 0; u < HD / 8; ++u) {
            uint4 w;
            w.x = pack_bf16x2(o[u * 8 + 0] * inv, o[u * 8 + 1] * inv);
            w.y = pack_bf16x2(o[u * 8 + 2] * inv, o[u * 8 + 3] * inv);
            w.z = pack_bf16x2(o[u * 8 + 4] * inv, o[u * 8 + 5] * inv);
            w.w = pack_bf16x2(o[u * 8 + 6] * inv, o[u * 8 + 7] * inv);
            dst[u] = w;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace

cudaError_t launch_attention_varlen(const void *qkv, const int32_t *cu_seqlens, int batch,
                                    int max_len, int heads, int head_dim, void *out,
                                    int64_t total_tokens, cudaStream_t s, fe_status *st)
{
    *st = FE_OK;
    if (batch == 0 || max_len == 0 || total_tokens == 0) return cudaSuccess;
    const int dim = heads * head_dim;
    CUtensorMap tm;
    fe_status r = make_tmap_2d(&tm, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, total_tokens, 3 * (int64_t)dim,
                               3 * (int64_t)dim, 128, HD);
    if (r != FE_OK) {
        *st = r;
        return cudaSuccess;
    }
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(attn_varlen_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(head_dim));
    dim3 grid((max_len + TQ - 1) / TQ, batch, heads);
    attn_varlen_tcgen05<<<grid, 128, SMEM_BYTES, s>>>(tm, cu_seqlens, dim,
                                                      static_cast<__nv_bfloat16 *>(out), scale_log2,
                                                      current_device_status_word());
    return cudaGetLastError();
}

}  // namespace fe
