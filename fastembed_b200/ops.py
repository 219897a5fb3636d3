"""Torch-tensor front end of the C ABI: each function checks shapes, passes raw
device pointers and the current torch stream to libfastembed_b200.so, and raises
FeError on a non-OK status.  PyTorch only supplies device memory and streams."""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import capi
from .capi import ACT, DTYPE, EPI, POOL, call


def _p(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def _s(t: torch.Tensor):
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _cuda(*ts):
    for t in ts:
        if t is not None and (not t.is_cuda or not t.is_contiguous()):
            raise ValueError("expected contiguous CUDA tensors")


# ---------------------------------------------------------------- fp32 op API
def sgemm_nn(a, b, m, n, k):
    _cuda(a, b)
    c = torch.empty(m * k, dtype=torch.float32, device=a.device)
    call("fe_sgemm_nn", _p(a), _p(b), _p(c), m, n, k, _s(a))
    return c


def sgemm_nt(a, b, m, n, k, bias=None):
    _cuda(a, b, bias)
    c = torch.empty(m * k, dtype=torch.float32, device=a.device)
    call("fe_sgemm_nt", _p(a), _p(b), _p(bias), _p(c), m, n, k, _s(a))
    return c


def unary(name, x):
    _cuda(x)
    y = torch.empty_like(x)
    call(f"fe_{name}_f32", _p(x), _p(y), x.numel(), _s(x))
    return y


def layer_norm_f32(x, g, b, dim, eps):
    _cuda(x, g, b)
    y = torch.empty_like(x)
    call("fe_layer_norm_f32", _p(x), _p(g), _p(b), _p(y), x.numel() // dim, dim, eps, _s(x))
    return y


def rms_norm_f32(x, w, dim, eps):
    _cuda(x, w)
    y = torch.empty_like(x)
    call("fe_rms_norm_f32", _p(x), _p(w), _p(y), x.numel() // dim, dim, eps, _s(x))
    return y


def softmax_rows_f32(x, dim):
    _cuda(x)
    y = torch.empty_like(x)
    call("fe_softmax_rows_f32", _p(x), _p(y), x.numel() // dim, dim, _s(x))
    return y


def softmax_scores_inplace(scores, heads, seq_len):
    _cuda(scores)
    call("fe_softmax_scores_inplace_f32", _p(scores), heads, seq_len, _s(scores))
    return scores


def mha_f32(x, wq, wk, wv, bq, bk, bv, heads, dim):
    _cuda(x, wq, wk, wv, bq, bk, bv)
    L = x.numel() // dim
    out = torch.empty(L * dim, dtype=torch.float32, device=x.device)
    nbytes = capi.lib().fe_mha_f32_workspace_bytes(L, dim, heads)
    ws = torch.empty(max(nbytes, 4), dtype=torch.uint8, device=x.device)
    call("fe_mha_f32", _p(x), _p(wq), _p(wk), _p(wv), _p(bq), _p(bk), _p(bv), _p(out), L, dim, heads,
         _p(ws), nbytes, _s(x))
    return out


# ---------------------------------------------------------- bf16 hot-path ops
def linear_bf16(x, w, bias=None, residual=None, epilogue="none", out_dtype="bf16"):
    """y = epilogue(x @ w.T): x [m,k] bf16, w [n,k] bf16."""
    _cuda(x, w, bias, residual)
    m, k = x.shape
    n = w.shape[0]
    ny = n // 2 if epilogue in ("swiglu", "geglu") else n
    y = torch.empty(m, ny, dtype=torch.bfloat16 if out_dtype == "bf16" else torch.float32, device=x.device)
    call("fe_linear_bf16", _p(x), _p(w), _p(bias), _p(residual), _p(y), m, n, k, EPI[epilogue],
         DTYPE[out_dtype], _s(x))
    return y


def attention_varlen(qkv, cu_seqlens, max_len, heads, head_dim=64):
    _cuda(qkv, cu_seqlens)
    T = qkv.shape[0]
    out = torch.empty(T, heads * head_dim, dtype=torch.bfloat16, device=qkv.device)
    call("fe_attention_varlen_bf16", _p(qkv), _p(cu_seqlens), cu_seqlens.numel() - 1, max_len, heads, head_dim,
         _p(out), T, _s(qkv))
    return out


def attention_gqa(qkv, cu_seqlens, max_len, q_heads, kv_heads, head_dim, causal, scale=None):
    """Grouped-query varlen attention (head_dim 128 / 256): qkv [T, (Hq + 2 Hkv) * hd] bf16."""
    _cuda(qkv, cu_seqlens)
    T = qkv.shape[0]
    scale = head_dim ** -0.5 if scale is None else scale
    out = torch.empty(T, q_heads * head_dim, dtype=torch.bfloat16, device=qkv.device)
    call("fe_attention_varlen_gqa_bf16", _p(qkv), _p(cu_seqlens), cu_seqlens.numel() - 1, max_len, q_heads, kv_heads,
         head_dim, 1 if causal else 0, scale, _p(out), T, _s(qkv))
    return out


def embed_layernorm(ids, cu_seqlens, word, pos, type_, gamma, beta, eps, pad_id=None):
    """pad_id None: BERT position rows; an int: the bge-m3 / XLM-R rows with that pad id."""
    _cuda(ids, cu_seqlens, word, pos, type_, gamma, beta)
    T = ids.numel()
    D = word.shape[1]
    h32 = torch.empty(T, D, dtype=torch.float32, device=ids.device)
    h16 = torch.empty(T, D, dtype=torch.bfloat16, device=ids.device)
    if pad_id is None:
        call("fe_embed_layernorm", _p(ids), _p(cu_seqlens), cu_seqlens.numel() - 1, T, _p(word), _p(pos),
             _p(type_), _p(gamma), _p(beta), D, word.shape[0], pos.shape[0], eps, _p(h32), _p(h16), _s(ids))
    else:
        call("fe_embed_layernorm_xlmr", _p(ids), _p(cu_seqlens), cu_seqlens.numel() - 1, T, _p(word), _p(pos),
             _p(type_), _p(gamma), _p(beta), D, word.shape[0], pos.shape[0], pad_id, eps, _p(h32), _p(h16),
             _s(ids))
    return h32, h16


def layernorm_dual(x, gamma, beta, eps, residual=None):
    _cuda(x, gamma, beta, residual)
    rows, D = x.shape
    h32 = torch.empty_like(x)
    h16 = torch.empty(rows, D, dtype=torch.bfloat16, device=x.device)
    call("fe_layernorm_dual", _p(x), _p(residual), _p(gamma), _p(beta), _p(h32), _p(h16), rows, D, eps, _s(x))
    return h32, h16


def linear_layernorm_workspace(m, n, device):
    """A zero-filled workspace for linear_layernorm of [m, n] rows (reusable across calls)."""
    size = C.c_size_t(0)
    call("fe_linear_layernorm_workspace_bytes", m, n, C.byref(size))
    return torch.zeros(max(int(size.value), 1), dtype=torch.uint8, device=device)


def linear_layernorm(x, w, bias, gamma, beta, h32, eps, workspace=None, want_h16=True):
    """h32 <- LayerNorm((x @ w.T + bias) + h32) * gamma + beta in place; returns (h32, h16)."""
    _cuda(x, w, bias, gamma, beta, h32)
    m, k = x.shape
    n = w.shape[0]
    if workspace is None:
        workspace = linear_layernorm_workspace(m, n, x.device)
    h16 = torch.empty(m, n, dtype=torch.bfloat16, device=x.device) if want_h16 else None
    call("fe_linear_layernorm_bf16", _p(x), _p(w), _p(bias), _p(gamma), _p(beta), _p(h32), _p(h16), m, n, k, eps,
         _p(workspace), workspace.numel(), _s(x))
    return h32, h16


def linear_rmsnorm(x, w, bias, rms_w, h32, eps, workspace=None, want_h16=True):
    """Pre-norm: h32 <- (x @ w.T + bias) + h32 in place; returns (h32, bf16 RMSNorm(h32) * rms_w)."""
    _cuda(x, w, bias, rms_w, h32)
    m, k = x.shape
    n = w.shape[0]
    if workspace is None:
        workspace = linear_layernorm_workspace(m, n, x.device)
    h16 = torch.empty(m, n, dtype=torch.bfloat16, device=x.device) if want_h16 else None
    call("fe_linear_rmsnorm_bf16", _p(x), _p(w), _p(bias), _p(rms_w), _p(h32), _p(h16), m, n, k, eps, _p(workspace),
         workspace.numel(), _s(x))
    return h32, h16


def linear_rmsnorm_deferred(x, w, bias, rms_w, h32, want_h16=True):
    """Pre-norm with the RMSNorm deferred: h32 <- (x @ w.T + bias) + h32 in place; returns
    (h32, bf16(h32 * rms_w), row_ss [m, parts] partial sums of h32^2) for a row-scaled consumer."""
    _cuda(x, w, bias, rms_w, h32)
    m, k = x.shape
    n = w.shape[0]
    parts = capi.lib().fe_linear_rmsnorm_deferred_parts(n)
    h16 = torch.empty(m, n, dtype=torch.bfloat16, device=x.device) if want_h16 else None
    row_ss = torch.empty(m, max(parts, 1), dtype=torch.float32, device=x.device)
    call("fe_linear_rmsnorm_deferred_bf16", _p(x), _p(w), _p(bias), _p(rms_w), _p(h32), _p(h16), _p(row_ss), m, n, k,
         _s(x))
    return h32, h16, row_ss


def linear_row_scaled(x, w, row_ss, eps, bias=None, residual=None, epilogue="none", out_dtype="bf16"):
    """linear_bf16 with row i of x @ w.T multiplied by 1 / sqrt(sum(row_ss[i]) / k + eps) first."""
    _cuda(x, w, row_ss, bias, residual)
    m, k = x.shape
    n = w.shape[0]
    ny = n // 2 if epilogue in ("swiglu", "geglu") else n
    y = torch.empty(m, ny, dtype=torch.bfloat16 if out_dtype == "bf16" else torch.float32, device=x.device)
    call("fe_linear_row_scaled_bf16", _p(x), _p(w), _p(bias), _p(residual), _p(y), m, n, k, EPI[epilogue],
         DTYPE[out_dtype], _p(row_ss), row_ss.shape[1], eps, _s(x))
    return y


def embed_scale(ids, word, scale):
    _cuda(ids, word)
    T = ids.numel()
    h32 = torch.empty(T, word.shape[1], dtype=torch.float32, device=ids.device)
    call("fe_embed_scale", _p(ids), T, _p(word), word.shape[0], word.shape[1], scale, _p(h32), _s(ids))
    return h32


def rms_norm_rows(x, w, eps, one_plus=False):
    _cuda(x, w)
    rows, D = x.shape
    o32 = torch.empty_like(x)
    o16 = torch.empty(rows, D, dtype=torch.bfloat16, device=x.device)
    call("fe_rms_norm_rows", _p(x), _p(w), 1 if one_plus else 0, eps, rows, D, _p(o32), _p(o16), _s(x))
    return o32, o16


def rms_sandwich(y, w_post, h32, w_next, eps, one_plus=True):
    """h32 += RMSNorm(y; w_post) in place; returns (RMSNorm(h32; w_next) fp32, bf16)."""
    _cuda(y, w_post, h32, w_next)
    rows, D = y.shape
    o32 = torch.empty(rows, D, dtype=torch.float32, device=y.device)
    o16 = torch.empty(rows, D, dtype=torch.bfloat16, device=y.device)
    fn = "fe_rms_sandwich_bf16" if y.dtype == torch.bfloat16 else "fe_rms_sandwich"
    call(fn, _p(y), _p(w_post), _p(h32), _p(w_next), 1 if one_plus else 0, eps, rows, D, _p(o32), _p(o16), _s(y))
    return o32, o16


def qk_norm_rope(qkv, cu_seqlens, q_heads, kv_heads, head_dim, q_w, k_w, eps, theta, one_plus=False):
    """In place on qkv [T, (Hq + 2 Hkv) * hd] bf16."""
    _cuda(qkv, cu_seqlens, q_w, k_w)
    call("fe_qk_norm_rope_bf16", _p(qkv), _p(cu_seqlens), cu_seqlens.numel() - 1, qkv.shape[0], q_heads, kv_heads,
         head_dim, _p(q_w), _p(k_w), 1 if one_plus else 0, eps, theta, _s(qkv))
    return qkv


def token_positions(cu_seqlens):
    """int32 [T]: each token's position in its sentence."""
    _cuda(cu_seqlens)
    B = cu_seqlens.numel() - 1
    T = int(cu_seqlens[-1].item()) if B > 0 else 0
    pos = torch.empty(max(T, 1), dtype=torch.int32, device=cu_seqlens.device)
    call("fe_token_positions", _p(cu_seqlens), B, _p(pos), _s(cu_seqlens))
    return pos[:T]


def linear_qk_norm_rope(x, w, q_w, k_w, positions, q_heads, kv_heads, head_dim, eps, theta, one_plus=False):
    """QKV projection [m, (Hq + 2 Hkv) hd] bf16 = x @ w.T with the q/k RMSNorm and RoPE fused
    into the GEMM epilogue."""
    _cuda(x, w, q_w, k_w, positions)
    m, k = x.shape
    y = torch.empty(m, (q_heads + 2 * kv_heads) * head_dim, dtype=torch.bfloat16, device=x.device)
    call("fe_linear_qk_norm_rope_bf16", _p(x), _p(w), _p(q_w), _p(k_w), _p(positions), _p(y), m, k, q_heads,
         kv_heads, head_dim, 1 if one_plus else 0, eps, theta, _s(x))
    return y


def linear_qk_norm_rope_scaled(x, w, q_w, k_w, positions, q_heads, kv_heads, head_dim, eps, theta, row_ss,
                               one_plus=False):
    """linear_qk_norm_rope on an input whose rows still need their RMSNorm factor (row_ss)."""
    _cuda(x, w, q_w, k_w, positions, row_ss)
    m, k = x.shape
    y = torch.empty(m, (q_heads + 2 * kv_heads) * head_dim, dtype=torch.bfloat16, device=x.device)
    call("fe_linear_qk_norm_rope_scaled_bf16", _p(x), _p(w), _p(q_w), _p(k_w), _p(positions), _p(y), m, k, q_heads,
         kv_heads, head_dim, 1 if one_plus else 0, eps, theta, _p(row_ss), row_ss.shape[1], _s(x))
    return y


def pool_l2(h, cu_seqlens, mode="cls"):
    _cuda(h, cu_seqlens)
    B = cu_seqlens.numel() - 1
    D = h.shape[1]
    out = torch.empty(B, D, dtype=torch.float32, device=h.device)
    call("fe_pool_l2", _p(h), _p(cu_seqlens), B, D, POOL[mode], _p(out), _s(h))
    return out


def device_status(device: int = 0) -> None:
    capi.check(capi.lib().fe_device_status(device), "fe_device_status")


# ------------------------------------------------------------------- engine
class Engine:
    """One device-resident encoder (fe_engine) on one GPU."""

    def __init__(self, shape, device: int = 0, pooling: str = "cls"):
        """`shape`: a workload.EncoderShape (post-LN BERT) or workload.RmsShape (Qwen3 /
        Gemma3 shapes, whose pooling comes with the family)."""
        self.shape = shape
        self.device = device
        h = C.c_void_p()
        if hasattr(shape, "family"):
            cfg = capi.RmsEncoderConfig(capi.FAMILY[shape.family], shape.vocab, shape.hidden, shape.layers,
                                        shape.q_heads, shape.kv_heads, shape.head_dim, shape.intermediate,
                                        shape.max_pos, shape.eps, shape.rope_theta, shape.rope_theta_local,
                                        shape.full_every, 0.0, POOL[shape.pooling])
            capi.check(capi.lib().fe_engine_create_rms(C.byref(cfg), device, C.byref(h)), "fe_engine_create_rms")
        else:
            pad_id = getattr(shape, "pad_id", -1)  # >= 0: the bge-m3 / XLM-R position rows
            cfg = capi.EncoderConfig(shape.vocab, shape.hidden, shape.layers, shape.heads, shape.intermediate,
                                     shape.max_pos, shape.type_vocab, shape.eps, ACT[shape.act], POOL[pooling],
                                     capi.POSITIONS["xlmr" if pad_id >= 0 else "bert"], max(pad_id, 0))
            capi.check(capi.lib().fe_engine_create(C.byref(cfg), device, C.byref(h)), "fe_engine_create")
        self._cfg = cfg
        self.h = h

    def close(self):
        if self.h:
            capi.lib().fe_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_weight(self, name: str, value) -> None:
        if isinstance(value, torch.Tensor) and value.is_cuda:
            v = value.contiguous().float()
            call("fe_engine_set_weight", self.h, name.encode(), _p(v), v.numel(), 1)
        else:
            v = np.ascontiguousarray(value, dtype=np.float32)
            call("fe_engine_set_weight", self.h, name.encode(), v.ctypes.data_as(C.c_void_p), v.size, 0)

    def load_weights(self, weights: dict) -> None:
        for name, v in weights.items():
            if name.startswith("pooler."):
                continue  # read but unused by the reference forward (sentence_transformers_impl.cpp:285-331)
            self.set_weight(name, v)
        missing = capi.lib().fe_engine_missing_weights(self.h)
        if missing:
            raise ValueError(f"{missing} weights missing")

    def load_safetensors(self, path: str) -> None:
        call("fe_engine_load_safetensors", self.h, path.encode())

    def encode_host(self, ids: np.ndarray, lengths: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        lengths = np.ascontiguousarray(lengths, dtype=np.int32)
        B, S = ids.shape
        out = np.empty((B, self.shape.hidden), np.float32)
        call("fe_engine_encode_host", self.h, ids.ctypes.data_as(C.c_void_p), lengths.ctypes.data_as(C.c_void_p),
             B, S, out.ctypes.data_as(C.c_void_p))
        return out

    def encode_packed(self, ids_dev: torch.Tensor, cu_dev: torch.Tensor, cu_host: np.ndarray,
                      out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        cu_host = np.ascontiguousarray(cu_host, dtype=np.int32)
        B = cu_host.size - 1
        if out is None:
            out = torch.empty(B, self.shape.hidden, dtype=torch.float32, device=ids_dev.device)
        st = stream if stream is not None else torch.cuda.current_stream(ids_dev.device)
        call("fe_engine_encode_packed", self.h, _p(ids_dev), _p(cu_dev), cu_host.ctypes.data_as(C.c_void_p), B,
             _p(out), C.c_void_p(st.cuda_stream))
        return out

    def set_profiling(self, on: bool) -> None:
        call("fe_engine_set_profiling", self.h, 1 if on else 0)

    def stats(self) -> dict:
        s = capi.EngineStats()
        call("fe_engine_get_stats", self.h, C.byref(s))
        return {k: getattr(s, k) for k, _ in s._fields_}


def pack(ids: np.ndarray, lengths: np.ndarray):
    """Host packing through the library's fe_pack_batch: (ids_packed, cu_seqlens)."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    lengths = np.ascontiguousarray(lengths, dtype=np.int32)
    B, S = ids.shape
    packed = np.empty(max(int(lengths.sum()), 1), np.int32)
    cu = np.empty(B + 1, np.int32)
    call("fe_pack_batch", ids.ctypes.data_as(C.c_void_p), lengths.ctypes.data_as(C.c_void_p), B, S,
         packed.ctypes.data_as(C.c_void_p), cu.ctypes.data_as(C.c_void_p))
    return packed[:int(lengths.sum())], cu


def plan_shards(shape, sorted_lengths: np.ndarray, parts: int) -> list[int]:
    """Contiguous cost-balanced cut points of a length-sorted batch (fe_plan_shards for the
    BERT family, whose cost adds a per-tile attention term to the projection FLOPs;
    fe_plan_shards_costs over the shape's own per-sentence FLOPs for the Qwen3 / Gemma3
    shapes)."""
    L = np.ascontiguousarray(sorted_lengths, dtype=np.int32)
    cuts = np.zeros(max(parts - 1, 1), np.int32)
    if hasattr(shape, "family"):
        if L.size > 1 and np.any(L[1:] > L[:-1]):
            raise ValueError("plan_shards: lengths must be sorted in descending order")
        costs = np.array([shape.shard_cost(int(x)) for x in L], np.float64)
        call("fe_plan_shards_costs", costs.ctypes.data_as(C.c_void_p), L.size, parts,
             cuts.ctypes.data_as(C.c_void_p))
    else:
        cfg = capi.EncoderConfig(shape.vocab, shape.hidden, shape.layers, shape.heads, shape.intermediate,
                                 shape.max_pos, shape.type_vocab, shape.eps, ACT[shape.act], 0)
        call("fe_plan_shards", C.byref(cfg), L.ctypes.data_as(C.c_void_p), L.size, parts,
             cuts.ctypes.data_as(C.c_void_p))
    return [int(c) for c in cuts[:parts - 1]]
