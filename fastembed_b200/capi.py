"""ctypes bindings of libfastembed_b200.so (the C ABI in include/fastembed_b200.h).

The library is the product; this module only binds it.  Importing fails loudly if
the shared library has not been built: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libfastembed_b200.so")

FE_OK = 0
STATUS = {0: "FE_OK", 1: "FE_ERR_INVALID_ARGUMENT", 2: "FE_ERR_CUDA", 3: "FE_ERR_OUT_OF_MEMORY",
          4: "FE_ERR_UNSUPPORTED", 5: "FE_ERR_DEVICE_TIMEOUT", 6: "FE_ERR_IO", 7: "FE_ERR_NOT_FOUND"}
EPI = {"none": 0, "bias": 1, "bias_gelu": 2, "bias_relu": 3, "bias_swish": 4, "bias_residual": 5, "swiglu": 6,
       "geglu": 7}
DTYPE = {"f32": 0, "bf16": 1}
POOL = {"cls": 0, "mean": 1, "last": 2}
ACT = {"gelu": 0, "relu": 1, "swish": 2}


class FeError(RuntimeError):
    def __init__(self, status: int, where: str, detail: str):
        super().__init__(f"{where}: {STATUS.get(status, status)}: {detail}")
        self.status = status


class EncoderConfig(C.Structure):
    _fields_ = [("vocab_size", C.c_int32), ("hidden", C.c_int32), ("layers", C.c_int32),
                ("heads", C.c_int32), ("intermediate", C.c_int32), ("max_position", C.c_int32),
                ("type_vocab", C.c_int32), ("layer_norm_eps", C.c_float), ("activation", C.c_int32),
                ("pooling", C.c_int32), ("positions", C.c_int32), ("pad_token_id", C.c_int32)]


POSITIONS = {"bert": 0, "xlmr": 1}


class RmsEncoderConfig(C.Structure):
    _fields_ = [("family", C.c_int32), ("vocab_size", C.c_int32), ("hidden", C.c_int32), ("layers", C.c_int32),
                ("q_heads", C.c_int32), ("kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("intermediate", C.c_int32), ("max_position", C.c_int32), ("rms_norm_eps", C.c_float),
                ("rope_theta", C.c_float), ("rope_theta_local", C.c_float), ("full_attention_every", C.c_int32),
                ("query_scale", C.c_float), ("pooling", C.c_int32)]


FAMILY = {"bert": 0, "qwen3": 1, "gemma3": 2}


class EngineStats(C.Structure):
    _fields_ = [("launches", C.c_int64), ("gemm_launches", C.c_int64), ("tokens", C.c_int64),
                ("gemm_ms", C.c_double), ("attention_ms", C.c_double), ("other_ms", C.c_double),
                ("gemm_flops", C.c_double), ("attention_flops", C.c_double)]


_lib = None

vp, i64, i32, f32, sz = C.c_void_p, C.c_int64, C.c_int32, C.c_float, C.c_size_t
_SIGS = {
    "fe_status_string": ([C.c_int], C.c_char_p),
    "fe_last_error_message": ([], C.c_char_p),
    "fe_device_status": ([C.c_int], C.c_int),
    "fe_set_wait_limit": ([C.c_int, C.c_uint64], C.c_int),
    "fe_version": ([], C.c_char_p),
    "fe_sgemm_nn": ([vp, vp, vp, i64, i64, i64, vp], C.c_int),
    "fe_sgemm_nt": ([vp, vp, vp, vp, i64, i64, i64, vp], C.c_int),
    "fe_gelu_f32": ([vp, vp, i64, vp], C.c_int),
    "fe_relu_f32": ([vp, vp, i64, vp], C.c_int),
    "fe_swish_f32": ([vp, vp, i64, vp], C.c_int),
    "fe_layer_norm_f32": ([vp, vp, vp, vp, i64, i64, f32, vp], C.c_int),
    "fe_rms_norm_f32": ([vp, vp, vp, i64, i64, f32, vp], C.c_int),
    "fe_softmax_rows_f32": ([vp, vp, i64, i64, vp], C.c_int),
    "fe_softmax_scores_inplace_f32": ([vp, i64, i64, vp], C.c_int),
    "fe_mha_f32_workspace_bytes": ([i64, i64, i64], sz),
    "fe_mha_f32": ([vp] * 8 + [i64, i64, i64, vp, sz, vp], C.c_int),
    "fe_mha_f32_noalloc": ([vp] * 8 + [i64, i64, i64, vp], C.c_int),
    "fe_linear_bf16": ([vp, vp, vp, vp, vp, i64, i64, i64, C.c_int, C.c_int, vp], C.c_int),
    "fe_attention_varlen_bf16": ([vp, vp, i32, i32, i32, i32, vp, i64, vp], C.c_int),
    "fe_embed_layernorm": ([vp, vp, i32, i64, vp, vp, vp, vp, vp, i32, i32, i32, f32, vp, vp, vp], C.c_int),
    "fe_embed_layernorm_xlmr": ([vp, vp, i32, i64, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32, vp, vp, vp], C.c_int),
    "fe_layernorm_dual": ([vp, vp, vp, vp, vp, vp, i64, i32, f32, vp], C.c_int),
    "fe_attention_varlen_gqa_bf16": ([vp, vp, i32, i32, i32, i32, i32, i32, f32, vp, i64, vp], C.c_int),
    "fe_linear_layernorm_workspace_bytes": ([i64, i64, C.POINTER(sz)], C.c_int),
    "fe_linear_rmsnorm_bf16": ([vp, vp, vp, vp, vp, vp, i64, i64, i64, f32, vp, sz, vp], C.c_int),
    "fe_linear_layernorm_bf16": ([vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, f32, vp, sz, vp], C.c_int),
    "fe_embed_scale": ([vp, i64, vp, i32, i32, f32, vp, vp], C.c_int),
    "fe_rms_norm_rows": ([vp, vp, i32, f32, i64, i32, vp, vp, vp], C.c_int),
    "fe_rms_sandwich": ([vp, vp, vp, vp, i32, f32, i64, i32, vp, vp, vp], C.c_int),
    "fe_rms_sandwich_bf16": ([vp, vp, vp, vp, i32, f32, i64, i32, vp, vp, vp], C.c_int),
    "fe_linear_qk_norm_rope_bf16": ([vp, vp, vp, vp, vp, vp, i64, i64, i32, i32, i32, i32, f32, f32, vp], C.c_int),
    "fe_linear_qk_norm_rope_scaled_bf16": ([vp, vp, vp, vp, vp, vp, i64, i64, i32, i32, i32, i32, f32, f32, vp, i32,
                                            vp], C.c_int),
    "fe_linear_rmsnorm_deferred_bf16": ([vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp], C.c_int),
    "fe_linear_rmsnorm_deferred_parts": ([i64], C.c_int32),
    "fe_linear_row_scaled_bf16": ([vp, vp, vp, vp, vp, i64, i64, i64, C.c_int, C.c_int, vp, i32, f32, vp], C.c_int),
    "fe_token_positions": ([vp, i32, vp, vp], C.c_int),
    "fe_qk_norm_rope_bf16": ([vp, vp, i32, i64, i32, i32, i32, vp, vp, i32, f32, f32, vp], C.c_int),
    "fe_pool_l2": ([vp, vp, i32, i32, C.c_int, vp, vp], C.c_int),
    "fe_engine_create": ([C.POINTER(EncoderConfig), C.c_int, C.POINTER(vp)], C.c_int),
    "fe_engine_create_rms": ([C.POINTER(RmsEncoderConfig), C.c_int, C.POINTER(vp)], C.c_int),
    "fe_engine_destroy": ([vp], C.c_int),
    "fe_engine_set_weight": ([vp, C.c_char_p, vp, sz, C.c_int], C.c_int),
    "fe_engine_load_safetensors": ([vp, C.c_char_p], C.c_int),
    "fe_engine_missing_weights": ([vp], i32),
    "fe_engine_encode_packed": ([vp, vp, vp, vp, i32, vp, vp], C.c_int),
    "fe_engine_encode_host": ([vp, vp, vp, i32, i32, vp], C.c_int),
    "fe_engine_set_profiling": ([vp, C.c_int], C.c_int),
    "fe_engine_get_stats": ([vp, C.POINTER(EngineStats)], C.c_int),
    "fe_plan_shards": ([C.POINTER(EncoderConfig), vp, i32, i32, vp], C.c_int),
    "fe_plan_shards_costs": ([vp, i32, i32, vp], C.c_int),
    "fe_pack_batch": ([vp, vp, i32, i32, vp, vp], C.c_int),
    "fe_wordpiece_create": ([C.c_char_p, C.POINTER(vp)], C.c_int),
    "fe_wordpiece_destroy": ([vp], C.c_int),
    "fe_wordpiece_encode": ([vp, C.c_char_p, sz, vp, sz, C.POINTER(sz)], C.c_int),
}


def lib() -> C.CDLL:
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m fastembed_b200.build` "
                              "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def check(status: int, where: str) -> None:
    if status != FE_OK:
        detail = lib().fe_last_error_message().decode(errors="replace")
        raise FeError(status, where, detail)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def exported_symbols() -> list[str]:
    return list(_SIGS)
