"""Python bindings of the CPU parity checker.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, by __graft_entry__.smoke() and by
bench.py's CPU-baseline leg, always as the checker or the timed CPU baseline and
never as the thing measured or shipped.  The product (fastembed_b200) does not
import this module.

Two interchangeable back ends share one C interface (oracle/fe_oracle.h):
  "port" -> oracle/_bin/libfe_oracle.so, the C restatement in fe_oracle.c;
  "ref"  -> oracle/_ref/libfe_ref.so, the reference's own CPU ops compiled from its
            sources (src/ops/cpu/*.cpp) and driven by ref_forward.cpp.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIBS: dict[str, C.CDLL] = {}

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


class Layer(C.Structure):
    _fields_ = [(n, C.POINTER(C.c_float)) for n in (
        "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "ln1_g", "ln1_b",
        "w1", "b1", "w2", "b2", "ln2_g", "ln2_b")]


class Bert(C.Structure):
    _fields_ = [("vocab", C.c_int), ("hidden", C.c_int), ("heads", C.c_int),
                ("intermediate", C.c_int), ("layers", C.c_int), ("max_pos", C.c_int),
                ("type_vocab", C.c_int), ("act", C.c_int), ("eps", C.c_float),
                ("word", C.POINTER(C.c_float)), ("pos", C.POINTER(C.c_float)),
                ("type", C.POINTER(C.c_float)), ("emb_ln_g", C.POINTER(C.c_float)),
                ("emb_ln_b", C.POINTER(C.c_float)), ("layer", C.POINTER(Layer)), ("pad_id", C.c_int)]


ACTS = {"gelu": 0, "relu": 1, "swish": 2}


def lib_path(kind: str) -> str:
    if kind == "port":
        return os.path.join(HERE, "_bin", "libfe_oracle.so")
    if kind == "ref":
        return os.path.join(HERE, "_ref", "libfe_ref.so")
    raise ValueError(kind)


def build() -> None:
    """Compile the checker (and, where the reference sources exist, oracle/_ref)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def available(kind: str) -> bool:
    return os.path.exists(lib_path(kind))


def load(kind: str = "port") -> C.CDLL:
    if kind in _LIBS:
        return _LIBS[kind]
    path = lib_path(kind)
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built (run make -C oracle)")
    lib = C.CDLL(path)
    p = "fe_oracle_" if kind == "port" else "fe_ref_"
    sz = C.c_size_t
    for name in ("matmul_nt", "matmul_nn"):
        f = getattr(lib, p + name)
        f.argtypes = [_f32p, _f32p, _f32p, sz, sz, sz]
        f.restype = None
    for name in ("gelu", "relu", "swish"):
        f = getattr(lib, p + name)
        f.argtypes = [_f32p, _f32p, sz]
        f.restype = None
    f = getattr(lib, p + "layer_norm")
    f.argtypes = [_f32p, _f32p, _f32p, _f32p, sz, sz, C.c_float]
    f.restype = None
    f = getattr(lib, p + "rms_norm")
    f.argtypes = [_f32p, _f32p, _f32p, sz, sz, C.c_float]
    f.restype = None
    f = getattr(lib, p + "softmax_rows")
    f.argtypes = [_f32p, _f32p, sz, sz]
    f.restype = None
    f = getattr(lib, p + "mha")
    f.argtypes = [_f32p] * 7 + [sz, sz, sz, _f32p]
    f.restype = None
    f = getattr(lib, p + "bert_forward")
    f.argtypes = [C.POINTER(Bert), _i32p, C.c_int, _f32p]
    f.restype = C.c_int
    f = getattr(lib, p + "bert_forward_batch")
    f.argtypes = [C.POINTER(Bert), _i32p, _i32p, C.c_int, C.c_int, _f32p, C.c_int]
    f.restype = C.c_int
    if kind == "port":
        f = lib.fe_oracle_position_rows
        f.argtypes = [_i32p, C.c_int, C.c_int, C.c_int, _i32p]
        f.restype = None
    if kind == "port" or hasattr(lib, "fe_oracle_fill_uniform_mt19937"):
        g = lib.fe_oracle_fill_uniform_mt19937
        g.argtypes = [C.c_uint32, C.c_float, C.c_float, _f32p, sz]
        g.restype = None
    lib._fe_prefix = p
    _LIBS[kind] = lib
    return lib


def _fn(kind, name):
    lib = load(kind)
    return getattr(lib, lib._fe_prefix + name)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------- op-level ----------------
def matmul_nt(a, b, m, n, k, kind="port"):
    out = np.empty(m * k, np.float32)
    _fn(kind, "matmul_nt")(_f32(a).ravel(), _f32(b).ravel(), out, m, n, k)
    return out


def matmul_nn(a, b, m, n, k, kind="port"):
    out = np.empty(m * k, np.float32)
    _fn(kind, "matmul_nn")(_f32(a).ravel(), _f32(b).ravel(), out, m, n, k)
    return out


def unary(name, x, kind="port"):
    x = _f32(x).ravel()
    out = np.empty_like(x)
    _fn(kind, name)(x, out, x.size)
    return out


def layer_norm(x, g, b, dim, eps, kind="port"):
    x = _f32(x).ravel()
    out = np.empty_like(x)
    _fn(kind, "layer_norm")(x, _f32(g).ravel(), _f32(b).ravel(), out, x.size, dim, eps)
    return out


def rms_norm(x, w, dim, eps, kind="port"):
    x = _f32(x).ravel()
    out = np.empty_like(x)
    _fn(kind, "rms_norm")(x, _f32(w).ravel(), out, x.size, dim, eps)
    return out


def softmax_rows(x, dim, kind="port"):
    x = _f32(x).ravel()
    out = np.empty_like(x)
    _fn(kind, "softmax_rows")(x, out, x.size, dim)
    return out


def mha(x, wq, wk, wv, bq, bk, bv, heads, dim, kind="port"):
    x = _f32(x).ravel()
    L = x.size // dim
    out = np.empty(L * dim, np.float32)
    _fn(kind, "mha")(x, _f32(wq).ravel(), _f32(wk).ravel(), _f32(wv).ravel(),
                     _f32(bq).ravel(), _f32(bk).ravel(), _f32(bv).ravel(), heads, dim, L, out)
    return out


def position_rows(ids, pad_id, max_pos):
    """Position-table rows of one sentence (BERT rows 0..L-1 for pad_id < 0, else the
    bge-m3 / XLM-R rows)."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    rows = np.empty(ids.size, np.int32)
    load("port").fe_oracle_position_rows(ids, ids.size, pad_id, max_pos, rows)
    return rows


def uniform_mt19937(count, seed=42, lo=-1.0, hi=1.0):
    """std::mt19937(seed) + uniform_real_distribution<float>(lo, hi): the generator
    of the reference's GTest inputs (tests/*_ops_test.cpp)."""
    out = np.empty(int(count), np.float32)
    load("port").fe_oracle_fill_uniform_mt19937(seed, lo, hi, out, out.size)
    return out


# ---------------- model-level ----------------
class Model:
    """ctypes view of a weight dict (HF names) as the oracle's fe_oracle_bert."""

    def __init__(self, shape, weights: dict):
        self.shape = shape
        self._keep = {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in weights.items()}
        P = lambda name: self._keep[name].ctypes.data_as(C.POINTER(C.c_float))
        layers = (Layer * shape.layers)()
        for l in range(shape.layers):
            p = f"encoder.layer.{l}."
            layers[l] = Layer(
                P(p + "attention.self.query.weight"), P(p + "attention.self.query.bias"),
                P(p + "attention.self.key.weight"), P(p + "attention.self.key.bias"),
                P(p + "attention.self.value.weight"), P(p + "attention.self.value.bias"),
                P(p + "attention.output.dense.weight"), P(p + "attention.output.dense.bias"),
                P(p + "attention.output.LayerNorm.weight"), P(p + "attention.output.LayerNorm.bias"),
                P(p + "intermediate.dense.weight"), P(p + "intermediate.dense.bias"),
                P(p + "output.dense.weight"), P(p + "output.dense.bias"),
                P(p + "output.LayerNorm.weight"), P(p + "output.LayerNorm.bias"))
        self._layers = layers
        self.struct = Bert(shape.vocab, shape.hidden, shape.heads, shape.intermediate,
                           shape.layers, shape.max_pos, shape.type_vocab, ACTS[shape.act],
                           shape.eps, P("embeddings.word_embeddings.weight"),
                           P("embeddings.position_embeddings.weight"),
                           P("embeddings.token_type_embeddings.weight"),
                           P("embeddings.LayerNorm.weight"), P("embeddings.LayerNorm.bias"),
                           C.cast(layers, C.POINTER(Layer)), getattr(shape, "pad_id", -1))

    def forward(self, ids, kind="port"):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(self.shape.hidden, np.float32)
        rc = _fn(kind, "bert_forward")(C.byref(self.struct), ids, ids.size, out)
        if rc != 0:
            raise ValueError(f"oracle forward failed with status {rc}")
        return out

    def forward_batch(self, ids, lengths, kind="port", threads=None):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        lengths = np.ascontiguousarray(lengths, dtype=np.int32)
        B, S = ids.shape
        out = np.empty((B, self.shape.hidden), np.float32)
        threads = threads or os.cpu_count() or 1
        rc = _fn(kind, "bert_forward_batch")(C.byref(self.struct), ids.ravel(), lengths, B, S,
                                             out.ravel(), threads)
        if rc != 0:
            raise ValueError(f"oracle batch forward failed with status {rc}")
        return out


# ---------------- tokenizer ----------------
class RefTokenizer:
    """The reference's own BGETokenizer (oracle/_ref/libfe_ref_tok.so: src/tokenizer.cpp
    compiled unmodified, driven by ref_tokenizer.cpp) with the [CLS] / [SEP] framing of
    SentenceTransformerImpl::tokenize (src/sentence_transformers_impl.cpp:11-27)."""

    PATH = os.path.join(HERE, "_ref", "libfe_ref_tok.so")

    @classmethod
    def available(cls) -> bool:
        return os.path.exists(cls.PATH)

    def __init__(self, vocab_path: str):
        lib = C.CDLL(self.PATH)
        lib.fe_ref_tok_create.argtypes = [C.c_char_p]
        lib.fe_ref_tok_create.restype = C.c_void_p
        lib.fe_ref_tok_destroy.argtypes = [C.c_void_p]
        lib.fe_ref_tok_destroy.restype = None
        lib.fe_ref_tok_encode.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, _i32p, C.c_size_t]
        lib.fe_ref_tok_encode.restype = C.c_long
        self._lib = lib
        self._h = lib.fe_ref_tok_create(vocab_path.encode())
        if not self._h:
            raise ValueError(f"the reference tokenizer rejected {vocab_path}")

    def encode(self, text: bytes) -> list[int]:
        buf = np.empty(4 * len(text) + 8, np.int32)
        n = self._lib.fe_ref_tok_encode(self._h, text, len(text), buf, buf.size)
        if n < 0 or n > buf.size:
            raise ValueError("the reference tokenizer failed")
        return buf[:n].tolist()

    def close(self) -> None:
        if self._h:
            self._lib.fe_ref_tok_destroy(self._h)
            self._h = None
