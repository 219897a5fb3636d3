"""Synthetic encoder workloads: model shapes, sentence lengths, token ids, weights.

The reference publishes no dataset or checkpoint for its benchmarks, so every
workload is synthetic and seeded:

* weights ~ N(0, 0.02) (seed 0), LayerNorm gamma = 1, beta = 0, biases N(0, 0.02),
  named exactly as the reference reads them from model.safetensors
  (src/sentence_transformers_impl.cpp:33, :132, :171, :192-193, :201-218, :285-286);
* token ids uniform in [100, vocab) with [CLS]=101 first and [SEP]=102 last, the
  framing the reference's tokenize() adds (src/sentence_transformers_impl.cpp:21-22);
  input seed 1;
* sentence lengths per shape below; sentences run unpadded (packed) on the device.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np

CLS_ID = 101
SEP_ID = 102
PAD_ID = 0


@dataclasses.dataclass(frozen=True)
class EncoderShape:
    name: str
    layers: int
    hidden: int
    heads: int
    intermediate: int
    vocab: int = 21128
    max_pos: int = 512
    type_vocab: int = 2
    eps: float = 1e-12
    act: str = "gelu"
    batch: int = 8
    lengths: tuple = ("uniform", 16, 128)
    pad_to: int = 128
    pad_id: int = -1  # >= 0: bge-m3 / XLM-R position rows with this pad_token_id

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    def flops_per_sentence(self, length: int) -> float:
        """Algorithmic FLOPs of one unpadded sentence:
        layers * [2 L (4 D^2 + 2 D F) + 4 L^2 D] (projections + QK^T + PV)."""
        D, F, L = self.hidden, self.intermediate, length
        return self.layers * (2.0 * L * (4 * D * D + 2 * D * F) + 4.0 * L * L * D)

    def gemm_flops_per_sentence(self, length: int) -> float:
        D, F, L = self.hidden, self.intermediate, length
        return self.layers * 2.0 * L * (4 * D * D + 2 * D * F)

    def attn_flops_per_sentence(self, length: int) -> float:
        return self.layers * 4.0 * length * length * self.hidden

    def shard_cost(self, length: int) -> float:
        """The cost fe_plan_shards balances, in projection FLOPs: the GEMM FLOPs plus, per
        head and layer, three times the full-tile FLOPs (4 x 128 x 128 x head_dim) for each
        (128-query, 128-key) attention tile the sentence occupies (the attention kernel's time
        goes by tiles, and a tile takes about that long at the projections' rate)."""
        tiles = -(-int(length) // 128)
        return self.gemm_flops_per_sentence(length) + self.layers * self.heads * tiles * tiles * 3.0 * 4.0 * 128 * 128 * self.head_dim


SHAPES = {
    # BGE-small-zh shape: 4 layers, D 512, 8 heads, FFN 2048; batch 8, L ~ U[16,128]
    "bge-small": EncoderShape("bge-small", 4, 512, 8, 2048, batch=8,
                              lengths=("uniform", 16, 128), pad_to=128),
    # BGE-base-zh shape: 12 layers, D 768, 12 heads, FFN 3072; batch 64, L ~ U[32,512]
    "bge-base": EncoderShape("bge-base", 12, 768, 12, 3072, batch=64,
                             lengths=("uniform", 32, 512), pad_to=512),
    # BGE-large-zh shape: 24 layers, D 1024, 16 heads, FFN 4096; batch 256,
    # L ~ lognormal(median 96, sigma 0.6) truncated to [8, 512]
    "bge-large": EncoderShape("bge-large", 24, 1024, 16, 4096, batch=256,
                              lengths=("lognormal", 96, 0.6, 8, 512), pad_to=512),
}


def sample_lengths(shape: EncoderShape, batch: int | None = None, seed: int = 1) -> np.ndarray:
    """Sentence lengths (including [CLS] and [SEP]) for `batch` sentences."""
    rng = np.random.default_rng(seed)
    b = shape.batch if batch is None else batch
    kind = shape.lengths[0]
    if kind == "uniform":
        lo, hi = shape.lengths[1], shape.lengths[2]
        return rng.integers(lo, hi + 1, size=b).astype(np.int32)
    if kind == "lognormal":
        median, sigma, lo, hi = shape.lengths[1:]
        out = np.empty(b, dtype=np.int32)
        n = 0
        while n < b:  # rejection-truncate to [lo, hi]
            v = np.round(rng.lognormal(math.log(median), sigma, size=2 * b)).astype(np.int64)
            v = v[(v >= lo) & (v <= hi)]
            take = min(b - n, v.size)
            out[n:n + take] = v[:take]
            n += take
        return out
    raise ValueError(f"unknown length distribution {kind!r}")


def sample_ids(shape: EncoderShape, lengths: np.ndarray, seed: int = 1, pad_to: int | None = None):
    """Right-padded ids [B, S] (PAD=0) and the matching 1/0 attention mask."""
    rng = np.random.default_rng(seed + 1000)
    S = int(max(pad_to or shape.pad_to, int(lengths.max()) if lengths.size else 1))
    B = lengths.size
    ids = np.zeros((B, S), dtype=np.int32)
    mask = np.zeros((B, S), dtype=np.int32)
    for b, L in enumerate(lengths):
        L = int(L)
        row = rng.integers(100, shape.vocab, size=L, dtype=np.int64).astype(np.int32)
        row[0] = CLS_ID
        if L > 1:
            row[L - 1] = SEP_ID
        ids[b, :L] = row
        mask[b, :L] = 1
    return ids, mask


def weight_names(shape: EncoderShape) -> list[tuple[str, tuple[int, ...], str]]:
    """(HF name, shape, init) for every tensor the encoder reads, in a fixed order."""
    D, F = shape.hidden, shape.intermediate
    out = [
        ("embeddings.word_embeddings.weight", (shape.vocab, D), "normal"),
        ("embeddings.position_embeddings.weight", (shape.max_pos, D), "normal"),
        ("embeddings.token_type_embeddings.weight", (shape.type_vocab, D), "normal"),
        ("embeddings.LayerNorm.weight", (D,), "ones"),
        ("embeddings.LayerNorm.bias", (D,), "zeros"),
    ]
    for l in range(shape.layers):
        p = f"encoder.layer.{l}."
        out += [
            (p + "attention.self.query.weight", (D, D), "normal"),
            (p + "attention.self.query.bias", (D,), "normal"),
            (p + "attention.self.key.weight", (D, D), "normal"),
            (p + "attention.self.key.bias", (D,), "normal"),
            (p + "attention.self.value.weight", (D, D), "normal"),
            (p + "attention.self.value.bias", (D,), "normal"),
            (p + "attention.output.dense.weight", (D, D), "normal"),
            (p + "attention.output.dense.bias", (D,), "normal"),
            (p + "attention.output.LayerNorm.weight", (D,), "ones"),
            (p + "attention.output.LayerNorm.bias", (D,), "zeros"),
            (p + "intermediate.dense.weight", (F, D), "normal"),
            (p + "intermediate.dense.bias", (F,), "normal"),
            (p + "output.dense.weight", (D, F), "normal"),
            (p + "output.dense.bias", (D,), "normal"),
            (p + "output.LayerNorm.weight", (D,), "ones"),
            (p + "output.LayerNorm.bias", (D,), "zeros"),
        ]
    out += [("pooler.dense.weight", (D, D), "normal"), ("pooler.dense.bias", (D,), "normal")]
    return out


def make_weights(shape: EncoderShape, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Seeded random-init FP32 weights, keyed by HF tensor name."""
    rng = np.random.default_rng(seed)
    w: dict[str, np.ndarray] = {}
    for name, shp, init in weight_names(shape):
        if init == "normal":
            a = rng.standard_normal(size=shp, dtype=np.float32)
            a *= np.float32(std)
        elif init == "ones":
            a = np.ones(shp, dtype=np.float32)
        else:
            a = np.zeros(shp, dtype=np.float32)
        w[name] = a
    return w


def config_json(shape: EncoderShape) -> dict:
    """The config.json keys the reference reads (src/sentence_transformers_impl.cpp:47-98,
    :189, :199, :240, :268, :413)."""
    xlmr = shape.pad_id >= 0
    return {
        "model_type": "xlm-roberta" if xlmr else "bert",
        "vocab_size": shape.vocab,
        "hidden_size": shape.hidden,
        "num_hidden_layers": shape.layers,
        "num_attention_heads": shape.heads,
        "intermediate_size": shape.intermediate,
        "hidden_act": shape.act,
        "layer_norm_eps": shape.eps,
        "max_position_embeddings": shape.max_pos,
        "type_vocab_size": shape.type_vocab,
        "pad_token_id": shape.pad_id if xlmr else 0,
    }


def balanced_cuts(shape: EncoderShape, sorted_lengths: np.ndarray, parts: int) -> list[int]:
    """Contiguous cut points of a length-sorted batch into `parts` slices whose costs
    (EncoderShape.shard_cost) are as equal as a greedy prefix cut gets them."""
    if parts <= 1:
        return []
    w = np.array([shape.shard_cost(int(L)) for L in sorted_lengths], dtype=np.float64)
    prefix = np.concatenate([[0.0], np.cumsum(w)])  # prefix[i] = work of the first i sentences
    total = prefix[-1]
    cuts: list[int] = []
    for r in range(1, parts):
        target = total * r / parts
        i = int(np.searchsorted(prefix, target))  # prefix[i-1] < target <= prefix[i]
        if i > 0 and (i >= prefix.size or target - prefix[i - 1] <= prefix[i] - target):
            i -= 1
        lo = cuts[-1] if cuts else 0
        cuts.append(int(min(max(i, lo), sorted_lengths.size)))
    return cuts


# ------------------------------------------------ pre-RMSNorm rotary encoders
@dataclasses.dataclass(frozen=True)
class RmsShape:
    """Qwen3 / Gemma3-shaped encoder (not in the reference; built from the model
    definitions).  `family` is "qwen3" (causal, SwiGLU, w norms, last-token pooling) or
    "gemma3" (bidirectional, GeGLU, (1 + w) norms, sandwich norms, mean pooling)."""
    name: str
    family: str
    layers: int
    hidden: int
    q_heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    max_pos: int = 32768
    eps: float = 1e-6
    rope_theta: float = 1e6
    rope_theta_local: float = 1e4
    full_every: int = 0
    batch: int = 8
    lengths: tuple = ("uniform", 16, 128)
    bf16_weights: bool = False  # weights drawn in FP32, then rounded to the nearest bf16 value

    @property
    def pooling(self) -> str:
        return "last" if self.family == "qwen3" else "mean"

    @property
    def causal(self) -> bool:
        return self.family == "qwen3"

    def _qkv(self) -> int:
        return (self.q_heads + 2 * self.kv_heads) * self.head_dim

    def gemm_flops_per_sentence(self, length: int) -> float:
        D, F, L, AO = self.hidden, self.intermediate, length, self.q_heads * self.head_dim
        return self.layers * 2.0 * L * (D * self._qkv() + AO * D + 3 * D * F)

    def attn_flops_per_sentence(self, length: int) -> float:
        pairs = length * (length + 1) / 2 if self.causal else length * length
        return self.layers * 4.0 * pairs * self.q_heads * self.head_dim

    def flops_per_sentence(self, length: int) -> float:
        return self.gemm_flops_per_sentence(length) + self.attn_flops_per_sentence(length)

    def shard_cost(self, length: int) -> float:
        """The cost the shard planner balances (fe_plan_shards_costs): the algorithmic FLOPs;
        these sentences fill most of their attention tiles."""
        return self.flops_per_sentence(length)


RMS_SHAPES = {
    # Qwen3-0.6B shape: 28 layers, D 1024, 16 q / 8 kv heads x 128, FFN 3072 SwiGLU, causal;
    # batch 128, L ~ U[64, 1024]; vocab 151,669; BF16 weights
    "qwen3-0.6b": RmsShape("qwen3-0.6b", "qwen3", 28, 1024, 16, 8, 128, 3072, 151669, batch=128,
                           lengths=("uniform", 64, 1024), bf16_weights=True),
    # Gemma-300M (EmbeddingGemma) shape: 24 layers, D 768, 3 q / 1 kv heads x 256, FFN 1152
    # GeGLU, bidirectional, every 6th layer global; batch 512, L ~ U[8, 256]
    "gemma-300m": RmsShape("gemma-300m", "gemma3", 24, 768, 3, 1, 256, 1152, 262144, max_pos=2048,
                           rope_theta=1e6, rope_theta_local=1e4, full_every=6, batch=512,
                           lengths=("uniform", 8, 256)),
    # two-layer test shapes
    "qwen3-tiny": RmsShape("qwen3-tiny", "qwen3", 2, 256, 4, 2, 128, 384, 1000, batch=6,
                           lengths=("uniform", 1, 300)),
    "gemma3-tiny": RmsShape("gemma3-tiny", "gemma3", 2, 768, 3, 1, 256, 1152, 1000, max_pos=2048, full_every=2,
                            batch=6, lengths=("uniform", 1, 300)),
}


def rms_weight_names(shape: RmsShape) -> list[tuple[str, tuple[int, ...], str]]:
    """(HF name, shape, init) of every tensor of the Qwen3Model / Gemma3TextModel layout.
    Norm weights: Qwen3 multiplies by w (init 1), Gemma3 by (1 + w) (init 0)."""
    D, F, hd = shape.hidden, shape.intermediate, shape.head_dim
    one = "zeros" if shape.family == "gemma3" else "ones"
    out = [("embed_tokens.weight", (shape.vocab, D), "normal")]
    for l in range(shape.layers):
        p = f"layers.{l}."
        out += [
            (p + "self_attn.q_proj.weight", (shape.q_heads * hd, D), "normal"),
            (p + "self_attn.k_proj.weight", (shape.kv_heads * hd, D), "normal"),
            (p + "self_attn.v_proj.weight", (shape.kv_heads * hd, D), "normal"),
            (p + "self_attn.o_proj.weight", (D, shape.q_heads * hd), "normal"),
            (p + "self_attn.q_norm.weight", (hd,), one),
            (p + "self_attn.k_norm.weight", (hd,), one),
            (p + "mlp.gate_proj.weight", (F, D), "normal"),
            (p + "mlp.up_proj.weight", (F, D), "normal"),
            (p + "mlp.down_proj.weight", (D, F), "normal"),
            (p + "input_layernorm.weight", (D,), one),
            (p + "post_attention_layernorm.weight", (D,), one),
        ]
        if shape.family == "gemma3":
            out += [(p + "pre_feedforward_layernorm.weight", (D,), one),
                    (p + "post_feedforward_layernorm.weight", (D,), one)]
    out += [("norm.weight", (D,), one)]
    return out


def round_to_bf16(a: np.ndarray) -> np.ndarray:
    """FP32 values rounded to the nearest bf16 value (ties to even), kept as FP32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def make_rms_weights(shape: RmsShape, seed: int = 0, std: float = 0.02,
                     norm_jitter: float = 0.0) -> dict[str, np.ndarray]:
    """Seeded random-init weights keyed by HF name (FP32 arrays; bf16 values when the
    shape has `bf16_weights`); `norm_jitter` adds N(0, jitter) to the norm weights
    (tests use it so that the weight form matters)."""
    rng = np.random.default_rng(seed)
    w: dict[str, np.ndarray] = {}
    for name, shp, init in rms_weight_names(shape):
        if init == "normal":
            a = rng.standard_normal(size=shp, dtype=np.float32) * np.float32(std)
        else:
            a = np.ones(shp, dtype=np.float32) if init == "ones" else np.zeros(shp, dtype=np.float32)
            if norm_jitter:
                a = a + rng.standard_normal(size=shp, dtype=np.float32) * np.float32(norm_jitter)
        w[name] = round_to_bf16(a) if shape.bf16_weights else a
    return w


def rms_hf_config(shape: RmsShape) -> dict:
    """transformers config keyword arguments of the same model (used by the oracle)."""
    common = dict(vocab_size=shape.vocab, hidden_size=shape.hidden, intermediate_size=shape.intermediate,
                  num_hidden_layers=shape.layers, num_attention_heads=shape.q_heads,
                  num_key_value_heads=shape.kv_heads, head_dim=shape.head_dim,
                  max_position_embeddings=shape.max_pos, rms_norm_eps=shape.eps, attention_bias=False)
    if shape.family == "qwen3":
        return dict(common, rope_theta=shape.rope_theta, hidden_act="silu", tie_word_embeddings=False)
    types = ["full_attention" if shape.full_every and (l + 1) % shape.full_every == 0 else "sliding_attention"
             for l in range(shape.layers)]
    return dict(common, hidden_activation="gelu_pytorch_tanh", use_bidirectional_attention=True,
                query_pre_attn_scalar=shape.head_dim, layer_types=types, sliding_window=2 * shape.max_pos + 1,
                rope_parameters={"full_attention": {"rope_type": "default", "rope_theta": shape.rope_theta},
                                 "sliding_attention": {"rope_type": "default", "rope_theta": shape.rope_theta_local}})


def sample_rms_lengths(shape: RmsShape, batch: int | None = None, seed: int = 1) -> np.ndarray:
    rng = np.random.default_rng(seed)
    _, lo, hi = shape.lengths
    return rng.integers(lo, hi + 1, size=batch or shape.batch).astype(np.int32)


def sample_rms_ids(shape: RmsShape, lengths: np.ndarray, seed: int = 1) -> np.ndarray:
    """Right-padded ids [B, max L] uniform in [100, vocab) (no framing tokens)."""
    rng = np.random.default_rng(seed + 1000)
    S = max(int(lengths.max()) if lengths.size else 1, 1)
    ids = np.zeros((lengths.size, S), dtype=np.int32)
    for b, L in enumerate(lengths):
        ids[b, :int(L)] = rng.integers(100, shape.vocab, size=int(L))
    return ids
