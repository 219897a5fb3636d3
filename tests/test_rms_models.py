"""Qwen3- and Gemma3-shaped encoders (pre-RMSNorm, rotary, grouped-query attention,
gated MLP).  Not in the reference; the oracle is transformers' Qwen3Model /
Gemma3TextModel on the CPU in FP32 (oracle/hf_oracle.py), pinned by committed
golden embeddings (tests/golden/gen_golden_rms.py).

Tolerance against the FP32 oracle, as for the BERT encoders: per-embedding cosine
>= 0.9999 and max-abs <= 2e-3 (bf16 tensor-core inputs, fp32 accumulation, fp32 residual
stream and norms)."""
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
SHAPES = ("qwen3-tiny", "gemma3-tiny")
FULL = ("qwen3-0.6b", "gemma-300m")  # the benchmark shapes at full depth


def _golden(name):
    return np.load(os.path.join(HERE, "golden", f"model_{name}.npz"))


def _close(got, ref):
    cos = (got * ref).sum(1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(ref, axis=1))
    return float(cos.min()), float(np.abs(got - ref).max())


@pytest.mark.parametrize("name", SHAPES)
def test_golden_inputs_regenerate(name):
    from tests.golden import gen_golden_rms as G
    g = _golden(name)
    shape, weights, lengths, ids = G.inputs(name)
    assert np.array_equal(g["lengths"], lengths) and np.array_equal(g["ids"], ids)
    assert str(g["digest"]) == G.digest(weights, ids)


@pytest.mark.parametrize("name", SHAPES)
def test_hf_oracle_reproduces_golden(name):
    from oracle import hf_oracle as H
    from tests.golden import gen_golden_rms as G
    shape, weights, lengths, ids = G.inputs(name)
    emb = H.embed(shape, weights, ids, lengths)
    assert np.allclose(emb, _golden(name)["embeddings"], atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("name", SHAPES)
def test_engine_matches_golden(cuda_dev, name):
    from fastembed_b200 import ops
    from tests.golden import gen_golden_rms as G
    shape, weights, lengths, ids = G.inputs(name)
    eng = ops.Engine(shape, 0)
    eng.load_weights(weights)
    got = eng.encode_host(ids, lengths)
    cmin, err = _close(got, _golden(name)["embeddings"])
    assert cmin >= 0.9999 and err <= 2e-3, (cmin, err)
    # batch invariance: one sentence alone equals its row of the batch
    one = eng.encode_host(ids[3:4], lengths[3:4])
    assert np.array_equal(one[0], got[3])
    eng.close()
    ops.device_status(0)


@pytest.mark.gpu
@pytest.mark.parametrize("name", SHAPES)
def test_engine_matches_hf_edge_lengths(cuda_dev, name):
    """Fresh weights and edge lengths (1, tile boundaries 128 / 129 / 256, multi-tile)
    against transformers run here on the CPU."""
    pytest.importorskip("transformers")
    from fastembed_b200 import ops, workload as W
    from oracle import hf_oracle as H
    shape = W.RMS_SHAPES[name]
    weights = W.make_rms_weights(shape, seed=5, norm_jitter=0.2)
    lengths = np.array([1, 2, 128, 129, 256, 257, 390], np.int32)
    ids = W.sample_rms_ids(shape, lengths, seed=7)
    ref = H.embed(shape, weights, ids, lengths)
    eng = ops.Engine(shape, 0)
    eng.load_weights(weights)
    got = eng.encode_host(ids, lengths)
    eng.close()
    cmin, err = _close(got, ref)
    assert cmin >= 0.9999 and err <= 2e-3, (cmin, err)
    ops.device_status(0)


@pytest.mark.parametrize("name", FULL)
def test_full_golden_inputs_regenerate(name):
    """The full-shape goldens were made from the benchmark's weights and batch."""
    from tests.golden import gen_golden_rms as G
    g = _golden(name)
    shape, weights, lengths, ids, index = G.full_inputs(name)
    assert np.array_equal(g["index"], index) and np.array_equal(g["lengths"], lengths[index])
    assert str(g["digest"]) == G.digest(weights, ids)
    e = _golden(f"{name}-edge")
    el, eids = G.edge_inputs(shape)
    assert np.array_equal(e["lengths"], el) and str(e["digest"]) == G.digest(weights, eids)


@pytest.mark.gpu
@pytest.mark.parametrize("name", FULL)
def test_engine_matches_full_depth_golden(cuda_dev, name):
    """The Qwen3-0.6B shape (28 layers x 1024, causal GQA, bf16-valued weights, 128
    sentences of U[64, 1024] tokens) and the EmbeddingGemma-300M shape (24 layers x 768,
    512 sentences of U[8, 256]) at full depth: the stored sentences (every 16th / 32nd
    of the batch by length, the longest included) run inside the whole benchmark batch,
    then an edge set up to 1024 tokens; each against transformers in FP32."""
    from fastembed_b200 import ops
    from tests.golden import gen_golden_rms as G
    g = _golden(name)
    shape, weights, lengths, ids, index = G.full_inputs(name)
    eng = ops.Engine(shape, 0)
    eng.load_weights(weights)
    got = eng.encode_host(ids, lengths)[index]
    cmin, err = _close(got, g["embeddings"])
    print(f"{name}: {index.size} sentences of the batch, min cos {cmin:.7f}, max abs {err:.3e}")
    assert cmin >= 0.9999 and err <= 2e-3, (cmin, err)
    e = _golden(f"{name}-edge")
    el, eids = G.edge_inputs(shape)
    got = eng.encode_host(eids, el)
    cmin, err = _close(got, e["embeddings"])
    print(f"{name}: edge lengths {el.tolist()}, min cos {cmin:.7f}, max abs {err:.3e}")
    assert cmin >= 0.9999 and err <= 2e-3, (cmin, err)
    eng.close()
    ops.device_status(0)
