"""Model-level parity: the engine's embeddings against the oracle (the reference's
CPU FP32 forward, unpadded per sentence) on identical seeded weights and ids.

Tolerance (stated for the TF32/BF16 tensor-core path): per-embedding cosine
>= 0.9999 and max-abs error <= 2e-3."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

COS_MIN = 0.9999
MAXABS = 2e-3


def _check(got, ref, label=""):
    cos = (got * ref).sum(1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(ref, axis=1))
    err = np.abs(got - ref).max(axis=1)
    print(f"{label}: {got.shape[0]} sentences, min cos {cos.min():.7f}, max abs {err.max():.3e}")
    assert cos.min() >= COS_MIN, cos.min()
    assert err.max() <= MAXABS, err.max()


def test_bge_small_batch_matches_oracle(cuda_dev, oracle_lib):
    from fastembed_b200 import ops, workload as W
    shape = W.SHAPES["bge-small"]
    weights = W.make_weights(shape)
    lengths = W.sample_lengths(shape)
    ids, mask = W.sample_ids(shape, lengths)
    ref = oracle_lib.Model(shape, weights).forward_batch(ids, lengths)
    eng = ops.Engine(shape, 0)
    eng.load_weights(weights)
    got = eng.encode_host(ids, lengths)
    _check(got, ref)
    # bit-exact batch invariance: each sentence alone gives the same vector
    for b in (0, 3, 7):
        one = eng.encode_host(ids[b:b + 1], lengths[b:b + 1])
        assert np.array_equal(one[0], got[b])
    eng.close()


def test_edge_lengths_match_oracle(cuda_dev, oracle_lib):
    """Lengths 1, 2, 127, 128, 129 and the position-table maximum 512."""
    from fastembed_b200 import ops, workload as W
    import dataclasses
    shape = dataclasses.replace(W.SHAPES["bge-small"], layers=2)
    weights = W.make_weights(shape, seed=4)
    lengths = np.array([1, 2, 127, 128, 129, 512], np.int32)
    ids, _ = W.sample_ids(shape, lengths, seed=7, pad_to=512)
    ref = oracle_lib.Model(shape, weights).forward_batch(ids, lengths)
    eng = ops.Engine(shape, 0)
    eng.load_weights(weights)
    _check(eng.encode_host(ids, lengths), ref)
    eng.close()


def test_rejects_too_long_and_bad_ids(cuda_dev):
    from fastembed_b200 import ops, workload as W
    from fastembed_b200.capi import FeError
    import dataclasses
    shape = dataclasses.replace(W.SHAPES["bge-small"], layers=1)
    eng = ops.Engine(shape, 0)
    eng.load_weights(W.make_weights(shape, seed=2))
    ids = np.full((1, 513), 200, np.int32)
    with pytest.raises(FeError):  # longer than the position table (sentence_transformers_impl.cpp:132-136)
        eng.encode_host(ids, np.array([513], np.int32))
    bad = np.full((1, 4), 200, np.int32)
    bad[0, 2] = shape.vocab + 5
    with pytest.raises(FeError):
        eng.encode_host(bad, np.array([4], np.int32))
    # the engine stays usable after a rejected call
    ok = eng.encode_host(np.full((1, 4), 200, np.int32), np.array([4], np.int32))
    assert abs(float(np.linalg.norm(ok)) - 1.0) < 1e-5
    eng.close()


@pytest.mark.parametrize("name", ["bge-small", "bge-base", "bge-large"])
def test_engine_matches_reference_golden(cuda_dev, name):
    """Stored embeddings of the reference's own CPU forward (tests/golden/model_*.npz:
    every sentence of the bge-small and bge-base batches, and every 8th sentence of the
    length-sorted bge-large batch, 32 of 256, the longest included) on the same seeded
    weights and ids; the sentences run inside their full batch on the GPU, and every
    stored sentence must meet the tolerance."""
    import os
    from fastembed_b200 import ops, workload as W
    from tests.golden import gen_golden as G
    gold = np.load(os.path.join(os.path.dirname(__file__), "golden", f"model_{name}.npz"))
    shape = W.SHAPES[name]
    weights = W.make_weights(shape)
    assert G.weights_hash(weights) == str(gold["weights_sha256"]), "weight generator changed"
    lengths = W.sample_lengths(shape)
    ids, _ = W.sample_ids(shape, lengths)
    assert G.sha(ids) == str(gold["ids_sha256"]), "id generator changed"
    eng = ops.Engine(shape, 0)
    eng.load_weights(weights)
    got = eng.encode_host(ids, lengths)
    assert np.array_equal(lengths[gold["index"]], gold["lengths"])
    _check(got[gold["index"]], gold["embeddings"], name)
    eng.close()


def test_engine_matches_reference_golden_edge_lengths(cuda_dev):
    """The full 24-layer bge-large shape at the position-table maximum (512 tokens), the
    query-tile boundaries 128 / 129 / 257 and one- and two-token sentences, against the
    reference's own CPU forward (tests/golden/model_bge-large-edge.npz)."""
    import os
    from fastembed_b200 import ops, workload as W
    from tests.golden import gen_golden as G
    gold = np.load(os.path.join(os.path.dirname(__file__), "golden", "model_bge-large-edge.npz"))
    shape = W.SHAPES["bge-large"]
    weights = W.make_weights(shape)
    assert G.weights_hash(weights) == str(gold["weights_sha256"]), "weight generator changed"
    lengths, ids = G.edge_inputs(shape)
    assert G.sha(ids) == str(gold["ids_sha256"]), "id generator changed"
    assert np.array_equal(lengths, gold["lengths"])
    eng = ops.Engine(shape, 0)
    eng.load_weights(weights)
    _check(eng.encode_host(ids, lengths), gold["embeddings"], "bge-large edge")
    eng.close()


def test_full_batch_properties_bge_large(cuda_dev):
    """Size-independent checks at the benchmark's full size (256 sentences): unit
    norms, run-to-run determinism, and bit-exact invariance to batch order and
    composition (each sentence's result does not depend on its neighbours)."""
    from fastembed_b200 import ops, workload as W
    shape = W.SHAPES["bge-large"]
    weights = W.make_weights(shape)
    lengths = W.sample_lengths(shape)
    ids, _ = W.sample_ids(shape, lengths)
    eng = ops.Engine(shape, 0)
    eng.load_weights(weights)
    a = eng.encode_host(ids, lengths)
    b = eng.encode_host(ids, lengths)
    assert np.array_equal(a, b)
    assert np.abs(np.linalg.norm(a, axis=1) - 1).max() < 1e-5
    perm = np.random.default_rng(0).permutation(lengths.size)
    c = eng.encode_host(ids[perm], lengths[perm])
    assert np.array_equal(c, a[perm])
    d = eng.encode_host(ids[17:40], lengths[17:40])
    assert np.array_equal(d, a[17:40])
    eng.close()


def test_xlmr_positions_match_oracle(cuda_dev, oracle_lib):
    """bge-m3 / XLM-R position rows (model_type "xlm-roberta", pad_token_id 1): pad ids
    inside sentences take row 0, the others rows 2, 3, ...; rows past the 48-row table
    become row 0 (sentence_transformers_impl.cpp:101-123, :139-155)."""
    from fastembed_b200 import ops, workload as W
    import dataclasses
    shape = dataclasses.replace(W.SHAPES["bge-small"], layers=2, max_pos=48, type_vocab=1, pad_id=1)
    weights = W.make_weights(shape, seed=21)
    lengths = np.array([1, 2, 5, 33, 46, 47, 48, 40], np.int32)
    ids, _ = W.sample_ids(shape, lengths, seed=22, pad_to=48)
    ids[2, 2] = 1
    ids[3, [0, 7, 8, 30]] = 1
    ids[7, 5:25] = 1
    ref = oracle_lib.Model(shape, weights).forward_batch(ids, lengths)
    eng = ops.Engine(shape, 0)
    eng.load_weights(weights)
    got = eng.encode_host(ids, lengths)
    _check(got, ref)
    for b in (3, 7):  # batch invariance, bit for bit
        assert np.array_equal(eng.encode_host(ids[b:b + 1], lengths[b:b + 1])[0], got[b])
    eng.close()


def test_host_encode_runs_large_batches_in_passes(cuda_dev, oracle_lib, monkeypatch):
    """fe_engine_encode_host splits a batch into device passes of at most
    FE_MAX_TOKENS_PER_PASS tokens (a longer sentence runs alone), so memory stays bounded
    for any batch.  With a 100-token cap the 40 sentences run in many passes: rows match
    the one-pass result within fp32 rounding (small passes take the 1-CTA GEMM and the
    two-launch norm) and the oracle within the model tolerance."""
    from fastembed_b200 import ops, workload as W
    import dataclasses
    shape = dataclasses.replace(W.SHAPES["bge-small"], layers=2)
    weights = W.make_weights(shape, seed=21)
    lengths = W.sample_lengths(shape, batch=40, seed=22)
    lengths[5] = 128  # longer than the cap: a pass of its own
    ids, _ = W.sample_ids(shape, lengths, seed=23, pad_to=128)
    eng = ops.Engine(shape, 0)
    eng.load_weights(weights)
    one_pass = eng.encode_host(ids, lengths)
    monkeypatch.setenv("FE_MAX_TOKENS_PER_PASS", "100")
    passes = eng.encode_host(ids, lengths)
    eng.close()
    assert np.abs(passes - one_pass).max() <= 1e-5
    _check(passes, oracle_lib.Model(shape, weights).forward_batch(ids, lengths))


def test_host_encode_more_sentences_than_one_pass_takes(cuda_dev):
    """70,000 two-token sentences: more than a device pass takes (65,535), so the call
    runs two passes.  The rows around the boundary equal a separate small call within
    fp32 rounding."""
    from fastembed_b200 import ops, workload as W
    import dataclasses
    shape = dataclasses.replace(W.SHAPES["bge-small"], layers=1)
    eng = ops.Engine(shape, 0)
    eng.load_weights(W.make_weights(shape, seed=31))
    rng = np.random.default_rng(32)
    n = 70000
    ids = np.stack([np.full(n, 101), rng.integers(1000, shape.vocab, n)], 1).astype(np.int32)
    lengths = np.full(n, 2, np.int32)
    out = eng.encode_host(ids, lengths)
    assert out.shape == (n, shape.hidden) and np.isfinite(out).all()
    lo, hi = 65530, 65541
    part = eng.encode_host(ids[lo:hi], lengths[lo:hi])
    eng.close()
    assert np.abs(out[lo:hi] - part).max() <= 1e-5


@pytest.mark.parametrize("family", ["bert", "qwen3", "gemma3"])
def test_empty_sentence_in_batch(cuda_dev, family):
    """A zero-length sentence inside a batch gives a zero row and leaves every other row
    as the batch without it gives it (bit for bit: the same passes run on the same tokens)."""
    from fastembed_b200 import ops, workload as W
    import dataclasses
    if family == "bert":
        shape = dataclasses.replace(W.SHAPES["bge-small"], layers=2)
        weights = W.make_weights(shape, seed=41)
        lengths = np.array([5, 0, 17, 0, 9], np.int32)
        ids, _ = W.sample_ids(shape, np.maximum(lengths, 2), seed=42, pad_to=32)  # rows of length 0 unused
    else:
        shape = W.RMS_SHAPES["qwen3-tiny" if family == "qwen3" else "gemma3-tiny"]
        weights = W.make_rms_weights(shape, seed=41)
        lengths = np.array([5, 0, 17, 0, 9], np.int32)
        ids = W.sample_rms_ids(shape, np.maximum(lengths, 2), seed=42)
    eng = ops.Engine(shape, 0)
    eng.load_weights(weights)
    got = eng.encode_host(ids, lengths)
    keep = lengths > 0
    ref = eng.encode_host(ids[keep], lengths[keep])
    eng.close()
    assert np.all(got[~keep] == 0)
    assert np.array_equal(got[keep], ref)
