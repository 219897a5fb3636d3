"""Model-level parity: the engine's embeddings against the oracle (the reference's
CPU FP32 forward, unpadded per sentence) on identical seeded weights and ids.

Tolerance (stated for the TF32/BF16 tensor-core path): per-embedding cosine
>= 0.9999 and max-abs error <= 2e-3."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

COS_MIN = 0.9999
MAXABS = 2e-3


def _check(got, ref):
    cos = (got * ref).sum(1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(ref, axis=1))
    assert cos.min() >= COS_MIN, cos.min()
    assert np.abs(got - ref).max() <= MAXABS, np.abs(got - ref).max()


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
