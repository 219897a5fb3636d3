"""The oracle, pinned: the C restatement (oracle/fe_oracle.c) must agree bit for bit
with the reference's own CPU ops (oracle/_ref, compiled from the reference sources)
and with the golden vectors those ops produced (tests/golden/, made by
tests/golden/gen_golden.py).  CPU only."""
import json
import os

import numpy as np
import pytest

from tests.golden import gen_golden as G

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


@pytest.fixture(scope="module")
def golden_ops():
    return np.load(os.path.join(GOLD, "ops_ref.npz"))


def test_ops_match_golden_vectors(oracle_lib, golden_ops):
    O = oracle_lib
    for (m, n, k) in G.MATMUL_SIZES:
        a, b = O.uniform_mt19937(m * n), O.uniform_mt19937(n * k)
        assert np.array_equal(O.matmul_nn(a, b, m, n, k), golden_ops[f"matmul_nn_{m}x{n}x{k}"])
        assert np.array_equal(O.matmul_nt(a, b, m, n, k), golden_ops[f"matmul_nt_{m}x{n}x{k}"])
    meta = json.load(open(os.path.join(GOLD, "ops_ref.json")))
    for n in G.RELU_SIZES:
        r = O.unary("relu", O.uniform_mt19937(n))
        assert G.sha(r) == meta[f"relu_{n}_sha256"]
    v = np.array(G.GELU_VALUES, np.float32)
    assert np.array_equal(O.unary("gelu", v), golden_ops["gelu_values"])
    assert np.array_equal(O.unary("swish", v), golden_ops["swish_values"])
    for d in G.LN_DIMS:
        x, g, b = O.uniform_mt19937(10 * d), O.uniform_mt19937(d), O.uniform_mt19937(d)
        for eps in G.LN_EPS:
            assert np.array_equal(O.layer_norm(x, g, b, d, eps), golden_ops[f"layer_norm_{d}_{eps:g}"])
        assert np.array_equal(O.rms_norm(x, g, d, 1e-5), golden_ops[f"rms_norm_{d}"])
        assert np.array_equal(O.softmax_rows(x, d), golden_ops[f"softmax_{d}"])
    for (L, D, H) in G.MHA_CASES:
        x, w, b = O.uniform_mt19937(L * D), O.uniform_mt19937(D * D), O.uniform_mt19937(D)
        assert np.array_equal(O.mha(x, w, w, w, b, b, b, H, D), golden_ops[f"mha_{L}_{D}_{H}"])


def test_generator_matches_reference_test_stream(oracle_lib):
    """First values of std::mt19937(42) through uniform_real_distribution<float>(-1,1)
    (the reference GTests' inputs)."""
    u = oracle_lib.uniform_mt19937(4)
    assert u.dtype == np.float32 and u.size == 4
    assert np.all(np.abs(u) <= 1.0)
    # each fresh generator restarts the stream: a shorter tensor is a prefix of a longer one
    assert np.array_equal(oracle_lib.uniform_mt19937(64)[:4], u)


@pytest.mark.parametrize("case", [(3, 17, 29), (64, 64, 64), (5, 1024, 7)])
def test_port_equals_reference_random_inputs(oracle_lib, case):
    O = oracle_lib
    if not O.available("ref"):
        pytest.skip("oracle/_ref not built here (reference sources absent); golden vectors still pin the port")
    m, n, k = case
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal(m * n).astype(np.float32)
    b = rng.standard_normal(n * k).astype(np.float32)
    assert np.array_equal(O.matmul_nt(a, b, m, n, k), O.matmul_nt(a, b, m, n, k, kind="ref"))
    assert np.array_equal(O.matmul_nn(a, b, m, n, k), O.matmul_nn(a, b, m, n, k, kind="ref"))
    x = (rng.standard_normal(n * 6) * 5).astype(np.float32)
    for name in ("gelu", "relu", "swish"):
        assert np.array_equal(O.unary(name, x), O.unary(name, x, kind="ref"))
    g = rng.standard_normal(n).astype(np.float32)
    bb = rng.standard_normal(n).astype(np.float32)
    assert np.array_equal(O.layer_norm(x, g, bb, n, 1e-12), O.layer_norm(x, g, bb, n, 1e-12, kind="ref"))
    assert np.array_equal(O.rms_norm(x, g, n, 1e-6), O.rms_norm(x, g, n, 1e-6, kind="ref"))
    assert np.array_equal(O.softmax_rows(x, n), O.softmax_rows(x, n, kind="ref"))


def test_port_equals_reference_forward(oracle_lib):
    O = oracle_lib
    if not O.available("ref"):
        pytest.skip("oracle/_ref not built here")
    import dataclasses
    from fastembed_b200 import workload as W
    shape = dataclasses.replace(W.SHAPES["bge-small"], layers=2, hidden=256, heads=4, intermediate=512,
                                vocab=500, act="gelu")
    w = W.make_weights(shape, seed=3)
    lengths = np.array([1, 2, 9, 40], np.int32)
    ids, _ = W.sample_ids(shape, lengths, seed=5, pad_to=40)
    m = O.Model(shape, w)
    assert np.array_equal(m.forward_batch(ids, lengths), m.forward_batch(ids, lengths, kind="ref"))
    for act in ("relu", "swish"):
        s2 = dataclasses.replace(shape, act=act)
        m2 = O.Model(s2, w)
        assert np.array_equal(m2.forward_batch(ids, lengths), m2.forward_batch(ids, lengths, kind="ref"))


@pytest.mark.parametrize("name,subset", [("bge-small", None), ("bge-base", "shortest")])
def test_model_golden(oracle_lib, name, subset):
    """The port reproduces the reference forward's stored embeddings bit for bit."""
    from fastembed_b200 import workload as W
    gold = np.load(os.path.join(GOLD, f"model_{name}.npz"))
    shape = W.SHAPES[name]
    weights = W.make_weights(shape)
    assert G.weights_hash(weights) == str(gold["weights_sha256"]), "weight generator changed"
    lengths = W.sample_lengths(shape)
    ids, _ = W.sample_ids(shape, lengths)
    assert G.sha(ids) == str(gold["ids_sha256"]), "id generator changed"
    idx = gold["index"]
    emb = gold["embeddings"]
    if subset == "shortest":
        j = int(np.argmin(gold["lengths"]))
        idx, emb = idx[j:j + 1], emb[j:j + 1]
    got = oracle_lib.Model(shape, weights).forward_batch(ids[idx], lengths[idx])
    assert np.array_equal(got, emb)


def test_forward_rejects_overlong_and_bad_ids(oracle_lib):
    import dataclasses
    from fastembed_b200 import workload as W
    shape = dataclasses.replace(W.SHAPES["bge-small"], layers=1, hidden=128, heads=2, intermediate=256,
                                vocab=300, max_pos=16)
    m = oracle_lib.Model(shape, W.make_weights(shape, seed=1))
    with pytest.raises(ValueError):
        m.forward(np.full(17, 120, np.int32))
    with pytest.raises(ValueError):
        m.forward(np.array([101, 300, 102], np.int32))


def test_xlmr_position_rows(oracle_lib):
    """bge-m3 / XLM-R rows (src/sentence_transformers_impl.cpp:101-123, :146-149): pad tokens
    row 0, the others 2, 3, ... in order, a row at or past the table row 0; BERT rows 0..L-1."""
    O = oracle_lib
    ids = np.array([0, 5, 1, 7, 1, 1, 9, 2], np.int32)
    assert O.position_rows(ids, -1, 512).tolist() == list(range(8))
    assert O.position_rows(ids, 1, 512).tolist() == [2, 3, 0, 4, 0, 0, 5, 6]
    assert O.position_rows(ids, 0, 512).tolist() == [0, 2, 3, 4, 5, 6, 7, 8]
    assert O.position_rows(ids, 1, 5).tolist() == [2, 3, 0, 4, 0, 0, 0, 0]  # rows >= 5 become 0
    rng = np.random.default_rng(3)
    for _ in range(50):
        L, pad, maxp = int(rng.integers(1, 60)), int(rng.integers(0, 4)), int(rng.integers(2, 70))
        x = rng.integers(0, 4, L).astype(np.int32)
        want, nxt = [], 2
        for v in x:
            r = 0 if v == pad else nxt
            nxt += v != pad
            want.append(r if r < maxp else 0)
        assert O.position_rows(x, pad, maxp).tolist() == want


def test_port_equals_reference_forward_xlmr(oracle_lib):
    """The bge-m3 position path of the port equals the reference-ops driver bit for bit,
    with pad ids inside sentences and rows running past the table."""
    O = oracle_lib
    if not O.available("ref"):
        pytest.skip("oracle/_ref not built here")
    import dataclasses
    from fastembed_b200 import workload as W
    shape = dataclasses.replace(W.SHAPES["bge-small"], layers=2, hidden=256, heads=4, intermediate=512,
                                vocab=500, max_pos=48, type_vocab=1, pad_id=1)
    w = W.make_weights(shape, seed=8)
    lengths = np.array([1, 3, 17, 48], np.int32)
    ids, _ = W.sample_ids(shape, lengths, seed=9, pad_to=48)
    ids[1, 1] = 1
    ids[2, [0, 5, 6]] = 1
    ids[3, 10:14] = 1
    m = O.Model(shape, w)
    got = m.forward_batch(ids, lengths)
    assert np.array_equal(got, m.forward_batch(ids, lengths, kind="ref"))
    # the rows differ from the BERT ones, so the outputs do
    bert = O.Model(dataclasses.replace(shape, pad_id=-1), w).forward_batch(ids, lengths)
    assert not np.allclose(got, bert)
