"""Generates the golden vectors under tests/golden/ from the reference itself.

Run here, where the reference sources exist:  make -C oracle && python tests/golden/gen_golden.py

Every output comes from oracle/_ref/libfe_ref.so: the reference's own CPU ops
(src/ops/cpu/cpu_matrix_ops.cpp, cpu_attention_ops.cpp, compiled from its sources)
driven by the restated forward in oracle/ref_forward.cpp.  Inputs are not stored
where they can be regenerated exactly:
  * op cases use the reference GTests' generator (a fresh std::mt19937(42) +
    uniform_real_distribution<float>(-1, 1) per tensor, tests/*_ops_test.cpp);
  * model cases use fastembed_b200.workload's seeded weights and ids; a hash of
    the generated weights is stored so a generator change is caught, not missed.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from fastembed_b200 import workload as W  # noqa: E402

# shapes of tests/matrix_ops_test.cpp:11-17, :62-63, :86-87 and tests/attention_ops_test.cpp:66-71
MATMUL_SIZES = [(2, 2, 2), (4, 5, 6), (16, 16, 16), (1, 1, 1), (100, 200, 300)]
RELU_SIZES = [1, 10, 1000, 1024 * 1024]
GELU_VALUES = [-2.5, -1.0, 0.0, 0.5, 1.0, 3.14]
LN_DIMS = [16, 32, 64, 128, 256, 1024]
LN_EPS = [1e-5, 1e-10]
MHA_CASES = [(10, 64, 4), (10, 128, 8), (10, 512, 16), (10, 1024, 16)]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def weights_hash(w: dict) -> str:
    h = hashlib.sha256()
    for k in sorted(w):
        h.update(k.encode())
        h.update(np.ascontiguousarray(w[k]).tobytes())
    return h.hexdigest()


def gen_ops() -> None:
    out: dict[str, np.ndarray] = {}
    meta: dict[str, str] = {}
    for (m, n, k) in MATMUL_SIZES:
        a = O.uniform_mt19937(m * n)
        b = O.uniform_mt19937(n * k)
        out[f"matmul_nn_{m}x{n}x{k}"] = O.matmul_nn(a, b, m, n, k, kind="ref")
        out[f"matmul_nt_{m}x{n}x{k}"] = O.matmul_nt(a, b, m, n, k, kind="ref")
    for n in RELU_SIZES:
        r = O.unary("relu", O.uniform_mt19937(n), kind="ref")
        if n <= 1000:
            out[f"relu_{n}"] = r
        meta[f"relu_{n}_sha256"] = sha(r)
    out["gelu_values"] = O.unary("gelu", np.array(GELU_VALUES, np.float32), kind="ref")
    out["swish_values"] = O.unary("swish", np.array(GELU_VALUES, np.float32), kind="ref")
    for d in LN_DIMS:
        x = O.uniform_mt19937(10 * d)
        g = O.uniform_mt19937(d)
        b = O.uniform_mt19937(d)
        for eps in LN_EPS:
            out[f"layer_norm_{d}_{eps:g}"] = O.layer_norm(x, g, b, d, eps, kind="ref")
        out[f"rms_norm_{d}"] = O.rms_norm(x, g, d, 1e-5, kind="ref")
        out[f"softmax_{d}"] = O.softmax_rows(x, d, kind="ref")
    for (L, D, H) in MHA_CASES:
        x = O.uniform_mt19937(L * D)
        w = O.uniform_mt19937(D * D)
        b = O.uniform_mt19937(D)
        out[f"mha_{L}_{D}_{H}"] = O.mha(x, w, w, w, b, b, b, H, D, kind="ref")
    np.savez_compressed(os.path.join(HERE, "ops_ref.npz"), **out)
    with open(os.path.join(HERE, "ops_ref.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)


def stride_pick(lengths: np.ndarray, stride: int) -> list[int]:
    """Every `stride`-th sentence of the batch sorted by length, longest first: a
    length-stratified sample that always holds the longest sentence."""
    order = np.argsort(-lengths, kind="stable")
    return sorted(int(i) for i in order[::stride])


# maximum and edge lengths at the bge-large depth: the position-table limit 512, query-tile
# boundaries 128 / 129 / 257, and one- and two-token sentences
EDGE_LENGTHS = (512, 511, 257, 129, 128, 2, 1)
EDGE_SEED = 3


def edge_inputs(shape):
    lengths = np.array(EDGE_LENGTHS, np.int32)
    ids, _ = W.sample_ids(shape, lengths, seed=EDGE_SEED, pad_to=512)
    return lengths, ids


def gen_model(name: str, stride: int = 1) -> None:
    shape = W.SHAPES[name]
    weights = W.make_weights(shape)
    lengths = W.sample_lengths(shape)
    ids, _ = W.sample_ids(shape, lengths)
    idx = stride_pick(lengths, stride)
    t0 = time.time()
    emb = O.Model(shape, weights).forward_batch(ids[idx], lengths[idx], kind="ref",
                                                threads=os.cpu_count())
    print(f"{name}: {len(idx)} sentences (lengths {lengths[idx].tolist()}) in {time.time() - t0:.1f}s")
    np.savez_compressed(os.path.join(HERE, f"model_{name}.npz"), index=np.array(idx, np.int32),
                        lengths=lengths[idx], embeddings=emb, ids_sha256=np.array(sha(ids)),
                        weights_sha256=np.array(weights_hash(weights)))


def gen_edge(name: str) -> None:
    shape = W.SHAPES[name]
    weights = W.make_weights(shape)
    lengths, ids = edge_inputs(shape)
    t0 = time.time()
    emb = O.Model(shape, weights).forward_batch(ids, lengths, kind="ref", threads=os.cpu_count())
    print(f"{name} edge lengths {lengths.tolist()} in {time.time() - t0:.1f}s")
    np.savez_compressed(os.path.join(HERE, f"model_{name}-edge.npz"), lengths=lengths, embeddings=emb,
                        ids_sha256=np.array(sha(ids)), weights_sha256=np.array(weights_hash(weights)))


if __name__ == "__main__":
    if not O.available("ref"):
        sys.exit("oracle/_ref is not built (make -C oracle with the reference sources present)")
    what = sys.argv[1:] or ["ops", "bge-small", "bge-base", "bge-large", "bge-large-edge"]
    if "ops" in what:
        gen_ops()
    if "bge-small" in what:
        gen_model("bge-small")  # the whole batch of 8
    if "bge-base" in what:
        gen_model("bge-base")  # the whole batch of 64
    if "bge-large" in what:
        gen_model("bge-large", stride=8)  # 32 of 256, every 8th by length, the longest included
    if "bge-large-edge" in what:
        gen_edge("bge-large")
