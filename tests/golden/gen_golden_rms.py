"""Generates the golden embeddings of the Qwen3- and Gemma3-shaped encoders.

    python tests/golden/gen_golden_rms.py [qwen3-tiny gemma3-tiny qwen3-0.6b gemma-300m]

These families are not in the reference: the outputs come from oracle/hf_oracle.py
(transformers' Qwen3Model / Gemma3TextModel on the CPU in FP32).  Inputs are regenerated
from fastembed_b200.workload's seeds; a hash of the generated weights and ids is stored so
that a generator change is caught.

* qwen3-tiny / gemma3-tiny: two-layer shapes with jittered norm weights, whole batch.
* qwen3-0.6b / gemma-300m: the full benchmark shapes (28 x 1024 and 24 x 768) with the
  benchmark's weights and batch (128 and 512 sentences); the stored sentences are every
  16th / 32nd of the batch by length, the longest included, plus an edge set of lengths
  up to 1024 (model_<name>-edge.npz).
"""
from __future__ import annotations

import hashlib
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from fastembed_b200 import workload as W  # noqa: E402
from oracle import hf_oracle as H  # noqa: E402

SHAPES = ("qwen3-tiny", "gemma3-tiny")
FULL = {"qwen3-0.6b": 16, "gemma-300m": 32}  # shape -> stride of the stored sample
EDGE_LENGTHS = {"qwen3-0.6b": (1024, 1023, 513, 129, 128, 2, 1),
                "gemma-300m": (1024, 512, 257, 256, 129, 128, 2, 1)}
WEIGHT_SEED, INPUT_SEED, NORM_JITTER, EDGE_SEED = 0, 1, 0.1, 3


def full_inputs(name: str):
    """The benchmark's weights and batch of a full shape, and the stored sample's rows."""
    shape = W.RMS_SHAPES[name]
    weights = W.make_rms_weights(shape, seed=WEIGHT_SEED)
    lengths = W.sample_rms_lengths(shape, seed=INPUT_SEED)
    ids = W.sample_rms_ids(shape, lengths, seed=INPUT_SEED)
    order = np.argsort(-lengths, kind="stable")
    index = np.sort(order[::FULL[name]]).astype(np.int32)
    return shape, weights, lengths, ids, index


def edge_inputs(shape):
    lengths = np.array(EDGE_LENGTHS[shape.name], np.int32)
    return lengths, W.sample_rms_ids(shape, lengths, seed=EDGE_SEED)


def inputs(name: str):
    shape = W.RMS_SHAPES[name]
    weights = W.make_rms_weights(shape, seed=WEIGHT_SEED, norm_jitter=NORM_JITTER)
    lengths = W.sample_rms_lengths(shape, seed=INPUT_SEED)
    ids = W.sample_rms_ids(shape, lengths, seed=INPUT_SEED)
    return shape, weights, lengths, ids


def digest(weights: dict, ids: np.ndarray) -> str:
    h = hashlib.sha256()
    for k in sorted(weights):
        h.update(k.encode())
        h.update(np.ascontiguousarray(weights[k]).tobytes())
    h.update(ids.tobytes())
    return h.hexdigest()


def main(names) -> None:
    for name in names:
        if name in FULL:
            shape, weights, lengths, ids, index = full_inputs(name)
            t0 = time.time()
            emb = H.embed(shape, weights, ids[index], lengths[index])
            np.savez_compressed(os.path.join(HERE, f"model_{name}.npz"), index=index, lengths=lengths[index],
                                embeddings=emb, digest=np.array(digest(weights, ids)))
            print(name, lengths[index].tolist(), f"{time.time() - t0:.0f}s", flush=True)
            el, eids = edge_inputs(shape)
            t0 = time.time()
            emb = H.embed(shape, weights, eids, el)
            np.savez_compressed(os.path.join(HERE, f"model_{name}-edge.npz"), lengths=el, embeddings=emb,
                                digest=np.array(digest(weights, eids)))
            print(name, "edge", el.tolist(), f"{time.time() - t0:.0f}s", flush=True)
            continue
        shape, weights, lengths, ids = inputs(name)
        emb = H.embed(shape, weights, ids, lengths)
        np.savez_compressed(os.path.join(HERE, f"model_{name}.npz"), lengths=lengths, ids=ids, embeddings=emb,
                            digest=np.array(digest(weights, ids)))
        print(name, lengths.tolist(), emb.shape)


if __name__ == "__main__":
    main(sys.argv[1:] or list(SHAPES) + list(FULL))
