"""Generates the golden embeddings of the Qwen3- and Gemma3-shaped test encoders.

    python tests/golden/gen_golden_rms.py

These families are not in the reference: the outputs come from oracle/hf_oracle.py
(transformers' Qwen3Model / Gemma3TextModel on the CPU in FP32).  Inputs are regenerated
from fastembed_b200.workload's seeds; a hash of the generated weights and ids is stored so
that a generator change is caught.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from fastembed_b200 import workload as W  # noqa: E402
from oracle import hf_oracle as H  # noqa: E402

SHAPES = ("qwen3-tiny", "gemma3-tiny")
WEIGHT_SEED, INPUT_SEED, NORM_JITTER = 0, 1, 0.1


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


def main() -> None:
    for name in SHAPES:
        shape, weights, lengths, ids = inputs(name)
        emb = H.embed(shape, weights, ids, lengths)
        np.savez_compressed(os.path.join(HERE, f"model_{name}.npz"), lengths=lengths, ids=ids, embeddings=emb,
                            digest=np.array(digest(weights, ids)))
        print(name, lengths.tolist(), emb.shape)


if __name__ == "__main__":
    main()
