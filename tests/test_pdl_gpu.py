"""Programmatic dependent launch (FE_PDL=1; off by default).  With it, the engine's
kernels are launched so that one may start (its CTAs resident, its set-up done) while
the previous kernel in the stream is still running; each waits for that kernel's
completion before it touches a buffer or allocates TMEM.  A kernel missing that wait
would race with its predecessor, so these tests run the same forward passes in child
processes with FE_PDL=0 (plain stream order) and FE_PDL=1 and require bit-identical
embeddings, twice per process.  The shapes are large enough to take the 2-CTA GEMM,
the fused projection + norm kernel and both attention kernels."""
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import dataclasses, sys
import numpy as np
from fastembed_b200 import ops, workload as W

out = {}
shape = dataclasses.replace(W.SHAPES["bge-large"], layers=2)
weights = W.make_weights(shape, seed=3)
lengths = W.sample_lengths(shape, batch=96, seed=4)
ids, _ = W.sample_ids(shape, lengths, seed=5, pad_to=512)
eng = ops.Engine(shape, 0)
eng.load_weights(weights)
out["bge_a"] = eng.encode_host(ids, lengths)
out["bge_b"] = eng.encode_host(ids, lengths)
eng.close()
for name in ("qwen3-0.6b", "gemma-300m"):
    shape = dataclasses.replace(W.RMS_SHAPES[name], layers=2, vocab=1000)
    weights = W.make_rms_weights(shape, seed=6)
    lengths = W.sample_rms_lengths(shape, batch=24, seed=7)
    ids = W.sample_rms_ids(shape, lengths, seed=8)
    eng = ops.Engine(shape, 0)
    eng.load_weights(weights)
    out[name + "_a"] = eng.encode_host(ids, lengths)
    out[name + "_b"] = eng.encode_host(ids, lengths)
    eng.close()
ops.device_status(0)
np.savez(sys.argv[1], **out)
"""


def _run(tmp_path, pdl):
    path = str(tmp_path / f"pdl{pdl}.npz")
    env = dict(os.environ, FE_PDL=str(pdl))
    r = subprocess.run([sys.executable, "-c", CHILD, path], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-4000:]
    return np.load(path)


@pytest.mark.gpu
def test_pdl_matches_stream_order(cuda_dev, tmp_path):
    plain = _run(tmp_path, 0)
    pdl = _run(tmp_path, 1)
    assert sorted(plain.files) == sorted(pdl.files)
    for k in plain.files:
        assert np.isfinite(plain[k]).all(), k
        assert np.array_equal(plain[k], pdl[k]), k
    for name in ("bge", "qwen3-0.6b", "gemma-300m"):
        assert np.array_equal(pdl[name + "_a"], pdl[name + "_b"]), name
