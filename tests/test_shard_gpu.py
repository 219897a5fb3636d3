"""The sharded data path with the GPU engine in every rank: two torch.distributed.run
processes (one per GPU, or both on GPU 0 when only one is visible) each encode their
cost-balanced contiguous slice of a length-sorted 64-sentence bge-base-shaped batch, and
the gathered slices must equal one engine's encode of the whole batch bit for bit (each
sentence's embedding does not depend on the rest of its batch).  The gloo test
(tests/test_shard_gloo.py) covers the same path on the CPU with the oracle in place of
the engine."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_two_rank_engine_shards_equal_one_engine(cuda_dev, tmp_path, monkeypatch):
    from fastembed_b200 import ops, workload as W
    from tests import shard_gpu_worker as SW
    shared = torch.cuda.device_count() < 2
    env = dict(os.environ)
    if shared:
        env["FE_LINEAR_NORM_FUSE"] = "0"  # two processes on one GPU: no cross-CTA waits
        monkeypatch.setenv("FE_LINEAR_NORM_FUSE", "0")  # the same launch forms in the reference run
    out = str(tmp_path / "sharded.npy")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "shard_gpu_worker.py"), out]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    sharded = np.load(out)
    shape, lengths, ids = SW.batch()
    eng = ops.Engine(shape, 0)
    eng.load_weights(W.make_weights(shape, seed=0))
    whole = eng.encode_host(ids, lengths)
    eng.close()
    assert np.array_equal(sharded, whole)
    assert np.abs(np.linalg.norm(whole, axis=1) - 1).max() < 1e-5
