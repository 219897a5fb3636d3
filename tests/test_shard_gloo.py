"""The multi-GPU data path on CPU: world_size-2 gloo ranks each take their
cost-balanced contiguous slice of a length-sorted batch (fe_plan_shards) and encode
it (here with the oracle standing in for the GPU engine); the gathered embeddings,
scattered back to the original order, must equal a single-process run bit for bit.
A rank that fails is seen by the others on the host, before any further work."""
import dataclasses
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _shape():
    from fastembed_b200 import workload as W
    return dataclasses.replace(W.SHAPES["bge-small"], layers=1, hidden=128, heads=2, intermediate=256,
                               vocab=400, batch=12, lengths=("uniform", 2, 40), pad_to=40)


def _batch():
    from fastembed_b200 import workload as W
    shape = _shape()
    lengths = W.sample_lengths(shape, seed=3)
    ids, _ = W.sample_ids(shape, lengths, seed=3)
    return shape, lengths, ids


def _worker(rank, world, port, result_path, fail_rank):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from fastembed_b200 import ops, workload as W
    from oracle import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    shape, lengths, ids = _batch()
    order = np.argsort(-lengths, kind="stable")
    cuts = ops.plan_shards(shape, lengths[order], world)
    bounds = [0] + cuts + [lengths.size]
    mine = order[bounds[rank]:bounds[rank + 1]]
    ok = torch.tensor([0 if rank == fail_rank else 1])
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)  # host-side health check before the step
    if int(ok) == 0:
        dist.destroy_process_group()
        return
    model = O.Model(shape, W.make_weights(shape, seed=2))
    emb = model.forward_batch(ids[mine], lengths[mine], threads=1)
    gathered = [None] * world
    dist.all_gather_object(gathered, (mine.tolist(), emb))
    if rank == 0:
        full = np.zeros((lengths.size, shape.hidden), np.float32)
        for idx, e in gathered:
            full[idx] = e
        np.save(result_path, full)
    dist.destroy_process_group()


def _run(world, tmp_path, fail_rank=-1):
    port = _free_port()
    out = str(tmp_path / "emb.npy")
    mp.start_processes(_worker, args=(world, port, out, fail_rank), nprocs=world, start_method="spawn", join=True)
    return out


def test_two_rank_shards_equal_single_process(tmp_path, oracle_lib):
    out = _run(2, tmp_path)
    from fastembed_b200 import workload as W
    shape, lengths, ids = _batch()
    ref = oracle_lib.Model(shape, W.make_weights(shape, seed=2)).forward_batch(ids, lengths, threads=1)
    assert np.array_equal(np.load(out), ref)


def test_failed_rank_is_detected_before_work(tmp_path, oracle_lib):
    out = _run(2, tmp_path, fail_rank=1)
    assert not os.path.exists(out)  # rank 0 stopped before encoding and wrote nothing
