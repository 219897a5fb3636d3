"""One rank of the sharded GPU encode checked by tests/test_shard_gpu.py (launched by
torch.distributed.run, not collected by pytest).

Every rank builds the same bge-base-shaped batch, sorts it by length, takes its
cost-balanced contiguous slice (fe_plan_shards), encodes the slice with its own engine on
GPU rank % device_count, and the slices are gathered over gloo to rank 0, which writes
the embeddings in the sorted order to the output file.  With fewer GPUs than ranks, the
ranks that share a GPU run every projection + norm step as two launches
(FE_LINEAR_NORM_FUSE=0, set by the test), so no kernel waits on another CTA's progress.

    python -m torch.distributed.run --nproc-per-node 2 ... tests/shard_gpu_worker.py OUT.npy
"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def batch():
    from fastembed_b200 import workload as W
    shape = W.SHAPES["bge-base"]
    lengths = W.sample_lengths(shape, seed=5)
    ids, _ = W.sample_ids(shape, lengths, seed=5)
    order = np.argsort(-lengths, kind="stable")
    return shape, np.ascontiguousarray(lengths[order]), np.ascontiguousarray(ids[order])


def main(out_path: str) -> int:
    from fastembed_b200 import ops, workload as W
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    device = rank % torch.cuda.device_count()
    torch.cuda.set_device(device)
    shape, lengths, ids = batch()
    cuts = ops.plan_shards(shape, lengths, world) if world > 1 else []
    bounds = [0] + list(cuts) + [lengths.size]
    lo, hi = bounds[rank], bounds[rank + 1]
    eng = ops.Engine(shape, device)
    eng.load_weights(W.make_weights(shape, seed=0))
    emb = eng.encode_host(np.ascontiguousarray(ids[lo:hi]), np.ascontiguousarray(lengths[lo:hi]))
    eng.close()
    ops.device_status(device)
    parts = [None] * world
    dist.all_gather_object(parts, (lo, hi, emb))
    if rank == 0:
        out = np.zeros((lengths.size, shape.hidden), np.float32)
        for a, b, e in parts:
            out[a:b] = e
        np.save(out_path, out)
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1]))
