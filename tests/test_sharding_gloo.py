"""The multi-GPU path splits the batch into contiguous shards with replicated weights and no
collective. This runs that split on CPU with two gloo ranks: each rank evaluates its shard with the
oracle, the shards are gathered, and the result must equal the full-batch evaluation (the batch
independence the backend's separability check relies on), and bench.py's shard arithmetic must
cover the batch exactly once."""
import os
import socket

import numpy as np
import torch.distributed as dist
import torch.multiprocessing as mp


def shard_of(total, world, rank):
    per = total // world + (1 if rank < total % world else 0)
    begin = rank * (total // world) + min(rank, total % world)
    return begin, per


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    from oracle.interp import Interpreter
    from shorokoo_b200.emit import graphs
    case = graphs.resnet(depth=18, batch=5, hw=(32, 32), seed=4, affine_scale=0.1)
    x = case.inputs[-1][1]
    begin, per = shard_of(5, world, rank)
    it = Interpreter(case.model, "fp32", threads=1)
    y = it.run({case.inputs[-1][0]: x[begin:begin + per]})[0]
    sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(sizes, torch.tensor([y.shape[0]]))
    mx = max(int(s) for s in sizes)
    pad = np.zeros((mx, y.shape[1]), np.float32)
    pad[: y.shape[0]] = y
    bufs = [torch.zeros(mx, y.shape[1]) for _ in range(world)]
    dist.all_gather(bufs, torch.from_numpy(pad))
    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)         # max-over-ranks timing reduction
    if rank == 0:
        got = np.concatenate([b.numpy()[: int(s)] for b, s in zip(bufs, sizes)])
        full = it.run({case.inputs[-1][0]: x})[0]
        q.put((float(np.abs(got - full).max() / np.abs(full).max()), float(t)))
    dist.destroy_process_group()


def test_two_rank_shards_match_full_batch():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(2, port, q), nprocs=2, join=True, start_method="spawn")
    err, tmax = q.get()
    assert err < 1e-5 and tmax == 2.0


def test_shard_arithmetic_covers_batch():
    for total in (1, 5, 64, 512):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_of(total, world, r) for r in range(world)]
            covered = []
            for b, n in spans:
                covered += list(range(b, b + n))
            assert covered == list(range(total))
