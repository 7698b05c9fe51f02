"""Multi-rank host logic on CPU (gloo, world_size 2): rank-wise row sharding with per-chunk
seeded data must reassemble exactly to the single-process result, and the max-over-ranks timing
reduction bench.py uses must pick the slowest rank."""
import os
import queue
import socket
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
import __graft_entry__  # noqa: E402  (spawned workers do not run conftest)

__graft_entry__.load_package()

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gpu_pipes_b200 import workloads as W
from oracle import mlp_oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = W.MGN_NODE.with_m(m)
        r0, n = W.shard_rows(m, world, rank)
        x = W.make_input(w, r0, n)
        layers, ln = W.make_weights(w)
        y = O.workload_forward(w, x, layers, ln)
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([n]))
        maxn = int(max(s.item() for s in sizes))
        pad = torch.zeros(maxn, w.n_out)
        pad[:n] = y
        parts = [torch.zeros(maxn, w.n_out) for _ in range(world)]
        dist.all_gather(parts, pad)
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            full = torch.cat([p[:int(s.item())] for p, s in zip(parts, sizes)])
            # a numpy array is pickled by value; a torch tensor would be shared through a file
            # descriptor owned by this process, which exits before the parent unpickles it
            q.put((full.numpy(), float(t.item())))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_reassembles():
    m, world = 70000, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, m, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = None
    for _ in range(120):
        try:
            got = q.get(timeout=1)
            break
        except queue.Empty:
            assert all(p.is_alive() or p.exitcode == 0 for p in procs), "a worker died"
    assert got is not None, "no result from rank 0"
    full, tmax = got
    full = torch.from_numpy(full)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    w = W.MGN_NODE.with_m(m)
    x = W.make_input(w)
    layers, ln = W.make_weights(w)
    ref = O.workload_forward(w, x, layers, ln)
    assert torch.equal(full, ref)
    assert tmax == 2.0
