"""Request sharding across ranks (multi-GPU path) on CPU with gloo.

Every rank runs the same seeded serving simulation and keeps the streams
assigned to it; there is no exchange on the data path. Two gloo ranks check
that the shards partition the active streams at every step, that the page
balance holds, and that the time reduction bench.py uses (max over ranks)
works."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _load_bench():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _rank(rank, world, port, out):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    bench = _load_bench()
    sim = bench.ServingSim(world, streams=64)
    owned_per_step = []
    for _ in range(40):
        sim.churn()
        owned_per_step.append(sorted(sid for sid, (r, _) in sim.active.items() if r == rank))
        sim.advance()
    gathered = [None] * world
    dist.all_gather_object(gathered, owned_per_step)
    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        out.put((gathered, float(t.item()), sorted(sim.active), list(sim.pages)))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_sharding_partitions_streams():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    gathered, tmax, active, pages = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert tmax == 2.0
    for step in range(40):
        a, b = set(gathered[0][step]), set(gathered[1][step])
        assert not (a & b)  # no stream on two GPUs
    assert set(gathered[0][-1]) | set(gathered[1][-1]) == set(active)
    assert max(pages) - min(pages) < 0.25 * max(pages)  # least-loaded assignment keeps KV balanced


def test_single_rank_sim_deterministic():
    bench = _load_bench()
    a, b = bench.ServingSim(1), bench.ServingSim(1)
    for _ in range(20):
        assert a.churn() == b.churn()
        a.advance()
        b.advance()
    assert a.active == b.active and len(a.active) > 400
