"""Request-sharded serving with host-side failure handling (CPU).

Workers here are the CPU oracle (test infrastructure, deterministic), so a
stream continued on another worker after a failure must give exactly the
outputs of an undisturbed run: the failover replays the stream's input
history, position by position. Failures are made on the host: a worker
call that raises, and a rank process that exits without a word (its
heartbeat stops). No GPU is involved."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from phonon_b200 import serving, synth

LAYERS = 2


class OracleWorker:
    """The serving worker protocol over the CPU oracle."""

    def __init__(self, model):
        self.model = model
        self.cache, self.length = {}, {}

    def pages(self):
        return sum(n // 16 + 1 for n in self.length.values())

    def open(self, sid, rows):
        c = self.model.new_stream(256)
        y = None
        for p, x in enumerate(rows):
            ok, y, _ = self.model.step(c, p, x)
            assert ok
        self.cache[sid], self.length[sid] = c, len(rows)
        return y

    def step(self, sids, x):
        out = []
        for i, sid in enumerate(sids):
            ok, y, _ = self.model.step(self.cache[sid], self.length[sid], x[i])
            assert ok
            self.length[sid] += 1
            out.append(y)
        return np.stack(out)

    def close(self, sid):
        self.model.free_stream(self.cache.pop(sid))
        self.length.pop(sid)


class FlakyWorker(OracleWorker):
    """Raises from its n-th step call on (a host-side fault)."""

    def __init__(self, model, fail_at_step=None, fail_open=False):
        super().__init__(model)
        self.fail_at_step, self.fail_open, self.calls = fail_at_step, fail_open, 0

    def open(self, sid, rows):
        if self.fail_open:
            raise RuntimeError("injected open failure")
        return super().open(sid, rows)

    def step(self, sids, x):
        self.calls += 1
        if self.fail_at_step is not None and self.calls >= self.fail_at_step:
            raise RuntimeError("injected step failure")
        return super().step(sids, x)


def _inputs(sid, position):
    return synth.Generator(1000 + 7919 * sid + position).normal(512).astype(np.float32)


def _run(server, prefixes, steps):
    outs = {}
    for sid, n in prefixes.items():
        server.open(sid, np.stack([_inputs(sid, p) for p in range(n)]))
    for k in range(steps):
        y = server.step({sid: _inputs(sid, n + k) for sid, n in prefixes.items()})
        for sid, n in prefixes.items():
            outs[(sid, n + k)] = y[sid]
    return outs


@pytest.fixture(scope="module")
def model(oracle):
    return oracle.model(synth.flow_weights(LAYERS, seed=0))


PREFIXES = {0: 5, 1: 19, 2: 3, 3: 11, 4: 8, 5: 16}


def test_failover_continues_bit_exact(model):
    ref = _run(serving.ShardedServer([OracleWorker(model)]), PREFIXES, 6)
    flaky = FlakyWorker(model, fail_at_step=3)
    server = serving.ShardedServer([OracleWorker(model), flaky, OracleWorker(model)])
    outs = _run(server, PREFIXES, 6)
    assert server.failed == [1] and server.live == [0, 2]
    moved = [sid for sid in PREFIXES if sid in flaky.cache]
    assert moved and server.migrations == len(moved)
    assert all(server.owner[sid] != 1 for sid in PREFIXES)
    for key, y in ref.items():
        assert np.array_equal(outs[key], y), key


def test_open_skips_failing_worker(model):
    server = serving.ShardedServer([FlakyWorker(model, fail_open=True), OracleWorker(model)])
    server.open(9, np.stack([_inputs(9, p) for p in range(4)]))
    assert server.owner[9] == 1 and server.failed == [0]


def test_least_pages_placement(model):
    server = serving.ShardedServer([OracleWorker(model), OracleWorker(model)])
    server.open(0, np.stack([_inputs(0, p) for p in range(40)]))  # 3 pages on worker 0
    server.open(1, np.stack([_inputs(1, p) for p in range(4)]))   # -> worker 1
    server.open(2, np.stack([_inputs(2, p) for p in range(4)]))   # worker 1 (1 page) < worker 0 (3)
    assert [server.owner[i] for i in (0, 1, 2)] == [0, 1, 1]


def test_no_worker_left(model):
    server = serving.ShardedServer([FlakyWorker(model, fail_at_step=1)])
    server.open(0, np.stack([_inputs(0, p) for p in range(3)]))
    with pytest.raises(serving.WorkerFailed):
        server.step({0: _inputs(0, 3)})


# ------------------------------------------------------ one process per rank
STEPS, DIE_AFTER, PACE = 14, 3, 0.25


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import sys
    import time
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "speech-mac_b200"))
    sys.path.insert(0, str(root))
    import torch.distributed as dist
    from oracle.oracle import Oracle
    from phonon_b200 import serving as sv
    from phonon_b200 import synth as sy
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, wait_for_workers=True)
    model = Oracle().model(sy.flow_weights(LAYERS, seed=0))
    hb = sv.Heartbeat(store, rank, world, timeout=1.0)
    shard = sv.RankShard(OracleWorker(model), rank, world, hb, _inputs)
    for sid, n in sorted(PREFIXES.items()):
        shard.open(sid, n)
    q.put(("owned", rank, sorted(s for s, r in shard.owner.items() if r == rank)))
    sent = set()
    for k in range(STEPS):
        shard.step(k)
        fresh = {key: y for key, y in shard.outputs.items() if key not in sent}
        sent |= set(fresh)
        q.put(("out", rank, fresh))
        if rank == world - 1 and k == DIE_AFTER:
            q.close()
            q.join_thread()  # the outputs it completed reach the parent
            os._exit(0)      # silent death: no resign, the heartbeat just stops
        time.sleep(PACE)
    q.put(("done", rank, sorted(shard.handled)))
    store.set(f"finished/{rank}", "1")
    if rank == 0:  # the store's server lives here; wait for the other survivor
        store.wait([f"finished/{r}" for r in range(world - 1)])


def test_rank_death_detected_and_streams_reprefilled(model):
    world = 3
    ref = _run(serving.ShardedServer([OracleWorker(model)]), PREFIXES, STEPS)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    outs, owned, handled = {}, {}, {}
    done = 0
    while done < world - 1:
        kind, rank, payload = q.get(timeout=60)
        if kind == "out":
            for key, y in payload.items():
                assert key not in outs, f"position {key} decoded twice"
                outs[key] = y
        elif kind == "owned":
            owned[rank] = payload
        else:
            handled[rank] = payload
            done += 1
    for p in procs:
        p.join(timeout=30)
    assert owned[world - 1], "the dying rank owned no stream"
    assert handled == {0: [world - 1], 1: [world - 1]}
    assert set(outs) == set(ref)  # every position of every stream, exactly once
    for key, y in ref.items():
        assert np.array_equal(outs[key], y), key
