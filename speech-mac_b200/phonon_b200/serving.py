"""Request-sharded decode serving across GPUs, with worker failures handled on the host.

Concurrent utterances are independent, so each stream lives on exactly one
worker (one GPU, one libphonon_cuda context): a new stream goes to the live
worker holding the fewest KV pages, and a step runs each worker's streams
as one batched step on that worker. Nothing crosses between GPUs.

Every stream keeps its input history on the host: the prefix rows and the
input of every decoded position. When a worker fails, its streams are
re-prefilled from that history on the surviving workers, and the step goes
on. A worker fails when one of its calls raises; in multi-process serving a
rank also fails when its heartbeat stops. The replay feeds the same inputs
to the same positions, so the continuation is the computation the failed
worker would have done. This is the scale-out rule of speech-mac's engine:
requests share the read-only weights and nothing else
(src/speech.h:40-41).

Two forms:
  ShardedServer   one process drives all workers (a host thread per call is
                  optional; the calls are independent).
  RankShard       one process per GPU (torch.distributed launch). Every rank
                  replays the same deterministic arrival schedule, owns its
                  share of the streams, and learns of dead ranks through
                  Heartbeat over the process group's store. No collective is
                  on the data path.
"""
import time

import numpy as np

WIDTH = 512


class WorkerFailed(RuntimeError):
    """A worker call failed; the server has moved its streams elsewhere."""


class CudaWorker:
    """One libphonon_cuda context on one GPU as a serving worker."""

    def __init__(self, context, capacity):
        self.ctx = context
        self.capacity = capacity
        self.slot = {}    # stream id -> context stream
        self.length = {}  # stream id -> positions in the cache

    def pages(self):
        return sum(len(self.ctx.pages(s)) for s in self.slot.values())

    def open(self, sid, rows):
        s = self.ctx.stream_alloc(self.capacity)
        try:
            last = self.ctx.append(s, np.asarray(rows, np.float32))
        except Exception:
            self.ctx.stream_free(s)
            raise
        self.slot[sid] = s
        self.length[sid] = len(rows)
        return last

    def step(self, sids, x):
        streams = [self.slot[i] for i in sids]
        pos = [self.length[i] for i in sids]
        y = self.ctx.step(streams, pos, np.asarray(x, np.float32))
        for i in sids:
            self.length[i] += 1
        return y

    def close(self, sid):
        self.ctx.stream_free(self.slot.pop(sid))
        self.length.pop(sid, None)


class ShardedServer:
    """Streams sharded over workers by KV pages; failed workers' streams are
    re-prefilled on the survivors from the host-side input history.

    open(sid, prefix) -> last prefix output; step({sid: x}) -> {sid: y};
    close(sid). `failed` lists the workers taken out of service."""

    def __init__(self, workers):
        self.workers = list(workers)
        self.live = list(range(len(self.workers)))
        self.failed = []
        self.owner = {}    # sid -> worker index
        self.history = {}  # sid -> list of input rows (prefix + decoded inputs)
        self.migrations = 0

    def _least_loaded(self, exclude=()):
        cands = [w for w in self.live if w not in exclude]
        if not cands:
            raise WorkerFailed("no live worker left")
        return min(cands, key=lambda w: (self.workers[w].pages(), w))

    def _fail(self, w):
        """Take worker w out of service and re-home its streams."""
        if w not in self.live:
            return
        self.live.remove(w)
        self.failed.append(w)
        for sid in sorted(s for s, o in self.owner.items() if o == w):
            self._place(sid)

    def _place(self, sid):
        """(Re)build stream sid from its history on the least-loaded live worker."""
        while True:
            w = self._least_loaded()
            try:
                self.workers[w].open(sid, np.stack(self.history[sid]))
            except Exception:
                self._fail(w)
                continue
            if sid in self.owner:
                self.migrations += 1
            self.owner[sid] = w
            return

    def open(self, sid, prefix):
        if sid in self.owner:
            raise ValueError(f"stream {sid} is already open")
        self.history[sid] = [np.asarray(r, np.float32) for r in prefix]
        while True:
            w = self._least_loaded()
            try:
                last = self.workers[w].open(sid, np.asarray(prefix, np.float32))
            except Exception:
                self._fail(w)
                continue
            self.owner[sid] = w
            return last

    def step(self, inputs):
        """Decode one position of every stream in `inputs` ({sid: x}); each
        worker runs its streams as one batch. A worker that fails is taken
        out and its streams (of this step too) continue on the survivors."""
        out = {}
        pending = dict(inputs)
        while pending:
            groups = {}
            for sid in sorted(pending):
                groups.setdefault(self.owner[sid], []).append(sid)
            for w, sids in groups.items():
                if w not in self.live:
                    continue  # re-homed during this step; the next pass runs them
                x = np.stack([pending[i] for i in sids])
                try:
                    y = self.workers[w].step(sids, x)
                except Exception:
                    self._fail(w)
                    continue
                for i, sid in enumerate(sids):
                    out[sid] = y[i]
                    self.history[sid].append(np.asarray(pending.pop(sid), np.float32))
        return out

    def close(self, sid):
        w = self.owner.pop(sid)
        self.history.pop(sid)
        if w in self.live:
            self.workers[w].close(sid)


class Heartbeat:
    """Liveness of the ranks of a torch.distributed job over a store
    (torch.distributed.TCPStore or the process group's).

    beat(step) records that this rank completed `step`; a rank that fails on
    its own raises the alarm with resign(). dead() returns the ranks that
    resigned or whose heartbeat has not advanced for `timeout` seconds of
    this rank's clock, with the last step each completed. The first rank to
    see a silent death records it in the store (compare-and-set), so every
    survivor acts on the same last step; a rank that finds itself recorded
    dead must stop (declared_dead())."""

    def __init__(self, store, rank, world, timeout=2.0):
        self.store, self.rank, self.world, self.timeout = store, rank, world, timeout
        self.seen = {}  # rank -> (last step, local time it was first seen)
        self.beat(-1)

    def beat(self, step):
        self.store.set(f"hb/{self.rank}", str(step))

    def resign(self, step):
        self.store.set(f"dead/{self.rank}", str(step))

    def _get(self, key):
        if self.store.check([key]):
            return int(self.store.get(key))
        return None

    def dead(self):
        now = time.monotonic()
        out = {}
        for r in range(self.world):
            if r == self.rank:
                continue
            resigned = self._get(f"dead/{r}")
            step = self._get(f"hb/{r}")
            if resigned is not None:
                out[r] = resigned
                continue
            last = self.seen.get(r)
            if last is None or last[0] != step:
                self.seen[r] = (step, now)
            elif now - last[1] > self.timeout:
                mine = str(-1 if step is None else step).encode()
                agreed = self.store.compare_set(f"dead/{r}", b"", mine)
                out[r] = int(agreed)
        return out

    def declared_dead(self):
        return self.store.check([f"dead/{self.rank}"])


def assign(load, live):
    """The live rank with the least load (ties: lowest rank)."""
    return min(live, key=lambda r: (load[r], r))


class RankShard:
    """This rank's share of a multi-process serving run.

    Every rank replays the same deterministic schedule: streams open with
    their prefixes, each placed on the live rank with the fewest KV pages,
    and decode step k decodes position prefix + k of every stream. A rank
    computes only its own streams. When Heartbeat reports a dead rank, every
    survivor computes the same re-placement of the dead rank's streams (in
    stream order, each to the survivor owning the fewest streams); a new
    owner re-prefills each stream from its input history through the last
    step the dead rank completed, decodes the steps the stream missed, and
    the stream goes on with the rest. `inputs(sid, position)` returns the
    input row of a position (prefix rows and decoded inputs alike), as a
    front end replaying its request log would."""

    def __init__(self, worker, rank, world, heartbeat, inputs):
        self.worker, self.rank, self.world, self.hb = worker, rank, world, heartbeat
        self.inputs = inputs
        self.live = list(range(world))
        self.pages = [0] * world
        self.owner = {}     # sid -> rank
        self.prefix = {}    # sid -> prefix length
        self.next = {}      # sid -> next position to decode (own streams)
        self.outputs = {}   # (sid, position) -> output row of the streams this rank decoded
        self.handled = set()

    def open(self, sid, prefix_len):
        r = assign(self.pages, self.live)
        self.owner[sid] = r
        self.prefix[sid] = prefix_len
        self.pages[r] += prefix_len // 16 + 1
        if r == self.rank:
            self.worker.open(sid, np.stack([self.inputs(sid, p) for p in range(prefix_len)]))
            self.next[sid] = prefix_len

    def _take_over(self, dead, last_step):
        """Re-place the streams of `dead`, which completed decode steps
        0..last_step (-1: none)."""
        self.live.remove(dead)
        count = {r: sum(1 for o in self.owner.values() if o == r) for r in self.live}
        for sid in sorted(s for s, r in self.owner.items() if r == dead):
            r = assign(count, self.live)
            count[r] += 1
            self.owner[sid] = r
            if r == self.rank:
                n = self.prefix[sid] + last_step + 1
                self.worker.open(sid, np.stack([self.inputs(sid, p) for p in range(n)]))
                self.next[sid] = n

    def _decode(self, sids):
        x = np.stack([self.inputs(s, self.next[s]) for s in sids])
        y = self.worker.step(sids, x)
        for i, s in enumerate(sids):
            self.outputs[(s, self.next[s])] = y[i]
            self.next[s] += 1

    def step(self, k):
        """Decode step k of this rank's streams (after taking over the streams
        of ranks found dead); returns the number of positions decoded."""
        if self.hb.declared_dead():
            raise RuntimeError(f"rank {self.rank} was declared dead by its peers")
        for r, last in sorted(self.hb.dead().items()):
            if r not in self.handled and r in self.live:
                self.handled.add(r)
                self._take_over(r, last)
        mine = sorted(s for s, r in self.owner.items() if r == self.rank)
        decoded = 0
        for s in mine:  # streams inherited behind the schedule catch up one position at a time
            while self.next[s] < self.prefix[s] + k:
                self._decode([s])
                decoded += 1
        if mine:
            self._decode(mine)
            decoded += len(mine)
        self.hb.beat(k)
        return decoded
