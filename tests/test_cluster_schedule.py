"""The ring protocol of the single-stream cluster step, checked on the CPU.

step_cluster_kernel (speech-mac_b200/csrc/phonon_cluster.cuh) has one copy
warp that fills three rings of shared-memory slots (weight units, LayerNorm
vectors, K/V pages) and eight compute warps that consume them; full and
empty mbarriers pair them up, and all warps of the CTA meet at five cluster
barriers per layer. A wrong refill schedule would not give wrong numbers, it
would hang (bounded by the kernel's 2 s wait budget) or silently reuse a slot.
This model replays, in the kernel's order, every wait, arrival, copy issue
and barrier of one CTA (the copy warp's per-phase refills, phonon_cluster.cuh
copy-warp loop; the compute warps' waits and releases per phase), under
random interleavings, and checks that

- every wait is eventually satisfied (no deadlock at any barrier),
- no waiter ever lags two phases behind an mbarrier (the parity would alias),
- no slot is refilled before every consumer of its previous unit released it.

Mbarriers are modelled by their completed-phase count; a copy completes its
full barrier when issued (the latency does not change the protocol)."""
import random

import pytest

UNITS_PER_LAYER = 12  # q, k, v, out, 4 x up, 4 x down
KV_SLOTS = 8
WARPS = 8


class Bar:
    def __init__(self, count):
        self.count, self.pending, self.phase = count, count, 0

    def arrive(self):
        self.pending -= 1
        assert self.pending >= 0
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count


def run(L, npc, w_slots, holds_last, seed, wait_release=True):
    rnd = random.Random(seed)
    n_units = UNITS_PER_LAYER * L
    wfull = [Bar(1) for _ in range(w_slots)]
    wempty = [Bar(WARPS) for _ in range(w_slots)]
    nfull, nempty = [Bar(1), Bar(1)], [Bar(1), Bar(1)]
    kfull = [Bar(1) for _ in range(KV_SLOTS)]
    kempty = [Bar(1) for _ in range(KV_SLOTS)]
    loaded = {}  # (ring, slot) -> index held and not yet released
    releases = {}

    def issue(ring, idx, nslots, full):
        key = (ring, idx % nslots)
        assert key not in loaded, f"{ring} slot {idx % nslots} refilled with {idx} before {loaded[key]} was released"
        loaded[key] = idx
        full[idx % nslots].arrive()

    def release(ring, idx, nslots, empty, consumers):
        releases[(ring, idx)] = releases.get((ring, idx), 0) + 1
        if releases[(ring, idx)] == consumers:
            assert loaded.pop((ring, idx % nslots)) == idx
        empty[idx % nslots].arrive()

    state = {"kv_next": 0, "kv_last_ok": -1}

    def refill_after(u):  # copy warp: unit u consumed -> unit u + w_slots into its slot
        if u + w_slots >= n_units:
            return
        if wait_release:
            yield ("wait", wempty[u % w_slots], u // w_slots)
        issue("w", u + w_slots, w_slots, wfull)

    def renorm_after(n):
        if n + 2 >= 2 * L:
            return
        yield ("wait", nempty[n & 1], n >> 1)
        issue("n", n + 2, 2, nfull)

    def issue_kv(limit):
        while state["kv_next"] < limit:
            n = state["kv_next"]
            layer, i = divmod(n, npc)
            if holds_last and i == npc - 1 and layer > state["kv_last_ok"]:
                break  # the appended page waits for its layer's phase A
            if n >= KV_SLOTS:
                yield ("wait", kempty[n % KV_SLOTS], n // KV_SLOTS - 1)
            issue("k", n, KV_SLOTS, kfull)
            state["kv_next"] += 1

    def copy_warp():
        for u in range(min(w_slots, n_units)):
            issue("w", u, w_slots, wfull)
        for n in range(min(2, 2 * L)):
            issue("n", n, 2, nfull)
        yield from issue_kv(min(npc, KV_SLOTS))
        for l in range(L):
            u0 = UNITS_PER_LAYER * l
            for k in range(3):  # A
                yield from refill_after(u0 + k)
            yield from renorm_after(2 * l)
            yield ("cluster",)
            state["kv_last_ok"] = l  # B
            yield from issue_kv(min((l + 1) * npc + KV_SLOTS, (l + 2) * npc, L * npc))
            yield ("cluster",)
            yield from refill_after(u0 + 3)  # C
            yield ("cluster",)
            for k in range(4, 8):  # D
                yield from refill_after(u0 + k)
            yield from renorm_after(2 * l + 1)
            yield ("cluster",)
            for k in range(8, 12):  # E
                yield from refill_after(u0 + k)
            yield ("cluster",)

    def use_unit(u):
        yield ("wait", wfull[u % w_slots], u // w_slots)
        release("w", u, w_slots, wempty, WARPS)

    def compute_warp(w):
        for l in range(L):
            u0 = UNITS_PER_LAYER * l
            if w == 0:  # LN1
                yield ("wait", nfull[(2 * l) & 1], l)
                release("n", 2 * l, 2, nempty, 1)
            yield ("csync",)
            for k in range(3):
                yield from use_unit(u0 + k)
            yield ("cluster",)
            for i in range(w, npc, KV_SLOTS):  # B: pages w, w + 8, ...
                n = l * npc + i
                yield ("wait", kfull[n % KV_SLOTS], n // KV_SLOTS)
                release("k", n, KV_SLOTS, kempty, 1)
            yield ("csync",)
            yield ("cluster",)
            yield ("csync",)  # C
            yield from use_unit(u0 + 3)
            yield ("cluster",)
            if w == 0:  # LN2
                yield ("wait", nfull[(2 * l + 1) & 1], l)
                release("n", 2 * l + 1, 2, nempty, 1)
            yield ("csync",)
            for k in range(4, 8):
                yield from use_unit(u0 + k)
            yield ("cluster",)
            for k in range(8, 12):  # E: every warp waits for and releases all four down units
                yield from use_unit(u0 + k)
            yield ("cluster",)

    actors = {"copy": copy_warp(), **{f"w{w}": compute_warp(w) for w in range(WARPS)}}
    blocked = {a: None for a in actors}
    done = set()
    while len(done) < len(actors):
        runnable = []
        for a in actors:
            if a in done:
                continue
            b = blocked[a]
            if b is None:
                runnable.append(a)
            elif b[0] == "wait":
                bar, phase = b[1], b[2]
                assert bar.phase <= phase + 1, f"{a} lags two phases behind an mbarrier"
                if bar.phase > phase:
                    runnable.append(a)
        if not runnable:
            live = [a for a in actors if a not in done]
            at_cluster = [a for a in live if blocked[a] and blocked[a][0] == "cluster"]
            at_csync = [a for a in live if blocked[a] and blocked[a][0] == "csync"]
            compute = [a for a in live if a != "copy"]
            if at_cluster and len(at_cluster) == len(live):
                for a in at_cluster:
                    blocked[a] = None
                continue
            if at_csync and sorted(at_csync) == sorted(compute):
                for a in at_csync:
                    blocked[a] = None
                continue
            raise AssertionError(f"deadlock: {blocked}")
        a = rnd.choice(runnable)
        try:
            blocked[a] = next(actors[a])
        except StopIteration:
            done.add(a)
            blocked[a] = None


@pytest.mark.parametrize("w_slots", [7, 9])  # fp32 and bf16 K/V
@pytest.mark.parametrize("L", [1, 2, 12])
@pytest.mark.parametrize("npc", [0, 1, 5, 8, 9, 17, 64])
def test_cluster_rings_never_deadlock_or_alias(L, npc, w_slots):
    for holds_last in ((False, True) if npc else (False,)):
        for seed in range(3):
            run(L, npc, w_slots, holds_last, seed)


def test_model_catches_a_refill_before_release():
    """The checker itself: a copy warp that refills a weight slot without
    waiting for its consumers' release is rejected."""
    with pytest.raises(AssertionError):
        for seed in range(10):
            run(2, 4, 7, False, seed, wait_release=False)
