"""The ring protocol of the single-stream cluster step, checked on the CPU.

step_cluster_kernel (speech-mac_b200/csrc/phonon_cluster.cuh) has one copy
warp that fills three rings of shared-memory slots (weight units, LayerNorm
vectors, K/V pages) and eight compute warps that consume them; full and
empty mbarriers pair them up. The copy warp issues every unit, norm and page
in the order the compute warps consume them, each after a bounded wait for
the release of its slot's previous contents; the compute warps meet at
named barriers between stages and at the exchanges with the other CTAs.
The first eight K/V pages of layer l + 1 are issued right after layer l's
out unit (their slots free once layer l's attention has read them). A
wrong protocol would not give wrong numbers, it would hang (bounded by the
kernel's 2 s wait budget) or silently reuse a slot. This model replays, in
the kernel's order, every wait, arrival and copy issue of one CTA (the copy
warp's issue sequence; the compute warps' waits and releases per stage: QKV
and up units in pairs, one out unit, down units read by two warps that each
count for four arrivals), under random interleavings, and checks that

- every wait is eventually satisfied (no deadlock),
- no waiter ever lags two phases behind an mbarrier (the parity would alias),
- no slot is refilled before every consumer of its previous unit released it.

Mbarriers are modelled by their completed-phase count; a copy completes its
full barrier when issued (the latency does not change the protocol); an
exchange with the other CTAs is a meeting point of the compute warps.

In the tensor-core form (tc) every warp runs the LayerNorms (fused with the
digit slicing) and every projection is an MMA issued by warps
0-3: for the four-unit projections (q/k/v, up, down) warp k waits for unit
k, issues its MMAs and commits them to an accumulator barrier (four arrivals
a phase); units 0-2 are released by a commit after their MMAs (modelled as
all eight arrivals at issue); for out, all four warps wait for the one unit.
The last unit (the row scales' holder) is released by all eight warps, warps
0-3 after they waited for the accumulator."""
import random

import pytest

UNITS_PER_LAYER = 13  # q0, q1, k, v, out, 4 x up, 4 x down
UNIT_OUT, UNIT_UP, UNIT_DOWN = 4, 5, 9
KV_SLOTS = 8
WARPS = 8


class Bar:
    def __init__(self, count):
        self.count, self.pending, self.phase = count, count, 0

    def arrive(self, n=1):
        self.pending -= n
        assert self.pending >= 0
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count


def run(L, npc, w_slots, seed, wait_release=True, tc=False):
    rnd = random.Random(seed)
    wfull = [Bar(1) for _ in range(w_slots)]
    wempty = [Bar(WARPS) for _ in range(w_slots)]
    nfull, nempty = Bar(1), Bar(WARPS if tc else 1)  # one LayerNorm slot; tc: every warp reads it
    accum = Bar(4)
    kfull = [Bar(1) for _ in range(KV_SLOTS)]
    kempty = [Bar(1) for _ in range(KV_SLOTS)]
    loaded = {}  # (ring, slot) -> index held and not yet released
    releases = {}

    def issue(ring, idx, nslots, full):
        key = (ring, idx % nslots)
        assert key not in loaded, f"{ring} slot {idx % nslots} refilled with {idx} before {loaded[key]} was released"
        loaded[key] = idx
        full[idx % nslots].arrive()

    def release(ring, idx, nslots, empty, consumers, weight=1):
        releases[(ring, idx)] = releases.get((ring, idx), 0) + weight
        if releases[(ring, idx)] == consumers:
            assert loaded.pop((ring, idx % nslots)) == idx
        empty[idx % nslots].arrive(weight)

    def copy_warp():
        state = {"u": 0, "k": 0}

        def unit():
            u = state["u"]
            state["u"] += 1
            if u >= w_slots and wait_release:
                yield ("wait", wempty[u % w_slots], u // w_slots - 1)
            issue("w", u, w_slots, wfull)

        def norm(n):
            if n >= 1:
                yield ("wait", nempty, n - 1)
            issue("n", n, 1, [nfull])

        def page():
            n = state["k"]
            state["k"] += 1
            if n >= KV_SLOTS:
                yield ("wait", kempty[n % KV_SLOTS], n // KV_SLOTS - 1)
            issue("k", n, KV_SLOTS, kfull)

        early = min(npc, KV_SLOTS)  # pages of the next layer issued after this layer's out unit
        for l in range(L):  # the compute warps' consumption order
            yield from norm(2 * l)
            for _k in range(UNIT_OUT):
                yield from unit()
            for _i in range(0 if l == 0 else early, npc):
                yield from page()
            yield from unit()  # out
            if l + 1 < L:
                for _i in range(early):
                    yield from page()
            yield from norm(2 * l + 1)
            for _k in range(UNIT_UP, UNITS_PER_LAYER):
                yield from unit()

    def wait_unit(u):
        yield ("wait", wfull[u % w_slots], u // w_slots)

    def projection(w, l, first, use, n=4):
        if tc:
            yield ("meet",)  # the digit rows sliced by all warps
            if w < 4:  # warp w's MMAs, their commit
                u = first + (w if n == 4 else 0)
                yield from wait_unit(u)
                if n == 4 and w < 3:
                    release("w", u, w_slots, wempty, WARPS, weight=WARPS)
                accum.arrive()
                yield ("wait", accum, use)
            release("w", first + n - 1, w_slots, wempty, WARPS)
        else:
            yield ("meet",)
            for k0 in (0, 2):  # units in pairs
                yield from wait_unit(first + k0)
                yield from wait_unit(first + k0 + 1)
                release("w", first + k0, w_slots, wempty, WARPS)
                release("w", first + k0 + 1, w_slots, wempty, WARPS)

    def compute_warp(w):
        for l in range(L):
            u0 = UNITS_PER_LAYER * l
            yield ("meet",)  # exchange of x (layer l > 0)
            if w == 1 or tc:  # LN1 (tc: every warp, fused with the digit slicing)
                yield ("wait", nfull, 2 * l)
                release("n", 2 * l, 1, [nempty], WARPS if tc else 1)
            yield from projection(w, l, u0, 4 * l)  # q/k/v
            yield ("meet",)
            for i in range(w, npc, WARPS):  # B: pages w, w + 8, ...
                n = l * npc + i
                yield ("wait", kfull[n % KV_SLOTS], n // KV_SLOTS)
                release("k", n, KV_SLOTS, kempty, 1)
            yield ("meet",)  # warp partials merged, message sent
            yield ("meet",)  # exchange of the messages, merge of the heads
            if tc:
                yield from projection(w, l, u0 + UNIT_OUT, 4 * l + 1, n=1)
            else:
                yield from wait_unit(u0 + UNIT_OUT)
                release("w", u0 + UNIT_OUT, w_slots, wempty, WARPS)
            yield ("meet",)  # exchange of h
            if w == 1 or tc:  # LN2
                yield ("wait", nfull, 2 * l + 1)
                release("n", 2 * l + 1, 1, [nempty], WARPS if tc else 1)
            yield from projection(w, l, u0 + UNIT_UP, 4 * l + 2)  # up
            yield ("meet",)  # exchange of g
            if tc:
                yield from projection(w, l, u0 + UNIT_DOWN, 4 * l + 3)
            else:
                u = u0 + UNIT_DOWN + (w >> 1)  # E: a down unit is read by two warps, four arrivals each
                yield from wait_unit(u)
                release("w", u, w_slots, wempty, WARPS, weight=WARPS // 2)

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
            compute = [a for a in actors if a != "copy" and a not in done]
            meeting = [a for a in compute if blocked[a] and blocked[a][0] == "meet"]
            if meeting and sorted(meeting) == sorted(compute):
                for a in meeting:
                    blocked[a] = None
                continue
            raise AssertionError(f"deadlock: {blocked}")
        a = rnd.choice(runnable)
        try:
            blocked[a] = next(actors[a])
        except StopIteration:
            done.add(a)
            blocked[a] = None


@pytest.mark.parametrize("tc", [False, True])  # CUDA-core rows, tensor-core q/k/v and up
@pytest.mark.parametrize("w_slots", [7, 8, 9])  # fp32 K/V, bf16 K/V (tensor-core form: 8)
@pytest.mark.parametrize("L", [1, 2, 12])
@pytest.mark.parametrize("npc", [0, 1, 5, 8, 9, 17, 64])
def test_cluster_rings_never_deadlock_or_alias(L, npc, w_slots, tc):
    for seed in range(3):
        run(L, npc, w_slots, seed, tc=tc)


def test_model_catches_a_refill_before_release():
    """The checker itself: a copy warp that refills a weight slot without
    waiting for its consumers' release is rejected."""
    for tc in (False, True):
        with pytest.raises(AssertionError):
            for seed in range(10):
                run(2, 4, 7, seed, wait_release=False, tc=tc)
