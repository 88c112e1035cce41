"""The mbarrier protocols of the tensor-core kernels, simulated on the host.

A kernel role waits for completion k of a barrier with a parity test
(``mbarrier.try_wait.parity`` with parity k & 1).  That test is only right
while the barrier has completed exactly k or k + 1 phases: at k - 1 it would
pass too early, at k + 2 it would read "not yet" forever.  Several waits in
the kernels rely on the order of the other roles to keep that window (a
split warp reusing an X_lo buffer checks ``empty`` of an older stage, the
attention producers check the scores' / P V commits of an older tile), so
this test plays every role of each protocol in random interleavings --
``tcgen05.commit`` arrivals land asynchronously, in issue order -- and checks
at every wait that the barrier is inside that window, and that the run ends
(no deadlock).  The protocols follow ``flux_b200/csrc/tc_gemm.cu``
(``tc_gemm_persistent_kernel``, ``tc_gemm_pair_kernel``) and
``flux_b200/csrc/tc_attention.cu``."""

from __future__ import annotations

import random
from collections import deque

import pytest


class Barrier:
    def __init__(self, name: str, count: int):
        self.name, self.count, self.pending, self.completed = name, count, count, 0

    def arrive(self):
        self.pending -= 1
        assert self.pending >= 0, f"{self.name}: more arrivals than the phase expects"
        if self.pending == 0:
            self.completed += 1
            self.pending = self.count


class Wait:
    def __init__(self, bar: Barrier, k: int):
        self.bar, self.k = bar, k


class Sim:
    """Roles are generators yielding Wait(bar, k); arrivals are made inline
    (``bar.arrive()``) or queued as tensor-core commits (``commit``), which
    land in issue order at random later times."""

    def __init__(self, seed: int):
        self.rng = random.Random(seed)
        self.commits: deque[Barrier] = deque()
        self.roles: list = []

    def commit(self, bar: Barrier):
        self.commits.append(bar)

    def run(self, max_events: int = 2_000_000):
        blocked = {i: None for i in range(len(self.roles))}
        done = set()
        for _ in range(max_events):
            runnable = []
            for i, role in enumerate(self.roles):
                if i in done:
                    continue
                w = blocked[i]
                if w is not None:
                    # the window the parity test needs, at every look
                    assert w.k <= w.bar.completed + 1 and w.bar.completed <= w.k + 1, (
                        f"{w.bar.name}: waiting for completion {w.k} with {w.bar.completed} done")
                    if w.bar.completed < w.k + 1:
                        continue
                runnable.append(i)
            choices = runnable + (["commit"] if self.commits else [])
            if not choices:
                assert len(done) == len(self.roles), "deadlock: every role waits and no commit is in flight"
                return
            pick = self.rng.choice(choices)
            if pick == "commit":
                self.commits.popleft().arrive()
                continue
            try:
                blocked[pick] = next(self.roles[pick])
            except StopIteration:
                done.add(pick)
                blocked[pick] = None
        raise AssertionError("the simulation did not finish")


def persistent_gemm(sim: Sim, tiles: int, nk: int):
    """tc_gemm_persistent_kernel: 4 TMA stages, 2 X_lo buffers, hi.hi groups
    of 2 stages in 3 buffers, one cross accumulator per tile."""
    S, G, PROMOTE = 4, 3, 2
    full = [Barrier(f"full{s}", 1) for s in range(S)]
    conv = [Barrier(f"conv{s}", 1) for s in range(S)]
    empty = [Barrier(f"empty{s}", 1) for s in range(S)]
    acc_full = [Barrier(f"acc_full{j}", 1) for j in range(G)]
    acc_empty = [Barrier(f"acc_empty{j}", 1) for j in range(G)]
    tile_full, tile_empty = Barrier("tile_full", 1), Barrier("tile_empty", 1)
    groups = (nk + PROMOTE - 1) // PROMOTE

    def producer():
        for i in range(tiles * nk):
            if i >= S:
                yield Wait(empty[i % S], i // S - 1)
            sim.commit(full[i % S])  # the TMA lands later, in order

    def split():
        for i in range(tiles * nk):
            yield Wait(full[i % S], i // S)
            if i >= 2:
                yield Wait(empty[(i - 2) % S], (i - 2) // S)  # X_lo buffer i % 2
            conv[i % S].arrive()

    def mma():
        group = 0
        for u in range(tiles):
            for j in range(nk):
                i = u * nk + j
                first, last = j % PROMOTE == 0, j % PROMOTE == PROMOTE - 1 or j == nk - 1
                yield Wait(conv[i % S], i // S)
                if j == 0 and u >= 1:
                    yield Wait(tile_empty, u - 1)
                if first and group >= G:
                    yield Wait(acc_empty[group % G], group // G - 1)
                sim.commit(empty[i % S])
                if last:
                    sim.commit(acc_full[group % G])
                    group += 1
                if j == nk - 1:
                    sim.commit(tile_full)

    def epilogue():
        group = 0
        for u in range(tiles):
            for _ in range(groups):
                yield Wait(acc_full[group % G], group // G)
                acc_empty[group % G].arrive()
                group += 1
            yield Wait(tile_full, u)
            tile_empty.arrive()

    sim.roles = [producer(), split(), mma(), epilogue()]


def pair_gemm(sim: Sim, tiles: int, nk: int):
    """tc_gemm_pair_kernel: per CTA 4 TMA stages and 3 X_lo buffers; the
    leader's MMA waits for both CTAs' split stage (conv, 2 arrivals: the
    leader's split and the peer's forwarder), commits to both CTAs' empty and
    acc_full; both epilogues release a group on the leader's acc_empty."""
    S, XLO, PROMOTE = 4, 3, 2
    full = [[Barrier(f"full{r}.{s}", 1) for s in range(S)] for r in range(2)]
    empty = [[Barrier(f"empty{r}.{s}", 1) for s in range(S)] for r in range(2)]
    conv = [Barrier(f"conv{s}", 2) for s in range(S)]
    sdone = [Barrier(f"sdone{s}", 1) for s in range(S)]
    acc_full = [[Barrier(f"acc_full{r}.{j}", 1) for j in range(2)] for r in range(2)]
    acc_empty = [Barrier(f"acc_empty{j}", 2) for j in range(2)]
    groups = (nk + PROMOTE - 1) // PROMOTE

    def producer(r):
        for i in range(tiles * nk):
            if i >= S:
                yield Wait(empty[r][i % S], i // S - 1)
            sim.commit(full[r][i % S])

    def split(r):
        for i in range(tiles * nk):
            yield Wait(full[r][i % S], i // S)
            if i >= XLO:
                yield Wait(empty[r][(i - XLO) % S], (i - XLO) // S)
            (conv if r == 0 else sdone)[i % S].arrive()

    def forwarder():
        for i in range(tiles * nk):
            yield Wait(sdone[i % S], i // S)
            conv[i % S].arrive()

    def mma():
        group = 0
        for u in range(tiles):
            for j in range(nk):
                i = u * nk + j
                first, last = j % PROMOTE == 0, j % PROMOTE == PROMOTE - 1 or j == nk - 1
                yield Wait(conv[i % S], i // S)
                if first and group >= 2:
                    yield Wait(acc_empty[group % 2], group // 2 - 1)
                for r in range(2):
                    sim.commit(empty[r][i % S])
                if last:
                    for r in range(2):
                        sim.commit(acc_full[r][group % 2])
                    group += 1

    def epilogue(r):
        group = 0
        for _ in range(tiles):
            for _ in range(groups):
                yield Wait(acc_full[r][group % 2], group // 2)
                acc_empty[group % 2].arrive()
                group += 1

    sim.roles = [producer(0), producer(1), split(0), split(1), forwarder(), mma(), epilogue(0), epilogue(1)]


def prefill_attention(sim: Sim, nt: int):
    """tc_prefill_attention_kernel: K and V^T rings of 2 stages refilled on
    the scores' (s_full) and P V (o_full) commits of the tile two back; two
    softmax sets take alternate tiles."""
    KS, VS = 2, 2
    q_full = Barrier("q_full", 1)
    k_full = [Barrier(f"k_full{s}", 1) for s in range(KS)]
    v_full = [Barrier(f"v_full{s}", 1) for s in range(VS)]
    s_full = [Barrier(f"s_full{x}", 1) for x in range(2)]
    p_full = [Barrier(f"p_full{x}", 1) for x in range(2)]
    o_full = [Barrier(f"o_full{x}", 1) for x in range(2)]

    def k_producer():
        sim.commit(q_full)
        for t in range(nt):
            if t >= KS:
                yield Wait(s_full[t & 1], (t - KS) >> 1)
            sim.commit(k_full[t % KS])

    def v_producer():
        for t in range(nt):
            if t >= VS:
                yield Wait(o_full[t & 1], (t - VS) >> 1)
            sim.commit(v_full[t % VS])

    def mma():
        yield Wait(q_full, 0)

        def scores(t):
            x, u = t & 1, t >> 1
            yield Wait(k_full[t % KS], t // KS)
            if u >= 1:
                yield Wait(o_full[x], u - 1)
            sim.commit(s_full[x])

        if nt > 0:
            yield from scores(0)
        for t in range(nt):
            if t + 1 < nt:
                yield from scores(t + 1)
            x, u = t & 1, t >> 1
            yield Wait(v_full[t % VS], t // VS)
            yield Wait(p_full[x], u)
            sim.commit(o_full[x])

    def softmax(x):
        for t in range(x, nt, 2):
            u = t >> 1
            yield Wait(s_full[x], u)
            p_full[x].arrive()
            yield Wait(o_full[x], u)

    sim.roles = [k_producer(), v_producer(), mma(), softmax(0), softmax(1)]


@pytest.mark.parametrize("tiles,nk", [(1, 1), (1, 18), (3, 18), (2, 48), (4, 3), (5, 2)])
def test_persistent_gemm_protocol(tiles, nk):
    for seed in range(40):
        sim = Sim(seed)
        persistent_gemm(sim, tiles, nk)
        sim.run()


@pytest.mark.parametrize("tiles,nk", [(1, 1), (1, 18), (3, 18), (2, 48), (4, 3), (5, 2)])
def test_pair_gemm_protocol(tiles, nk):
    for seed in range(40):
        sim = Sim(seed)
        pair_gemm(sim, tiles, nk)
        sim.run()


@pytest.mark.parametrize("nt", [1, 2, 3, 4, 9, 40])
def test_prefill_attention_protocol(nt):
    for seed in range(60):
        sim = Sim(seed)
        prefill_attention(sim, nt)
        sim.run()


def test_the_window_check_catches_an_alias():
    """The same attention producer with three K stages released by s_full
    (the form rejected for aliasing) fails the window check."""
    failures = 0
    for seed in range(60):
        sim = Sim(seed)
        prefill_attention(sim, 12)
        # rebuild the K producer with three stages released by s_full of tile t - 3
        k_full = [Barrier(f"k_full{s}", 1) for s in range(3)]
        s_full = [Barrier(f"s_full{x}", 1) for x in range(2)]

        def k_producer():
            for t in range(12):
                if t >= 3:
                    yield Wait(s_full[t & 1], (t - 3) >> 1)
                sim.commit(k_full[t % 3])

        def scores_only():
            for t in range(12):
                yield Wait(k_full[t % 3], t // 3)
                sim.commit(s_full[t & 1])

        sim.roles = [k_producer(), scores_only()]
        try:
            sim.run()
        except AssertionError:
            failures += 1
    assert failures > 0
