"""A host-side model of the mbarrier protocol of the tcgen05 GEMM pipelines (idol.cpp_b200/csrc/q8_gemm.cu), run under
random out-of-order completion of the stage copies.

An mbarrier parity wait only tells the current phase from the one before it, so a waiter that can run two phases
ahead of a barrier passes early. In both GEMM kernels the dequantisation warps form two groups that take alternate k
stages; with an odd number S of stage slots, stage i and stage i - S of one slot belong to different groups, and the
group of stage i can reach its wait on the slot's `full` barrier while the copies of stage i - S are still in flight.
The kernels therefore first wait for a commit that implies stage i - S was consumed (the slot's previous commit in the
one-CTA kernel, the A slot's in the persistent kernel). This model checks that, with those waits, no group reads a
slot before its own stage's copies have landed and no A slot is rewritten before the MMA that read it has completed,
and that dropping the ordering wait with an odd S does break (so the model can see the failure it guards against).
"""
import heapq
import random

import pytest


class Barrier:
    """mbarrier phase and arrival count; wait(parity) passes while the current phase's parity differs from it."""

    def __init__(self, count):
        self.count = count
        self.pending = count
        self.phase = 0

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count

    def passed(self, parity):
        return (self.phase & 1) != parity


def simulate(S, SA, nks, seed, order_waits=True, persistent=False):
    """One run of producer, two dequant groups and the MMA thread over nks stages. Copies land after a random delay
    (out of order); dequant and MMA steps take random times. Returns the list of protocol violations (a deadlock
    among them: an early pass corrupts the arrival counts of later phases)."""
    rng = random.Random(seed)
    full = [Barrier(1) for _ in range(S)]
    empty = [Barrier(1) for _ in range(S)]
    afull = [Barrier(1) for _ in range(SA)]  # one arrival per group (its four warps folded into one)
    slot_holds = [None] * S
    committed = [False] * nks
    events, seq, now = [], [0], [0]
    violations = []

    def at(t, fn):
        seq[0] += 1
        heapq.heappush(events, (t, seq[0], fn))

    def producer():
        for i in range(nks):
            s, u = i % S, i // S
            if i >= S:
                yield ("wait", empty[s], (u - 1) & 1)

            def land(i=i, s=s):
                slot_holds[s] = i
                full[s].arrive()

            at(now[0] + rng.randint(1, 40), land)
            yield ("sleep", 1)

    def group(g):
        for i in range(g, nks, 2):
            s, u = i % S, i // S
            if persistent:
                # q8_gemm_persistent_kernel: the A-slot wait (commit of stage i - SA) comes first; with SA == S
                # (S even) there is none, the slot's own full barrier implying that commit.
                if order_waits and SA < S and i >= SA:
                    r = i - SA
                    yield ("wait", empty[r % S], (r // S) & 1)
                yield ("wait", full[s], u & 1)
                if not order_waits and SA < S and i >= SA:
                    r = i - SA
                    yield ("wait", empty[r % S], (r // S) & 1)
            else:
                # q8_gemm_kernel: with an odd S, the slot's previous commit first (A slot = stage slot, SA = S).
                if order_waits and S % 2 == 1 and i >= S:
                    yield ("wait", empty[s], (u - 1) & 1)
                yield ("wait", full[s], u & 1)
            if slot_holds[s] != i:
                violations.append(f"stage {i} read slot {s} holding stage {slot_holds[s]} at t={now[0]}")
            if i >= SA and not committed[i - SA]:
                violations.append(f"stage {i} rewrote A slot {i % SA} before the MMA of stage {i - SA}")
            yield ("sleep", rng.randint(1, 6))
            afull[i % SA].arrive()

    def mma():
        for i in range(nks):
            yield ("wait", afull[i % SA], (i // SA) & 1)
            yield ("sleep", rng.randint(2, 5))
            committed[i] = True
            empty[i % S].arrive()

    waiting = {}

    def step(agent):
        try:
            op = next(agent)
        except StopIteration:
            return
        if op[0] == "sleep":
            at(now[0] + op[1], lambda: step(agent))
        else:
            waiting[agent] = op

    for agent in (producer(), group(0), group(1), mma()):
        at(0, lambda agent=agent: step(agent))
    while True:
        progressed = True
        while progressed:
            progressed = False
            for agent, (_, bar, parity) in list(waiting.items()):
                if bar.passed(parity):
                    del waiting[agent]
                    step(agent)
                    progressed = True
        if not events:
            break
        t, _, fn = heapq.heappop(events)
        now[0] = t
        fn()
    if waiting:
        violations.append("deadlock: " + ", ".join(f"a wait on parity {parity}" for _, _, parity in waiting.values()))
    elif not all(committed):
        violations.append("not every stage was multiplied")
    return violations


# (S, SA, persistent): the shipped configurations of both kernels.
CONFIGS = [(5, 5, False), (4, 4, False), (6, 6, False), (5, 4, True), (6, 4, True), (4, 4, True), (8, 8, True)]


@pytest.mark.parametrize("S,SA,persistent", CONFIGS)
def test_no_stage_is_read_before_it_lands(S, SA, persistent):
    for seed in range(300):
        assert simulate(S, SA, 47, seed, persistent=persistent) == [], (S, SA, persistent, seed)


@pytest.mark.parametrize("S,SA,persistent", [(5, 5, False), (5, 4, True)])
def test_the_model_sees_the_race_without_the_ordering_wait(S, SA, persistent):
    bad = sum(bool(simulate(S, SA, 47, seed, order_waits=False, persistent=persistent)) for seed in range(300))
    assert bad > 0
