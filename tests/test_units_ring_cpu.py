"""The persistent decode kernel's page ring, checked on the CPU.

``paged_decode_units_kernel`` (miniserve_b200/csrc/paged_attention.cuh) splits its consumer warps
into two groups that take the CTA's work units alternately.  Pages reach the consumers through
slots of a shared-memory ring: a producer warp waits for a slot's ``empty`` barrier, arms its
``full`` barrier with the page's byte count and issues the TMA load; a consumer warp waits for
``full`` by parity, reads the page and arrives on ``empty``.

A parity wait (``mbarrier.try_wait.parity p``) passes whenever the barrier's current phase parity
differs from p, so a wait for a slot's fill k is exact only while fill k - 1 has completed: if it
has not, the barrier's parity already differs from k's and the wait passes at once, on stale data.
This test restates the protocol as agents over mbarrier phases (TMA loads complete at a random
later step), runs random schedules, and checks that every page a consumer reads is the one it
waited for and that every agent finishes.

Three layouts are simulated:
- as shipped: each group has its own producer warp and half of the ring (4 slots for its 2
  warps), so within a group a slot's previous fill is a page the same warp consumed (or the
  group's previous unit, finished before the group's merge barrier);
- a variant that was built and not kept: both groups on one ring fed by one producer in unit
  order.  There a group can wait for a slot whose previous fill belongs to the other group and
  has not landed yet; the simulation finds that stale read, which shows the check works;
- per-group rings of 5 slots (considered for a deeper ring): the group's warps take its pages in
  turn, so with an odd slot count a slot's previous fill is the other warp's page, and the
  simulation finds the same stale read.  Hence the kernel's static_assert that the slots of a
  group are a multiple of its warps.
"""

from __future__ import annotations

import random

import pytest

CONSUMER_WARPS, STAGES, GROUPS = 4, 8, 2
GROUP_WARPS = CONSUMER_WARPS // GROUPS


class Bar:
    """An mbarrier with arrival count 1 and an optional transaction count."""

    def __init__(self) -> None:
        self.phase = 0  # completed phases
        self.arrived = False
        self.tx = 0

    def _maybe_complete(self) -> None:
        if self.arrived and self.tx == 0:
            self.arrived = False
            self.phase += 1

    def arrive(self, tx: int = 0) -> bool:
        """False when this phase already had its one arrival (more than the count allows)."""
        if self.arrived:
            return False
        self.arrived = True
        self.tx += tx
        self._maybe_complete()
        return True

    def complete_tx(self, tx: int) -> None:
        self.tx -= tx
        self._maybe_complete()

    def try_wait_parity(self, p: int) -> bool:
        return (self.phase & 1) != p


def simulate(units: list[int], per_group_rings: bool, seed: int, stages: int = STAGES) -> list[str]:
    """Run one CTA over units with the given page counts; returns the violations found."""
    rng = random.Random(seed)
    errors: list[str] = []
    full = [Bar() for _ in range(stages)]
    empty = [Bar() for _ in range(stages)]
    slot_page: list[object] = [None] * stages  # what the slot holds (a page id once loaded)
    in_flight: list[tuple[int, object]] = []  # TMA loads issued, not yet landed: (slot, page)

    def group_units(g: int) -> list[int]:
        return [i for i in range(len(units)) if i % GROUPS == g]

    # Page ids are (unit, page); the ring sequence of a producer is its units' pages in order.
    if per_group_rings:
        gs = stages // GROUPS
        producers = [(g, [(u, j) for u in group_units(g) for j in range(units[u])], g * gs, gs)
                     for g in range(GROUPS)]
    else:
        producers = [(-1, [(u, j) for u in range(len(units)) for j in range(units[u])], 0, stages)]

    def producer(seq: list[tuple[int, int]], base: int, n: int):
        for g, page in enumerate(seq):
            s = base + g % n
            if g >= n:
                while not empty[s].try_wait_parity(((g // n) - 1) & 1):
                    yield False
            if not full[s].arrive(tx=1):
                errors.append(f"second arrival on full[{s}] in one phase")
            in_flight.append((s, page))
            yield True

    def consumer(grp: int, gw: int):
        if per_group_rings:
            base, n = grp * (stages // GROUPS), stages // GROUPS
        else:
            base, n = 0, stages
        g0 = 0
        for u in range(len(units)):
            mine = u % GROUPS == grp
            if not mine:
                if not per_group_rings:
                    g0 += units[u]  # the other group's pages come first in the shared ring
                continue
            # unit start: group barrier (the query tile), then the pages, then the merge barrier
            yield ("bar", grp, u, 0)
            for j in range(gw, units[u], GROUP_WARPS):
                gj = g0 + j
                s = base + gj % n
                while not full[s].try_wait_parity((gj // n) & 1):
                    yield False
                if slot_page[s] != (u, j):
                    errors.append(f"group {grp} read {slot_page[s]} for page {(u, j)} in slot {s}")
                if not empty[s].arrive():
                    errors.append(f"second arrival on empty[{s}] in one phase")
                yield True
            yield ("bar", grp, u, 1)
            g0 += units[u]

    agents: dict[str, object] = {}
    for g, seq, base, n in producers:
        agents[f"p{g}"] = producer(seq, base, n)
    for grp in range(GROUPS):
        for gw in range(GROUP_WARPS):
            agents[f"c{grp}.{gw}"] = consumer(grp, gw)
    parked: dict[str, tuple] = {}  # agents waiting at a group barrier
    live = set(agents)
    steps = 0
    while live or in_flight:
        steps += 1
        if steps > 200_000:
            errors.append("no progress")
            break
        # Land a TMA load now and then (loads complete in order of a random pick).
        if in_flight and rng.random() < 0.3:
            s, page = in_flight.pop(rng.randrange(len(in_flight)))
            slot_page[s] = page
            full[s].complete_tx(1)
            continue
        runnable = [a for a in live if a not in parked]
        if not runnable:
            if in_flight:
                continue
            errors.append(f"deadlock: parked {sorted(parked)}")
            break
        name = rng.choice(runnable)
        try:
            r = next(agents[name])
        except StopIteration:
            live.discard(name)
            continue
        if isinstance(r, tuple):
            parked[name] = r
            # release the group barrier once every warp of the group is parked on it
            grp = r[1]
            members = [f"c{grp}.{w}" for w in range(GROUP_WARPS)]
            if all(parked.get(m) == r for m in members):
                for m in members:
                    del parked[m]
    return errors


def _random_units(rng: random.Random) -> list[int]:
    return [rng.randint(1, 20) for _ in range(rng.randint(1, 8))]


def test_per_group_rings_never_read_a_stale_slot() -> None:
    rng = random.Random(7)
    for seed in range(120):
        units = _random_units(rng)
        errors = simulate(units, per_group_rings=True, seed=seed)
        assert not errors, (units, errors[:3])


@pytest.mark.parametrize("units", [[10, 10], [3, 17, 5, 9], [1], [20, 1, 20, 1, 20]])
def test_per_group_rings_fixed_cases(units: list[int]) -> None:
    for seed in range(20):
        assert not simulate(units, per_group_rings=True, seed=seed)


def test_shared_ring_variant_reads_stale_slots() -> None:
    """The two groups on one ring: some schedule lets a group pass a wait on a slot whose
    previous fill (the other group's page) has not landed."""
    found = []
    for seed in range(20):
        errors = simulate([10, 10, 10, 10], per_group_rings=False, seed=seed)
        if errors:
            found.append(errors[0])
    assert found, "the stale-parity read of the shared-ring variant was not found"


def test_odd_slot_count_per_group_reads_stale_slots() -> None:
    """5 slots per group for 2 warps: the slot of page j + 5 last held page j, the other warp's,
    which some schedule has not landed when the first warp waits on it."""
    found = []
    for seed in range(40):
        errors = simulate([12, 12, 12, 12], per_group_rings=True, seed=seed, stages=10)
        if errors:
            found.append(errors[0])
    assert found, "the stale-parity read of an odd slot count was not found"
