"""The tensor-core prefill kernel's K/V ring, checked on the CPU with parity waits.

``prefill_tc_kernel`` (miniserve_b200/csrc/prefill_tc.cuh) streams K and V blocks through a
3-slot ring in the order K_0, K_1, V_0, K_2, V_1, ...: the producer waits for a slot's ``empty``
barrier and loads the next block into it; the S issuer (S = Q K_j^T for each tile) and the P*V
issuer (O += P V_j) wait for the slot's ``full`` barrier and, once their MMAs complete, release it.

Those ``full`` waits are parity waits (``mbarrier.test_wait.parity``): a wait for a slot's fill k
passes whenever the barrier's phase parity differs from k's, so it is exact only while the slot's
previous fill has completed.  The slot's previous fill is the other issuer's block (V_j's slot
last held K_j, K_j's held V_{j-3}), so each issuer must take its wait only once something it has
observed implies that fill landed:
* the P*V issuer waits for V_j after the first P(j) is ready (P(j) follows S(j), which read K_j);
* the S issuer waits for K_j after the first tile's s_free(j - 1), which that tile's softmax
  arrives on after its wait for P*V(j - 3), which read V_{j-3}.
The kernel used to take both waits first (V_j right after issuing P*V(j - 1), K_j before any
s_free), which was correct only while loads landed in time.  This test restates the protocol as
agents over barrier phases, with loads landing and MMAs completing at random later steps, and
checks every block an MMA reads: the wait order as shipped never reads a stale slot, and the
earlier order does under some schedules.
"""

from __future__ import annotations

import random

NS = 3


class Bar:
    """Completed-phase counter of an mbarrier with one expected arrival per phase."""

    def __init__(self) -> None:
        self.phase = 0

    def arrive(self) -> None:
        self.phase += 1

    def parity_ok(self, k: int) -> bool:
        """mbarrier.test_wait.parity for phase k: true when the current phase parity differs."""
        return (self.phase & 1) != (k & 1)


def simulate(n_a: int, n_b: int, gated: bool, seed: int) -> list[str]:
    """One CTA whose tiles see n_a and n_b blocks; returns the stale reads and stalls found."""
    rng = random.Random(seed)
    nblk = max(n_a, n_b)
    nt = (n_a, n_b)
    errors: list[str] = []

    def pos_k(j: int) -> int:
        return 0 if j == 0 else 2 * j - 1

    def pos_v(j: int) -> int:
        return 2 * j + 2 if j + 1 < nblk else 2 * j + 1

    items = {}
    for j in range(nblk):
        items[pos_k(j)] = ("K", j)
        items[pos_v(j)] = ("V", j)
    full, empty = [Bar() for _ in range(NS)], [Bar() for _ in range(NS)]
    content: list[object] = [None] * NS
    s_full, s_free, p_full, pv_done = ([0, 0] for _ in range(4))  # completed phases per tile
    events: list[tuple] = []  # pending asynchronous completions

    def wait_full(p: int, who: str):
        s, k = p % NS, p // NS
        while not full[s].parity_ok(k):
            yield
        if full[s].phase != k + 1:
            errors.append(f"{who} passed the wait for position {p} with {full[s].phase} fills of slot {s}")

    def producer():
        for p in range(2 * nblk):
            s = p % NS
            if p >= NS:
                while not empty[s].parity_ok(p // NS - 1):
                    yield
            events.append(("land", s, items[p]))
            yield

    def s_issuer():
        for j in range(nblk):
            tiles = [t for t in (0, 1) if j < nt[t]]
            waited = False
            if not gated:
                yield from wait_full(pos_k(j), f"S({j})")
                waited = True
            for t in tiles:
                while j > 0 and s_free[t] < j:
                    yield
                if not waited:
                    yield from wait_full(pos_k(j), f"S({j})")
                    waited = True
                if content[pos_k(j) % NS] != ("K", j):
                    errors.append(f"S_{t}({j}) read {content[pos_k(j) % NS]}")
                events.append(("s_done", t, j, t == tiles[-1], pos_k(j) % NS))
                yield

    def pv_issuer():
        for j in range(nblk):
            pend = [t for t in (0, 1) if j < nt[t]]
            waited = False
            if not gated:
                yield from wait_full(pos_v(j), f"PV({j})")
                waited = True
            while pend:
                ready = [t for t in pend if p_full[t] > j]
                if not ready:
                    yield
                    continue
                if not waited:
                    yield from wait_full(pos_v(j), f"PV({j})")
                    waited = True
                t = ready[0]
                if content[pos_v(j) % NS] != ("V", j):
                    errors.append(f"PV_{t}({j}) read {content[pos_v(j) % NS]}")
                pend.remove(t)
                events.append(("pv_done", t, j, not pend, pos_v(j) % NS))
                yield

    def softmax(t: int):
        for j in range(nt[t]):
            while s_full[t] <= j:
                yield
            s_free[t] += 1
            while j > 0 and pv_done[t] < j:
                yield
            p_full[t] += 1
            yield
        while nt[t] > 0 and pv_done[t] < nt[t]:
            yield

    agents = {"prod": producer(), "s": s_issuer(), "pv": pv_issuer(), "sm0": softmax(0), "sm1": softmax(1)}
    live = dict(agents)
    for _ in range(200_000):
        if not live and not events:
            return errors
        if events and (not live or rng.random() < 0.25):
            ev = events.pop(rng.randrange(len(events)))
            if ev[0] == "land":
                _, s, item = ev
                content[s] = item
                full[s].arrive()
            else:  # an MMA completed; the issuer's commit releases the slot after its last tile
                kind, t, j, last, slot = ev
                if kind == "s_done":
                    s_full[t] += 1
                else:
                    pv_done[t] += 1
                if last:
                    empty[slot].arrive()
            continue
        name = rng.choice(list(live))
        try:
            next(live[name])
        except StopIteration:
            del live[name]
    errors.append(f"no progress (tiles {n_a}, {n_b})")
    return errors


def test_shipped_wait_order_never_reads_a_stale_slot() -> None:
    for n_a in range(0, 9):
        for n_b in range(1, 9):
            for seed in range(12):
                errors = simulate(n_a, n_b, gated=True, seed=seed)
                assert not errors, (n_a, n_b, seed, errors[:3])


def test_shipped_wait_order_on_config3_like_tiles() -> None:
    for n_a, n_b in ((5, 12), (3, 12), (8, 9), (0, 7)):
        for seed in range(150):
            errors = simulate(n_a, n_b, gated=True, seed=seed)
            assert not errors, (n_a, n_b, seed, errors[:3])


def test_earlier_wait_order_reads_stale_slots() -> None:
    """Both issuers' early waits pass on a slot whose previous fill had not landed."""
    found = [e for n_a, n_b in ((5, 8), (3, 12), (8, 8), (2, 6)) for seed in range(150)
             for e in simulate(n_a, n_b, gated=False, seed=seed)]
    assert any(e.startswith("S(") for e in found), "no stale K wait found"
    assert any(e.startswith("PV(") for e in found), "no stale V wait found"
