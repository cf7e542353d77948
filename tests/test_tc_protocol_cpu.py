"""Deadlock freedom of the tensor-core prefill kernel's barrier protocol, checked on the CPU.

``prefill_tc_kernel`` (miniserve_b200/csrc/prefill_tc.cuh) runs five cooperating agents per CTA:
the TMA producer (a 3-slot K/V ring: K_0, K_1, V_0, K_2, V_1, ...), the S issuer, the P*V issuer
and the two softmax warpgroups (tile A, tile B), which hand work to each other through
mbarriers.  Every wait in the kernel is bounded, so on a GPU a wait cycle shows up only as a
timeout status bit after tens of milliseconds.  This test restates the protocol as sequential
agents over mbarrier phases (instant loads and MMAs: only the dependencies matter) and runs it to
completion for every pair of per-tile block counts up to 40.

The P*V issuer serves the two tiles of an entry in the order their P becomes ready (it polls
both barriers), so the simulation lets it take whichever tile is ready.

The simulator also runs a variant that was tried and not kept (the two warpgroups sharing the
long tile's blocks and taking turns through their exponentials, with the second warpgroup taking
two blocks ahead); that variant closes a wait cycle through the 3-slot ring, which shows that
the check finds cycles.
"""

from __future__ import annotations

NS = 3  # K/V ring slots


class Bar:
    """An mbarrier: a phase completes after `count` arrivals."""

    def __init__(self, count: int = 1) -> None:
        self.count, self.arrived, self.phase = count, 0, 0

    def arrive(self) -> None:
        self.arrived += 1
        if self.arrived == self.count:
            self.arrived, self.phase = 0, self.phase + 1

    def done(self, k: int) -> bool:
        return self.phase > k


def _shared_order(n_s: int, n_l: int, s1: int, lead: int) -> list[tuple[int, int]]:
    """Work order of the shared-blocks variant: blocks 0 .. n_s-1 serve both warpgroups, then the
    second's forward blocks and the first's backward blocks alternate, the second `lead` first."""
    out = [(w, 3) for w in range(n_s)]
    t1 = t0 = 0
    last1 = lead == 0
    while True:
        rem1, rem0 = s1 - n_s - t1, n_l - s1 - t0
        if rem1 <= 0 and rem0 <= 0:
            return out
        if rem0 <= 0 or (rem1 > 0 and (t1 < lead or not last1)):
            out.append((n_s + t1, 2))
            t1 += 1
            last1 = True
        else:
            out.append((n_l - 1 - t0, 1))
            t0 += 1
            last1 = False


def run_protocol(nb_a: int, nb_b: int, has_b: bool, shared: bool = False, lead: int = 0) -> bool:
    """True when every agent finishes for a CTA whose tiles see nb_a / nb_b blocks.

    shared=False: the kernel as shipped (warpgroup t runs tile t's blocks; the entries of the
    work order are blocks 0 .. max-1, each serving the tiles that see it).  shared=True: the
    variant described in the module docstring."""
    if not shared:
        n_a, n_b = nb_a, (nb_b if has_b else 0)
        order = [(j, (1 if j < n_a else 0) | (2 if j < n_b else 0)) for j in range(max(n_a, n_b))]
        runs = {0: [n_a], 1: [n_b]}
        turns = False
        n_blk0 = n_blk1 = 0
    else:
        tl = 1 if (has_b and nb_b >= nb_a) else 0
        n_s = (nb_a if tl == 1 else nb_b) if has_b else 0
        n_l = nb_b if tl == 1 else nb_a
        s1 = (n_s + n_l + 1) // 2
        merge = n_l > s1
        order = _shared_order(n_s, n_l, s1, lead)
        runs = {0: [n_s, n_l - s1 if merge else 0], 1: [s1]}
        turns = True
        n_blk0, n_blk1 = n_s + (n_l - s1 if merge else 0), s1
    n_w = len(order)

    def pos_k(w: int) -> int:
        return 0 if w == 0 else 2 * w - 1

    def pos_v(w: int) -> int:
        return 2 * w + 2 if w + 1 < n_w else 2 * w + 1

    full, empty = [Bar() for _ in range(NS)], [Bar() for _ in range(NS)]
    s_full, s_free, p_full, pv_done, turn = ([Bar(), Bar()] for _ in range(5))

    def producer():
        for p in range(2 * n_w):
            if p >= NS:
                yield lambda p=p: empty[p % NS].done(p // NS - 1)
            full[p % NS].arrive()

    def s_issuer():
        issued = [0, 0]
        for w, (_, slots) in enumerate(order):
            yield lambda p=pos_k(w): full[p % NS].done(p // NS)
            for sl in (0, 1):
                if (slots >> sl) & 1:
                    if issued[sl] > 0:
                        yield lambda sl=sl, k=issued[sl] - 1: s_free[sl].done(k)
                    s_full[sl].arrive()
                    issued[sl] += 1
            empty[pos_k(w) % NS].arrive()

    def pv_issuer():
        # Within an entry the shipped kernel issues the tiles in the order their P becomes ready
        # (it polls both); the variant issues them in tile order.
        issued = [0, 0]
        for w, (_, slots) in enumerate(order):
            yield lambda p=pos_v(w): full[p % NS].done(p // NS)
            pend = [sl for sl in (0, 1) if (slots >> sl) & 1]
            while pend:
                if turns:
                    ready = [pend[0]]
                    yield lambda sl=pend[0], k=issued[pend[0]]: p_full[sl].done(k)
                else:
                    yield lambda pend=tuple(pend), k=tuple(issued): any(
                        p_full[sl].done(k[sl]) for sl in pend)
                    ready = [sl for sl in pend if p_full[sl].done(issued[sl])]
                for sl in ready:
                    pv_done[sl].arrive()
                    issued[sl] += 1
                    pend.remove(sl)
            empty[pos_v(w) % NS].arrive()

    def softmax(sl: int):
        c = 0
        for n in runs[sl]:
            for k in range(n):
                yield lambda c=c: s_full[sl].done(c)
                s_free[sl].arrive()  # S released right after it is read
                if turns and ((c >= 1 and c - 1 < n_blk1) if sl == 0 else c < n_blk0):
                    yield lambda c=c: turn[sl].done(c - 1 if sl == 0 else c)
                if turns and (c < n_blk1 if sl == 0 else c + 1 < n_blk0):
                    turn[1 - sl].arrive()
                if k > 0:
                    yield lambda c=c: pv_done[sl].done(c - 1)  # P buffer free again
                p_full[sl].arrive()
                c += 1
            if n > 0:
                yield lambda c=c: pv_done[sl].done(c - 1)

    agents = [producer(), s_issuer(), pv_issuer(), softmax(0), softmax(1)]
    waits: list = [None] * len(agents)
    finished = [False] * len(agents)
    progress = True
    while progress:
        progress = False
        for i, agent in enumerate(agents):
            while not finished[i]:
                if waits[i] is not None and not waits[i]():
                    break
                try:
                    waits[i] = next(agent)
                except StopIteration:
                    finished[i] = True
                progress = True
    return all(finished)


def test_shipped_protocol_never_deadlocks() -> None:
    # The planner gives tile A no more blocks than tile B, but the kernel does not rely on it.
    stuck = [(a, b) for a in range(41) for b in range(41) if not run_protocol(a, b, True)]
    stuck += [(a, 0) for a in range(41) if not run_protocol(a, 0, False)]
    assert not stuck, f"wait cycle for per-tile block counts {stuck[:10]}"


def test_the_check_finds_wait_cycles() -> None:
    """The shared-blocks variant with turns deadlocks when its second warpgroup runs two blocks
    ahead and the long tile has a few blocks more than the short one (config 3's longest
    zig-zag pair sees 5 and 12); with the first warpgroup leading it is free of cycles."""
    assert not run_protocol(0, 5, True, shared=True, lead=2)
    assert not run_protocol(5, 12, True, shared=True, lead=2)
    assert run_protocol(2, 2, True, shared=True, lead=2)
    assert all(run_protocol(a, b, True, shared=True, lead=0) for a in range(20) for b in range(20))
