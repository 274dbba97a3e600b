"""CPU model of the int8 kernel's int8-tile ring (frn_fused_linear_w8.cu).

One loader thread fills QST slots in k-block order.  Four converter warps
take the k-block sequence in turn (warp w: k-blocks w, w+4, ...).  A
converter waits on its slot's `qfull` mbarrier, then releases the slot on
`qempty`.

mbarrier waits are by phase parity: `try_wait.parity(P)` succeeds once the
phase of parity P has completed, which also holds while the barrier sits in
the phase after one of parity P.  A waiter that arrives two phases early
therefore passes at once.

The model runs random interleavings: loads land out of order after random
latencies, and conversions take random times.  It checks two invariants:
- every converter converts exactly the tile of its k-block, after it landed;
- no load is issued into a slot before that slot's previous tile was released.

The protocol without the converters' release wait (waiting on `qfull` by
parity alone) is run as a planted mistake: the model must catch it.
"""
import random

import pytest


class MBarrier:
    """Phase-parity mbarrier: `count` arrivals (and the landing of any
    announced copy) complete the current phase."""

    def __init__(self, count: int):
        self.count = count
        self.phase = 0          # index of the current, incomplete phase
        self.arrived = 0
        self.pending_copies = 0

    def arrive(self, copies: int = 0):
        self.arrived += 1
        self.pending_copies += copies
        self._maybe_complete()

    def copy_landed(self):
        self.pending_copies -= 1
        self._maybe_complete()

    def _maybe_complete(self):
        if self.arrived == self.count and self.pending_copies == 0:
            self.phase += 1
            self.arrived = 0

    def try_wait_parity(self, parity: int) -> bool:
        # Succeeds once the phase of this parity has completed, i.e. while
        # the current (incomplete) phase has the other parity.
        return (self.phase & 1) != parity


def simulate(seed: int, fixed: bool, n_kblocks: int = 96, qst: int = 5, warps: int = 4):
    """One random interleaving.  Returns a list of invariant violations."""
    rng = random.Random(seed)
    qfull = [MBarrier(1) for _ in range(qst)]
    qempty = [MBarrier(1) for _ in range(qst)]
    slot_tile = [None] * qst        # tile that has landed in the slot
    slot_busy = [False] * qst       # a tile is in flight into or sitting in the slot
    in_flight = []                  # (land_time, slot, tile)
    violations = []
    now = 0

    # loader state
    next_load = 0
    # converter state: index into its k-block list, step within one k-block, busy-until
    conv = [{"u": w, "step": 0, "until": 0} for w in range(warps)]

    def loader_step():
        nonlocal next_load
        if next_load >= n_kblocks:
            return False
        u = next_load
        s = u % qst
        if not qempty[s].try_wait_parity(((u // qst) & 1) ^ 1):
            return False
        if slot_busy[s]:
            violations.append(f"load {u} issued into slot {s} before its tile was released")
        slot_busy[s] = True
        qfull[s].arrive(copies=1)
        in_flight.append((now + rng.randint(1, 40), s, u))
        next_load += 1
        return True

    def converter_step(c):
        u = c["u"]
        if u >= n_kblocks or now < c["until"]:
            return False
        s, ph = u % qst, (u // qst) & 1
        if c["step"] == 0:          # the fix: the slot's previous use released first
            if fixed and not qempty[s].try_wait_parity(ph ^ 1):
                return False
            c["step"] = 1
            return True
        if c["step"] == 1:          # the tile landed
            if not qfull[s].try_wait_parity(ph):
                return False
            if slot_tile[s] != u:
                violations.append(f"k-block {u} converted from slot {s} holding {slot_tile[s]}")
            c["step"] = 2
            c["until"] = now + rng.randint(1, 12)   # conversion time
            return True
        # step 2: conversion done -> release the slot, take the next k-block
        slot_busy[s] = False
        slot_tile[s] = None
        qempty[s].arrive()
        c["u"] += warps
        c["step"] = 0
        return True

    for _ in range(200000):
        progressed = False
        # land copies whose time has come, in random order among them
        due = [f for f in in_flight if f[0] <= now]
        rng.shuffle(due)
        for f in due:
            in_flight.remove(f)
            _, s, u = f
            slot_tile[s] = u
            qfull[s].copy_landed()
            progressed = True
        agents = ["L"] + list(range(warps))
        rng.shuffle(agents)
        for a in agents:
            progressed |= loader_step() if a == "L" else converter_step(conv[a])
        if next_load >= n_kblocks and all(c["u"] >= n_kblocks for c in conv) and not in_flight:
            break
        if not progressed:  # jump to the next landing or end of a conversion
            events = [f[0] for f in in_flight] + [c["until"] for c in conv if c["until"] > now]
            if not events:
                violations.append(f"deadlock at t={now}")
                break
            now = min(events)
    else:
        violations.append("did not finish")
    return violations


def test_fixed_protocol_never_converts_a_missing_tile():
    for seed in range(300):
        v = simulate(seed, fixed=True)
        assert not v, f"seed {seed}: {v[:3]}"


@pytest.mark.parametrize("qst", [4, 5, 6, 8])
def test_fixed_protocol_at_every_ring_depth(qst):
    for seed in range(100):
        v = simulate(1000 + seed, fixed=True, qst=qst)
        assert not v, f"QST={qst} seed {seed}: {v[:3]}"


def test_parity_only_wait_is_caught():
    """The planted mistake: converters that wait on `qfull` by parity alone
    convert tiles that have not landed once loads complete out of order."""
    found = [v for seed in range(300) for v in simulate(seed, fixed=False)]
    assert any("converted from slot" in v for v in found)
