"""CPU model of the CTA pair's error drain (gemm_sm100.cuh, teardown).

In a cta_group::2 pair both CTAs' TMA loads of a pipeline stage are credited to the
leader's full barrier for that stage: the leader arms it (arrive + expect_tx of both
CTAs' bytes) and each CTA's bytes complete part of the transaction count when they
land. After an abort, the leader walks the last S stage indices of the larger of the
two producers' issued counts: a stage the leader never armed is armed for the peer's
bytes alone, a stage the peer never loaded has its bytes taken off
(mbarrier.complete_tx), and each phase is waited for, so no load is still in flight
when the CTAs exit.

This model plays the protocol with random interleavings of issue, landing and
consumption and a random abort point, then applies the drain and checks:
  * every stage either CTA issued has landed once the drained phases have completed;
  * no fix-up ever touches a phase that had already completed (an arrive or
    complete_tx on a completed phase would corrupt the next one);
  * the drain never waits on a phase that cannot complete.
"""
from __future__ import annotations

import random

import pytest

STAGE = 3  # bytes of one CTA's share of a stage, in arbitrary units


class Barrier:
    """mbarrier with an arrival count of 1 and a signed transaction count."""

    def __init__(self):
        self.phase = 0      # completed phases
        self.pending = 1    # arrivals still expected in the current phase
        self.tx = 0         # transaction bytes still expected (may go negative)

    def _maybe_complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending, self.tx = 1, 0

    def arrive_expect_tx(self, nbytes):
        assert self.pending == 1, "second arrive in one phase"
        self.tx += nbytes
        self.pending -= 1
        self._maybe_complete()

    def complete_tx(self, nbytes):
        self.tx -= nbytes
        self._maybe_complete()


def play(S, n_stages, rng, abort_at):
    full = [Barrier() for _ in range(S)]
    issued = {"lead": 0, "peer": 0}
    consumed = 0
    in_flight = []  # (who, stage index) loads issued but not landed
    steps = 0
    aborted = False
    while True:
        steps += 1
        if steps == abort_at:
            aborted = True
        moves = []
        for who in ("lead", "peer"):
            i = issued[who]
            # a producer issues stage i once the MMA consumed stage i - S
            if not aborted and i < n_stages and consumed >= i - S + 1:
                moves.append(("issue", who))
        if in_flight:
            moves.append(("land", None))
        i = consumed
        if not aborted and i < n_stages and full[i % S].phase > i // S:
            moves.append(("consume", None))
        if not moves:
            break
        kind, who = rng.choice(moves)
        if kind == "issue":
            i = issued[who]
            if who == "lead":
                full[i % S].arrive_expect_tx(2 * STAGE)
            in_flight.append((who, i))
            issued[who] += 1
        elif kind == "land":
            _, i = in_flight.pop(rng.randrange(len(in_flight)))
            full[i % S].complete_tx(STAGE)
        else:
            consumed += 1
    return full, issued, consumed, in_flight


def drain(full, S, il, ip, in_flight, rng):
    hi = max(il, ip)
    for i in range(max(hi - S, 0), hi):
        b = full[i % S]
        done = b.phase > i // S
        if i >= il:
            assert not done, "fix-up on a completed phase (leader never armed it)"
            b.arrive_expect_tx(STAGE)
        elif i >= ip:
            assert not done, "fix-up on a completed phase (peer never loaded it)"
            b.complete_tx(STAGE)
        # wait: loads still in flight land in any order meanwhile
        while b.phase <= i // S:
            assert in_flight, f"stage {i} cannot complete"
            _, j = in_flight.pop(rng.randrange(len(in_flight)))
            full[j % S].complete_tx(STAGE)
    return in_flight


@pytest.mark.parametrize("S", [2, 3, 4])
def test_drain_completes_every_in_flight_stage(S):
    rng = random.Random(1000 + S)
    for _ in range(3000):
        n_stages = rng.randint(1, 24)
        abort_at = rng.randint(1, 80)
        full, issued, consumed, in_flight = play(S, n_stages, rng, abort_at)
        il, ip = issued["lead"], issued["peer"]
        # the producers can be at most S stages apart
        assert abs(il - ip) <= S
        left = drain(full, S, il, ip, in_flight, rng)
        # every load of a stage in the drained window has landed
        lo = max(max(il, ip) - S, 0)
        assert not [j for _, j in left if j >= lo], left
        # loads below the window were consumed, hence landed, before the abort
        assert not [j for _, j in left if j < lo], left
