"""A host model of the expert-parallel peer-memory exchange (tideway_b200/csrc/ep_p2p.cu).

Every rank runs, per exchange s (one MoE layer): dispatch -- store its rows into every peer's
receive rows, raise its dispatch flag to s on every peer, wait until every peer's dispatch
flag in its own header reads s; the FFN over the received rows; combine -- store each
received row's partial into its source's return rows, raise its combine flag to s on every
peer, wait until every combine flag reads s, read the returned partials.  Flags hold the
exchange count and are never cleared; waits test for equality.  Stores to different peers
land in any order and ranks run at random relative speeds.

Checked for 2 to 8 ranks: every read sees the rows of its own exchange, no row is
overwritten before its reader consumed the previous exchange's contents, no flag moves past
the count its reader waits for, and every rank finishes.  Dropping one rule (the combine
wait) makes the model find stale reads.
"""

from __future__ import annotations

import random

import pytest

# phases of one exchange on one rank
DW, DF, DWAIT, FFN, CW, CF, CWAIT, CREAD = range(8)


def simulate(world: int, steps: int, seed: int, combine_wait: bool = True):
    rng = random.Random(seed)
    recv = [[0] * world for _ in range(world)]    # recv[d][src]: exchange whose rows landed
    back = [[0] * world for _ in range(world)]    # back[d][src]: exchange of src's partials
    fdisp = [[0] * world for _ in range(world)]   # dispatch flags in d's header, per source
    fcomb = [[0] * world for _ in range(world)]
    consumed_recv = [0] * world                   # last exchange whose rows the FFN read
    consumed_back = [0] * world                   # last exchange whose partials were read
    phase = [DW] * world
    step = [1] * world
    todo = [list(range(world)) for _ in range(world)]  # peers not yet stored to / flagged
    problems = []

    def finished(r):
        return step[r] > steps

    for _ in range(steps * world * world * 40):
        live = [r for r in range(world) if not finished(r)]
        if not live:
            break
        r = rng.choice(live)
        s, ph = step[r], phase[r]
        if ph in (DW, DF, CW, CF):
            d = todo[r].pop(rng.randrange(len(todo[r])))  # one peer's store lands
            if ph == DW:
                if consumed_recv[d] < s - 1:
                    problems.append(("receive rows overwritten before read", r, d, s))
                recv[d][r] = s
            elif ph == CW:
                if consumed_back[d] < s - 1:
                    problems.append(("return rows overwritten before read", r, d, s))
                back[d][r] = s
            else:
                flags = fdisp if ph == DF else fcomb
                if flags[d][r] != s - 1:
                    problems.append(("flag skipped a count", r, d, s))
                flags[d][r] = s
            if not todo[r]:
                todo[r] = list(range(world))
                phase[r] += 1
        elif ph in (DWAIT, CWAIT):
            flags = fdisp if ph == DWAIT else fcomb
            if any(f > s for f in flags[r]):
                problems.append(("flag ahead of its waiter", r, s))
            if ph == CWAIT and not combine_wait:
                phase[r] += 1
            elif all(f == s for f in flags[r]):
                phase[r] += 1
        elif ph == FFN:
            if any(v != s for v in recv[r]):
                problems.append(("FFN read rows of another exchange", r, s))
            consumed_recv[r] = s
            phase[r] += 1
        else:  # CREAD
            if any(v != s for v in back[r]):
                problems.append(("combine read partials of another exchange", r, s))
            consumed_back[r] = s
            phase[r], step[r] = DW, s + 1
    return problems, all(finished(r) for r in range(world))


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_exchange_protocol_is_race_free_and_finishes(world):
    for seed in range(25):
        problems, done = simulate(world, 12, seed)
        assert not problems, (world, seed, problems[:3])
        assert done, (world, seed)


def test_without_the_combine_wait_partials_are_read_stale():
    found = sum(len(simulate(4, 12, seed, combine_wait=False)[0]) for seed in range(25))
    assert found > 0
