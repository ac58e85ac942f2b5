"""A host model of the expert FFN kernels' work-item claiming (tideway_b200/csrc/ffn_sched.cuh).

Up items (segment u, up tile) come from one counter in segment order; every up item's chunks
are published by `per_tile` epilogue warps, and the arrival that completes a segment's count
(`up_target`: up tiles x per_tile x route chunks) appends the segment to the ready list; down
items are tickets over that list; a producer whose ticket names a slot not yet listed keeps
it pending and claims up work meanwhile.  The model runs several producers (each busy for a
random time on the item it claimed, its epilogue publishing only after that) and the epilogue
arrivals with random interleavings and checks that every item is claimed once, that a down
item starts only after every arrival of its segment's up items, and that the launch drains.
It also shows what a target that counts fewer epilogue warps than publish would do: down
items starting before their activations are complete.
"""

from __future__ import annotations

import random

import pytest


def up_target(tu: int, per_tile: int, n: int, n_cap: int) -> int:
    return tu * per_tile * ((n + n_cap - 1) // n_cap)


def simulate(seg_routes, tu, td, n_cap, per_tile, target_warps, producers, seed):
    rng = random.Random(seed)
    U = len(seg_routes)
    up_ctr = down_ctr = 0
    ready = []                      # slots in completion order
    up_done = [0] * U               # arrivals per segment
    arrivals_left = {}              # up item -> arrivals still to publish
    claimed = []
    early = 0
    pending = [None] * producers    # a down ticket per producer
    up_left = [True] * producers
    finished = [False] * producers
    busy = [0] * producers          # turns left on the producer's current item
    streaming = [None] * producers  # its up item, published once streamed
    n_up, n_dn = U * tu, U * td
    for _ in range(200000):
        if all(finished) and not arrivals_left and not any(streaming):
            break
        # an epilogue warp publishes one arrival of some finished up item
        if arrivals_left and rng.random() < 0.5:
            item = rng.choice(sorted(arrivals_left))
            u = item[1]
            arrivals_left[item] -= 1
            if arrivals_left[item] == 0:
                del arrivals_left[item]
            up_done[u] += 1
            if up_done[u] == up_target(tu, target_warps, seg_routes[u], n_cap):
                ready.append(u)
            continue
        p = rng.randrange(producers)
        if finished[p]:
            continue
        if busy[p]:  # the producer's CTA is still streaming its last item
            busy[p] -= 1
            if busy[p] == 0 and streaming[p] is not None:
                item, chunks = streaming[p]
                arrivals_left[item] = per_tile * chunks  # its epilogue may now publish
                streaming[p] = None
            continue
        if pending[p] is None:
            if down_ctr >= n_dn:
                finished[p] = True
                continue
            if not up_left[p] or down_ctr < len(ready) * td:
                x = down_ctr
                down_ctr += 1
                pending[p] = x
        if pending[p] is not None:
            x = pending[p]
            if x // td < len(ready):
                u = ready[x // td]
                full = up_target(tu, per_tile, seg_routes[u], n_cap)
                if up_done[u] < full:
                    early += 1
                claimed.append(("down", u, x % td))
                pending[p] = None
                busy[p] = rng.randint(1, 24)
                continue
        if up_left[p]:
            x = up_ctr
            up_ctr += 1
            if x < n_up:
                u, tile = divmod(x, tu)
                claimed.append(("up", u, tile))
                chunks = (seg_routes[u] + n_cap - 1) // n_cap
                streaming[p] = (("up", u, tile), chunks)
                busy[p] = rng.randint(1, 24)
                continue
            up_left[p] = False
    drained = all(finished) and not arrivals_left and not any(streaming)
    return claimed, early, drained


@pytest.mark.parametrize("seg_routes,n_cap,per_tile", [([3, 1, 2, 8] * 2, 16, 8),
                                                       ([40, 17, 160, 1] * 2, 16, 8),
                                                       ([300, 90, 5] * 2, 160, 16),
                                                       ([1] * 12, 16, 8)])
def test_claims_are_complete_and_down_waits_for_every_up_arrival(seg_routes, n_cap, per_tile):
    tu, td = 3, 4
    overlapped = 0
    for seed in range(30):
        claimed, early, drained = simulate(seg_routes, tu, td, n_cap, per_tile, per_tile, 5,
                                           seed)
        assert drained, seed
        assert early == 0, seed
        U = len(seg_routes)
        want = {("up", u, t) for u in range(U) for t in range(tu)} | \
               {("down", u, t) for u in range(U) for t in range(td)}
        assert sorted(claimed) == sorted(want)  # every item exactly once
        first_down = next(i for i, c in enumerate(claimed) if c[0] == "down")
        last_up = max(i for i, c in enumerate(claimed) if c[0] == "up")
        overlapped += first_down < last_up
    assert overlapped > 0  # some runs start down work while up work is still being claimed


def test_a_target_for_fewer_warps_than_publish_starts_down_items_early():
    """Sixteen epilogue warps publish every chunk while the target counts eight."""
    early = sum(simulate([300, 90, 5] * 2, 3, 4, 160, 16, 8, 5, seed)[1] for seed in range(30))
    assert early > 0
