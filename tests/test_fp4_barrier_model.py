"""A host model of the NVFP4 FFN kernel's stage pipeline and its mbarrier parity waits.

The kernel (tideway_b200/csrc/expert_gemm_fp4_tc.cu) moves every 256-K stage `it` through:
a TMA load into smem stage it % S (after the MMAs of stage it - S freed it), a fill of TMEM
A stage it % A by dequant group it % G (after the load landed and the MMAs of stage it - A
freed the A stage), and 16 MMAs by issuer it % I (after the fill), which complete some time
later.  Waits are mbarrier parity waits: a waiter for phase m of a barrier passes as soon as
the barrier's completed-phase count has a parity different from m's -- correct only when the
count is exactly m + 1 when it passes (a count of m - 1, the phase before still open, also
passes: the hazard).

The model runs the agents with random delays and checks, for the kernel's barrier indexing
(stage modulo lcm(stages, consumers)), that no wait ever passes on the wrong phase and that
every data dependency holds; for the indexing by stage alone (one barrier per smem or A
stage, consumed by several groups or issuers), it finds the hazard.
"""

from __future__ import annotations

import math
import random

import pytest


class Barrier:
    def __init__(self):
        self.done = 0  # completed phases

    def passes(self, phase: int) -> bool:
        return (self.done & 1) != (phase & 1)


def simulate(S: int, A: int, G: int, I: int, single_consumer: bool, stages: int, seed: int):
    """Returns (wrong passes, dependency violations, stages whose MMAs completed) of one random
    run."""
    rng = random.Random(seed)
    nF = math.lcm(S, G) if single_consumer else S
    nAE = math.lcm(A, G) if single_consumer else A
    nAF = math.lcm(A, I) if single_consumer else A
    full = [Barrier() for _ in range(nF)]
    done = [Barrier() for _ in range(S)]
    afull = [Barrier() for _ in range(nAF)]
    aempty = [Barrier() for _ in range(nAE)]
    loaded, filled, mma_done = set(), set(), set()
    pending = []  # (time, kind, stage): TMA landings and MMA completions in flight
    wrong, violations = 0, 0
    nxt_load = 0
    nxt_fill = list(range(G))   # each group's next stage
    nxt_mma = list(range(I))    # each issuer's next stage
    t = 0

    def full_idx(it):
        return it % nF

    def aempty_idx(it):  # the barrier stage `it` waits on (committed by MMA(it - A))
        return it % nAE

    def aempty_phase(it):
        return (it - A) // nAE if single_consumer else (it - A) // A

    for _ in range(stages * 40):
        t += 1
        # completions land at random times
        for ev in [e for e in pending if e[0] <= t]:
            pending.remove(ev)
            _, kind, it = ev
            if kind == "load":
                loaded.add(it)
                full[full_idx(it)].done += 1
            else:
                mma_done.add(it)
                done[it % S].done += 1
                aempty[(it + A) % nAE].done += 1
        agent = rng.randrange(1 + G + I)
        if agent == 0:  # producer: smem stage free?
            it = nxt_load
            if it < stages and (it < S or done[it % S].passes((it - S) // S)):
                if it >= S and (it - S) not in mma_done:
                    wrong += 1
                pending.append((t + rng.randint(1, 30), "load", it))
                nxt_load += 1
        elif 1 <= agent <= G:  # dequant group
            g = agent - 1
            it = nxt_fill[g]
            if it >= stages:
                continue
            ph = it // nF
            if not full[full_idx(it)].passes(ph):
                continue
            if it not in loaded:
                wrong += 1
            if it >= A:
                if not aempty[aempty_idx(it)].passes(aempty_phase(it)):
                    continue
                if (it - A) not in mma_done:
                    wrong += 1
            if it not in loaded or (it >= A and (it - A) not in mma_done):
                violations += 1
            filled.add(it)
            afull[it % nAF].done += 1
            nxt_fill[g] += G
        else:  # MMA issuer
            i = agent - 1 - G
            it = nxt_mma[i]
            if it >= stages:
                continue
            if not afull[it % nAF].passes(it // nAF):
                continue
            if it not in filled:
                wrong += 1
                violations += 1
            pending.append((t + rng.randint(5, 60), "mma", it))
            nxt_mma[i] += I
    return wrong, violations, len(mma_done)


@pytest.mark.parametrize("S,A,G,I", [(6, 3, 4, 2), (3, 2, 4, 2), (2, 2, 4, 1), (6, 3, 2, 2),
                                     (3, 2, 2, 2), (6, 3, 1, 1)])
def test_single_consumer_barriers_never_pass_on_the_wrong_phase(S, A, G, I):
    for seed in range(40):
        wrong, violations, completed = simulate(S, A, G, I, True, 120, seed)
        assert wrong == 0 and violations == 0, (S, A, G, I, seed)
        assert completed == 120, (S, A, G, I, seed, completed)  # the pipeline drained


def test_shared_barriers_do_pass_on_the_wrong_phase():
    """Indexing by smem or A stage alone (several groups or issuers per barrier): the model
    finds waits that pass with the phase before still open -- the race the kernel had."""
    found = sum(simulate(3, 2, 4, 2, False, 120, seed)[0] for seed in range(40))
    assert found > 0
