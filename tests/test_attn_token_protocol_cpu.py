"""The turn-taking protocol of attention variant 4 (flash_fwd3_kernel<true>, attn3.cuh), checked
on a model: two softmax warps of one SM sub-partition (tile 0 with n0 key blocks, tile 1 with
n1), each with a token mbarrier (one arrival per phase) and a done flag. The model keeps the
hardware's parity rule (try_wait.parity(P) succeeds once the barrier's current phase parity
differs from P) and runs the warps' steps in random orders. It checks that the exponential
phases of the two warps never overlap, that they alternate tile 0, tile 1, tile 0, ... while
both warps have blocks left, and that both warps always finish (no wait is left without an
arrival or a done flag to end it)."""
import random

import pytest


class Barrier:
    def __init__(self):
        self.completed = 0  # phases completed (one arrival completes a phase)

    def arrive(self):
        self.completed += 1

    def try_wait(self, parity: int) -> bool:
        return (self.completed & 1) != parity


def run(n0: int, n1: int, rng: random.Random):
    token = [Barrier(), Barrier()]
    done = [False, False]
    n = [n0, n1]
    # per warp: program counter over the steps of block j
    state = [{"j": 0, "step": "top"} for _ in range(2)]
    in_exp = [False, False]
    order = []
    steps = 0
    while not (state[0]["step"] == "end" and state[1]["step"] == "end"):
        steps += 1
        assert steps < 10000, "no progress: a wait never ends"
        ready = []
        for t in range(2):
            st = state[t]
            if st["step"] == "end":
                continue
            if st["step"] == "wait":
                j = st["j"]
                parity = ((j - 1) if t == 0 else j) & 1
                if not (token[t].try_wait(parity) or done[1 - t]):
                    continue  # blocked this round
            ready.append(t)
        assert ready, "deadlock"
        t = rng.choice(ready)
        st = state[t]
        if st["step"] == "top":
            if st["j"] >= n[t]:
                st["step"] = "finish"
            else:
                first = t == 0 and st["j"] == 0
                st["step"] = "exp" if first else "wait"
        elif st["step"] == "wait":
            st["step"] = "exp"
        elif st["step"] == "exp":
            assert not in_exp[1 - t], "both warps in their exponentials at once"
            in_exp[t] = True
            order.append((t, st["j"]))
            st["step"] = "exp_end"
        elif st["step"] == "exp_end":
            in_exp[t] = False
            token[1 - t].arrive()  # the partner's turn
            st["j"] += 1
            st["step"] = "top"
        elif st["step"] == "finish":
            done[t] = True
            st["step"] = "end"
    return order


@pytest.mark.parametrize("n0,n1", [(1, 1), (1, 3), (2, 4), (5, 7), (4, 4), (9, 9), (3, 0), (1, 0), (6, 8)])
def test_turns_alternate_and_both_warps_finish(n0, n1):
    for seed in range(200):
        order = run(n0, n1, random.Random(seed))
        assert sorted(o for o in order if o[0] == 0) == [(0, j) for j in range(n0)]
        assert sorted(o for o in order if o[0] == 1) == [(1, j) for j in range(n1)]
        # while both warps have blocks left the turns go 0, 1, 0, 1, ... block by block
        both = min(n0, n1)
        assert order[:2 * both] == [(t, j) for j in range(both) for t in (0, 1)]
        # the rest belongs to the warp with more blocks, in block order
        rest = order[2 * both:]
        assert rest == sorted(rest)
