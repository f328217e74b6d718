"""The peer-memory exchange's slot protocol (dotllm_b200/csrc/tp.cu), modelled on the CPU.

Every rank owns receive slots [parity][source rank][element].  Exchange number g (the sequence
number + 1) stores each element of a rank's contribution as a word tagged g into every peer's
slot [g % parities][own rank][element], then waits on its own slots for the other ranks' words
tagged g.  A rank's next exchange starts only after its current one finished (stream order,
one kernel per exchange).  The model runs the ranks under random interleavings, one word store
or one slot read per step, and checks the two properties the kernels rely on:

* no store overwrites a word that its reader has not yet taken;
* every word a rank takes carries the value its writer sent in the same exchange.

Exchanges differ in length (the residual sums are batch x hidden floats, the argmax max-reduce
two words per key), as in the step.  With two parities both properties hold for any schedule;
the planted variant with one parity breaks them, which shows the checks can fail.
"""
import random

import pytest


class Violation(Exception):
    pass


def _simulate(tp, lengths, parities, seed):
    rng = random.Random(seed)
    # slot[(owner, parity, src, e)] = (gen, value, taken)
    slot = {}
    # per rank: exchange index, phase ("push" or "wait"), and the queue of word operations left
    state = []
    for r in range(tp):
        state.append({"x": 0, "ops": None})

    def value(src, g, e):
        return (src * 1_000_003 + g * 10_007 + e) % 999_983

    def start(r):
        st = state[r]
        if st["x"] >= len(lengths):
            st["ops"] = None
            return
        g = st["x"] + 1
        n = lengths[st["x"]]
        pushes = [("push", q, e) for e in range(n) for q in range(tp) if q != r]
        waits = [("wait", q, e) for e in range(n) for q in range(tp) if q != r]
        # the kernel's threads run concurrently: pushes in any order, then waits in any order
        rng.shuffle(pushes)
        rng.shuffle(waits)
        st["ops"] = pushes + waits
        st["g"] = g

    for r in range(tp):
        start(r)
    steps = 0
    while True:
        live = [r for r in range(tp) if state[r]["ops"] is not None]
        if not live:
            return steps
        # ranks whose next operation can run now (a wait blocks until its word arrived)
        ready = []
        for r in live:
            st = state[r]
            if not st["ops"]:
                ready.append(r)
                continue
            kind, q, e = st["ops"][0]
            if kind == "push":
                ready.append(r)
            else:
                word = slot.get((r, st["g"] % parities, q, e))
                if word is not None and word[0] == st["g"]:
                    ready.append(r)
        if not ready:
            raise Violation("deadlock: every live rank waits")
        r = rng.choice(ready)
        st = state[r]
        steps += 1
        if not st["ops"]:  # exchange finished: the next kernel starts
            st["x"] += 1
            start(r)
            continue
        kind, q, e = st["ops"].pop(0)
        g = st["g"]
        if kind == "push":
            key = (q, g % parities, r, e)
            old = slot.get(key)
            if old is not None and not old[2]:
                raise Violation(f"rank {r} exchange {g} overwrote an untaken word of exchange {old[0]} at {key}")
            slot[key] = (g, value(r, g, e), False)
        else:
            key = (r, g % parities, q, e)
            gen, v, _ = slot[key]
            if v != value(q, g, e):
                raise Violation(f"rank {r} exchange {g} took a wrong value at {key}")
            slot[key] = (gen, v, True)


LENGTHS = [8, 8, 2, 8, 8, 2, 5, 1, 8, 3, 8, 8, 2]  # sums of several sizes and argmax key pairs


@pytest.mark.parametrize("tp", [2, 3, 4, 8])
def test_two_parities_hold_under_random_schedules(tp):
    for seed in range(40 if tp < 8 else 10):
        _simulate(tp, LENGTHS, parities=2, seed=seed)


def test_one_parity_breaks():
    """Planted mistake in the model: with one receive buffer a fast rank's next exchange
    overwrites words a slow peer has not taken yet, under some schedule."""
    broke = 0
    for seed in range(40):
        try:
            _simulate(2, LENGTHS, parities=1, seed=seed)
        except Violation:
            broke += 1
    assert broke > 0
