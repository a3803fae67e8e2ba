"""The expert-parallel exchange protocol of moe.cu, restated on the host and
run under many interleavings of the ranks (CPU only).

Per MoE invocation v (v = 1, 2, ...), rank r:
  publish: writes its arrival word (tag v) into every rank's buffer, then its
           selected experts' slot rows, tagged v, into half v & 1 of every
           rank's buffer;
  combine: waits until every arrival word in its own buffer reads at least v,
           then until each slot it needs in half v & 1 carries tag v, and
           reads it;
  advance: v += 1.
A rank's next publish follows its combine (stream order).  The protocol must
never deadlock however the ranks interleave, and no slot a rank still has to
read may be overwritten by invocation v + 2 first.  A combine that waits for
arrival words to read exactly v (instead of at least v) deadlocks as soon as a
faster rank has published v + 1; the second case shows it.
"""
import random

import pytest


def run(n_ranks, n_inv, owners, seed, exact_arrival=False):
    """Interleave n_ranks ranks over n_inv invocations; owners[v] = the rank
    that runs the (single) routed expert of invocation v.  Returns the
    slot values each rank combined, or None on a deadlock."""
    rng = random.Random(seed)
    arrive = [[0] * n_ranks for _ in range(n_ranks)]   # arrive[buffer][rank]
    slots = [[0, 0] for _ in range(n_ranks)]           # slots[buffer][half] = tag
    state = [("publish", 1) for _ in range(n_ranks)]
    read = [[] for _ in range(n_ranks)]

    def can_step(r):
        phase, v = state[r]
        if phase == "done":
            return False
        if phase == "publish":
            return True
        ok = (lambda a: a == v) if exact_arrival else (lambda a: a >= v)
        return all(ok(a) for a in arrive[r]) and slots[r][v & 1] == v

    while True:
        ready = [r for r in range(n_ranks) if can_step(r)]
        if not ready:
            return read if all(s[0] == "done" for s in state) else None
        r = rng.choice(ready)
        phase, v = state[r]
        if phase == "publish":
            for b in range(n_ranks):
                arrive[b][r] = v
            if owners[v] == r:
                for b in range(n_ranks):
                    # a hazard: overwriting a slot of invocation v - 2 that a
                    # rank has not combined yet
                    assert not (slots[b][v & 1] == v - 2 and state[b] == ("combine", v - 2)), (b, v)
                    slots[b][v & 1] = v
            state[r] = ("combine", v)
        else:
            read[r].append(slots[r][v & 1])
            state[r] = ("publish", v + 1) if v < n_inv else ("done", v)


@pytest.mark.parametrize("n_ranks", [2, 3, 4, 8])
def test_protocol_never_deadlocks_and_reads_its_own_invocation(n_ranks):
    n_inv = 24
    for seed in range(200):
        rng = random.Random(seed)
        # seed-dependent routing, including long runs on one rank
        owners = [0] + [0 if seed % 3 == 0 else rng.randrange(n_ranks) for _ in range(n_inv)]
        read = run(n_ranks, n_inv, owners, seed)
        assert read is not None, (n_ranks, seed)
        for r in range(n_ranks):
            assert read[r] == list(range(1, n_inv + 1)), (r, read[r])


def test_exact_arrival_match_deadlocks():
    """The arrival test must be 'at least v': with 'exactly v' a rank that
    has published v + 1 blocks the others' combine of v."""
    deadlocked = sum(run(2, 12, [0] * 13, seed, exact_arrival=True) is None for seed in range(100))
    assert deadlocked > 0
