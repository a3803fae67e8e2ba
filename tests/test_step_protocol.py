"""The tagged-vector protocol of the persistent decode step (step.cu),
restated on the host and run under random interleavings of its CTAs (CPU
only).

Per layer the stages are QKV (reads HIDDEN, writes QKV), attention (only the
attention CTAs: read QKV, write ATTN), O (reads ATTN, writes HIDDEN), gate/up
(reads HIDDEN, writes ACT) and down (reads ACT, writes HIDDEN); after the
last layer the LM head reads HIDDEN and every CTA counts its arrival, CTA 0
then publishes TOKEN, which the next step's first QKV stage reads instead of
HIDDEN (the embedding row of that token).  A GEMV stage's CTAs each write a
slice of the output vector as tagged words of the next version; a reader
waits word by word until a word carries the version it expects.  The CTAs
that run no attention pass straight on to the O stage.

The kernel has no grid barrier, so it relies on one property: no CTA ever
overwrites a word that another CTA has yet to read at its old version (a
reader would then wait for a version that never comes).  The model checks it
at every write, and checks that every interleaving finishes (no deadlock)
with every read seeing exactly the version it expected.
"""
import random

import pytest

BUFS = ("HIDDEN", "QKV", "ATTN", "ACT", "TOKEN")


def stage_list(n_layers):
    """(kind, input buffer, output buffer) per stage of one step."""
    st = []
    for layer in range(n_layers):
        st.append(("gemv", "TOKEN" if layer == 0 else "HIDDEN", "QKV"))
        st.append(("attn", "QKV", "ATTN"))
        st.append(("gemv", "ATTN", "HIDDEN"))
        st.append(("gemv", "HIDDEN", "ACT"))
        st.append(("gemv", "ACT", "HIDDEN"))
    st.append(("lm", "HIDDEN", None))
    return st


def programs(n_cta, attn_ctas, n_layers, n_steps):
    """Each CTA's action list: ("read", buf, writer, version) for every slice
    it needs, then ("write", buf, version) of its own slice; the LM head's
    arrival and CTA 0's token publish close each step."""
    ver = {b: 0 for b in BUFS}
    prog = [[] for _ in range(n_cta)]
    for _ in range(n_steps):
        for kind, src, dst in stage_list(n_layers):
            if src == "TOKEN":
                writers = [0]
            elif src == "ATTN":
                writers = attn_ctas
            else:
                writers = list(range(n_cta))
            if kind == "lm":
                for c in range(n_cta):
                    prog[c] += [("read", src, w, ver[src]) for w in writers]
                    prog[c].append(("arrive",))
                prog[0].append(("collect", n_cta))
                ver["TOKEN"] += 1
                prog[0].append(("write", "TOKEN", ver["TOKEN"]))
                continue
            out_writers = attn_ctas if kind == "attn" else list(range(n_cta))
            ver[dst] += 1
            for c in out_writers:
                prog[c] += [("read", src, w, ver[src]) for w in writers]
                prog[c].append(("write", dst, ver[dst]))
    return prog


def run(n_cta, attn_ctas, n_layers, n_steps, seed, prog=None):
    rng = random.Random(seed)
    prog = prog or programs(n_cta, attn_ctas, n_layers, n_steps)
    # words[buf][writer] = the version of writer's slice of buf; the token
    # starts at version 0 (the prompt's token is in place before the launch)
    words = {b: [0] * n_cta for b in BUFS}
    arrivals = 0
    pc = [0] * n_cta

    def blocked(c):
        if pc[c] >= len(prog[c]):
            return True
        a = prog[c][pc[c]]
        if a[0] == "read":
            _, buf, w, v = a
            assert words[buf][w] <= v, f"CTA {c} wanted {buf}[{w}] v{v}, found v{words[buf][w]} (overwritten)"
            return words[buf][w] < v
        if a[0] == "collect":
            return arrivals < a[1]
        return False

    while True:
        ready = [c for c in range(n_cta) if not blocked(c)]
        if not ready:
            return all(pc[c] >= len(prog[c]) for c in range(n_cta))
        c = rng.choice(ready)
        a = prog[c][pc[c]]
        if a[0] == "write":
            _, buf, v = a
            # the property: nobody still needs the old version of this word
            for o in range(n_cta):
                if pc[o] < len(prog[o]):
                    for b in prog[o][pc[o]:]:
                        if b[0] == "read" and b[1] == buf and b[2] == c:
                            assert b[3] >= v, (f"CTA {c} writes {buf} v{v} while CTA {o} "
                                               f"still has to read v{b[3]}")
                            break
            words[buf][c] = v
        elif a[0] == "arrive":
            arrivals += 1
        elif a[0] == "collect":
            arrivals = 0
        pc[c] += 1


@pytest.mark.parametrize("n_cta,attn", [(2, [0]), (4, [1, 2]), (6, [0, 1, 2, 3, 4, 5]), (5, [4])])
def test_step_protocol_finishes_and_never_overwrites_unread_words(n_cta, attn):
    for seed in range(150):
        assert run(n_cta, attn, n_layers=3, n_steps=3, seed=seed), (n_cta, attn, seed)


def test_model_detects_an_unsafe_schedule():
    """The checker itself: a CTA that wrote its O-stage output without
    waiting for the attention output (dropping its reads of ATTN) can
    overwrite HIDDEN while slower CTAs still read the old version; some
    interleaving shows it."""
    n_cta, attn = 3, [1]
    prog = programs(n_cta, attn, 2, 1)
    prog[0] = [a for a in prog[0] if not (a[0] == "read" and a[1] == "ATTN")]
    found = 0
    for seed in range(200):
        try:
            run(n_cta, attn, 2, 1, seed, prog=[list(x) for x in prog])
        except AssertionError as e:
            assert "HIDDEN" in str(e), e
            found += 1
    assert found > 0
