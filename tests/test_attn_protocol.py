"""A CPU model of the attention kernel's mbarrier protocol
(``ptxgen/tmpl_attn.py`` ``_emit_tc``): the TMA warp, the two MMA-issuing
warps (S = Q.K^T and O += P.V^T) and the softmax warps as generators of
waits, arrivals and commits, run under random schedules with the hardware's
``try_wait.parity`` rule (a wait on parity P passes while the barrier's
current phase has the other parity).  Each issuing warp's commits complete in
its own issue order, the two warps' interleave arbitrarily, TMA completions
come in any order, and the softmax's O-rescale wait on ``pv_done`` is taken
at random, as it is taken only when a row's max moves.

Checked for every stage count and Q placement the template uses: no
deadlock, and every wait passes on exactly the phase it means -- never on a
stale phase two behind (parity aliasing).  The same model with a single
``p_full`` barrier, or with the epilogue waiting ``pv_done`` instead of the
per-unit ``o_full``, finds the hazards those versions had."""

import random

import pytest


class Bar:
    def __init__(self, count):
        self.count = self.pending = count
        self.phase = 0                    # completed phases

    def arrive(self, w):
        self.pending -= w
        assert self.pending >= 0
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count

    def passes(self, parity):
        return (self.phase & 1) != parity


def _roles(units, nkv, kvst, q_tmem, rng, per_buffer_p=True, o_full=True, issuers=2):
    W = lambda name, n: ("wait", name, n & 1, n)                  # noqa: E731
    Wi = lambda name, n: ("wait", name, (n & 1) ^ 1, n - 1)       # "empty" waits  # noqa: E731

    def pfull(g):
        return (f"p_full{g & 1}", g >> 1) if per_buffer_p else ("p_full", g)

    def prod():
        g = 0
        for u in range(units):
            if not q_tmem:
                yield Wi("q_empty", u)
                yield ("tma", "q_full")
            for _ in range(nkv):
                st, n = g % kvst, g // kvst
                yield Wi(f"k_empty{st}", n)
                yield ("tma", f"k_full{st}")
                yield Wi(f"v_empty{st}", n)
                yield ("tma", f"v_full{st}")
                g += 1

    def mma():
        def qk(g):
            st = g % kvst
            yield W(f"k_full{st}", g // kvst)
            yield Wi(f"s_free{g & 1}", g >> 1)
            yield ("commit", f"s_full{g & 1}")
            yield ("commit", f"k_empty{st}")

        def pv(g):
            st = g % kvst
            name, n = pfull(g)
            yield W(name, n)
            yield W(f"v_full{st}", g // kvst)
            yield ("commit", "pv_done")
            yield ("commit", f"v_empty{st}")
            yield ("commit", f"s_free{g & 1}")

        g = 0
        for u in range(units):
            yield W("q_full", u)
            yield from qk(g)
            for j in range(nkv):
                last = j + 1 == nkv
                if kvst > 1:
                    if not last:
                        yield from qk(g + 1)
                    yield from pv(g)
                else:
                    yield from pv(g)
                    if not last:
                        yield from qk(g + 1)
                g += 1
            if o_full:
                yield ("commit", "o_full")
            if not q_tmem:
                yield ("commit", "q_empty")

    def qk_warp():                         # the two-issuer form: S = Q.K^T ...
        g = 0
        for u in range(units):
            yield W("q_full", u)
            for _ in range(nkv):
                yield from qk(g)
                g += 1
            if not q_tmem:
                yield ("commit", "q_empty")

    def pv_warp():                         # ... and O += P.V^T from another warp
        g = 0
        for u in range(units):
            for _ in range(nkv):
                yield from pv(g)
                g += 1
            yield ("commit", "o_full")

    def qk(g):
        st = g % kvst
        yield W(f"k_full{st}", g // kvst)
        yield Wi(f"s_free{g & 1}", g >> 1)
        yield ("commit", f"s_full{g & 1}")
        yield ("commit", f"k_empty{st}")

    def pv(g):
        st = g % kvst
        name, n = pfull(g)
        yield W(name, n)
        yield W(f"v_full{st}", g // kvst)
        yield ("commit", "pv_done")
        yield ("commit", f"v_empty{st}")
        yield ("commit", f"s_free{g & 1}")

    def softmax():                         # one warp of four; 32 arrivals each
        g = 0
        for u in range(units):
            if q_tmem:
                yield ("arrive", "q_full", 32)
            for j in range(nkv):
                yield W(f"s_full{g & 1}", g >> 1)
                if j and rng.random() < 0.3:
                    yield W("pv_done", g - 1)
                yield ("arrive", pfull(g)[0], 32)
                g += 1
            yield W("o_full", u) if o_full else W("pv_done", g - 1)

    issue = ({"mma": mma()} if issuers == 1 else {"mma_qk": qk_warp(), "mma_pv": pv_warp()})
    return {"prod": prod(), **issue, **{f"sm{i}": softmax() for i in range(4)}}


def run(units, nkv, kvst, q_tmem, seed, **kw):
    rng = random.Random(seed)
    bars = {}

    def bar(name):
        if name not in bars:
            if name.startswith("p_full") or (name == "q_full" and q_tmem):
                bars[name] = Bar(128)
            else:
                bars[name] = Bar(1)
        return bars[name]

    gens = _roles(units, nkv, kvst, q_tmem, rng, **kw)
    cur = {r: next(g) for r, g in gens.items()}
    tma = []
    commits = {r: [] for r in gens if r.startswith("mma")}   # in order per issuing thread
    while cur or tma or any(commits.values()):
        ready = [r for r, op in cur.items()
                 if op[0] != "wait" or bar(op[1]).passes(op[2])]
        choices = (ready + (["TMA"] if tma else [])
                   + [("COMMIT", r) for r, q in commits.items() if q])
        if not choices:
            return "deadlock"
        c = rng.choice(choices)
        if c == "TMA":
            bar(tma.pop(rng.randrange(len(tma)))).arrive(1)
            continue
        if isinstance(c, tuple):
            bar(commits[c[1]].pop(0)).arrive(1)
            continue
        op = cur[c]
        if op[0] == "wait":
            b, meant = bar(op[1]), op[3]
            if meant >= 0 and b.phase != meant + 1:
                return f"alias: {c} waited {op[1]} phase {meant}, barrier at {b.phase}"
        elif op[0] == "tma":
            tma.append(op[1])
        elif op[0] == "commit":
            commits[c].append(op[1])
        else:
            bar(op[1]).arrive(op[2])
        try:
            cur[c] = next(gens[c])
        except StopIteration:
            del cur[c]
    return "ok"


SHAPES = [(1, 1), (1, 2), (2, 1), (3, 3), (2, 5), (4, 4), (3, 7)]


@pytest.mark.parametrize("issuers", [2, 1])
@pytest.mark.parametrize("q_tmem", [False, True])
@pytest.mark.parametrize("kvst", [1, 2, 3])
def test_protocol_has_no_deadlock_or_aliasing(kvst, q_tmem, issuers):
    """``issuers=2`` is the kernel (QK and PV from two warps, each warp's
    commits in its own order); ``issuers=1`` the earlier single-warp form."""
    for units, nkv in SHAPES:
        for seed in range(150):
            r = run(units, nkv, kvst, q_tmem, seed, issuers=issuers)
            assert r == "ok", (units, nkv, seed, r)


@pytest.mark.parametrize("variant", [{"per_buffer_p": False}, {"o_full": False}])
def test_model_finds_the_old_hazards(variant):
    found = any(run(u, n, 2, False, seed, issuers=1, **variant) != "ok"
                for u, n in SHAPES for seed in range(150))
    assert found
