"""A CPU model of the mbarrier protocol of the two-query-tile bf16 attention
kernel (``ptxgen/tmpl_attn2q.py``): the TMA warp, the one MMA-issuing warp
and two softmax warpgroups (one per 128-row query tile, four warps each) as
generators of waits, arrivals and commits, run under random schedules with
the hardware's ``try_wait.parity`` rule (a wait on parity P passes while the
barrier's current phase has the other parity).  The issuing thread's commits
complete in its issue order, TMA completions come in any order, and a
softmax warp's O-rescale wait on its tile's ``pv_done`` is taken at random,
as the kernel takes it only when a row's max moves.

Per key block g the MMA thread issues, for tiles A and B,
``S_X = Q_X K_g^T`` (into S_X, once ``pv_done_X`` says P_X of block g-1 --
written over S_X -- has been read) and ``O_X += P_X V_g`` (once the tile's
softmax has arrived on ``p_full_X``), in the order
QK_A(g), QK_B(g), PV_A(g), QK_A(g+1), PV_B(g), QK_B(g+1), ...

TMEM contents are tracked too: an MMA stays in flight until a later commit
of the issuing thread completes, in-flight MMAs may execute in any order,
and a conflicting access to S_X or O_X is a hazard.

Checked for the stage counts the kernel can use: no deadlock, no hazard, and
every wait passes on exactly the phase it means (no parity aliasing).
Dropping the ``pv_done`` wait before a QK is shown to break.  A separate
"O_X released" barrier is not needed: the tile's softmax warps are also its
epilogue warps, so their ``p_full_X`` arrivals for a unit's first block
come after they have read the previous unit's O_X -- the model runs
without one."""

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


def _roles(units, nkv, kvst, rng, o_empty=False, qk_waits_pv=True):
    W = lambda name, n: ("wait", name, n & 1, n)                  # noqa: E731
    Wi = lambda name, n: ("wait", name, (n & 1) ^ 1, n - 1)       # "empty" waits  # noqa: E731

    def prod():
        g = 0
        for u in range(units):
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
        # S_X = Q_X K_g^T: S_X is free once PV_X(g-1) has read P_X from it
        def qk(x, g, last_b):
            st = g % kvst
            yield W(f"k_full{st}", g // kvst)
            if g and qk_waits_pv:
                yield W(f"pv_done{x}", g - 1)
            # the state the MMA writes: S_X may not be read by a PV any more
            yield ("write", f"S{x}", g)
            yield ("commit", f"s_full{x}")
            if x == "B":
                yield ("commit", f"k_empty{st}")
                if last_b:
                    yield ("commit", "q_empty")

        def pv(x, g, first):
            st = g % kvst
            yield W(f"p_full{x}", g)
            yield W(f"v_full{st}", g // kvst)
            if first and o_empty:
                yield Wi(f"o_empty{x}", u_of[g])
            yield ("read", f"S{x}", g)       # P_X of block g, over S_X
            yield ("write", f"O{x}", u_of[g])  # O_X of this unit
            yield ("commit", f"pv_done{x}")
            if x == "B":
                yield ("commit", f"v_empty{st}")

        g = 0
        for u in range(units):
            yield W("q_full", u)
            yield from qk("A", g, False)
            yield from qk("B", g, nkv == 1)
            for j in range(nkv):
                last = j + 1 == nkv
                yield from pv("A", g, j == 0)
                if not last:
                    yield from qk("A", g + 1, False)
                yield from pv("B", g, j == 0)
                if not last:
                    yield from qk("B", g + 1, j + 2 == nkv)
                g += 1

    def softmax(x):                        # one warp of four; 32 arrivals each
        g = 0
        for u in range(units):
            for j in range(nkv):
                yield W(f"s_full{x}", g)
                yield ("read", f"S{x}", g)       # the scores of block g
                if j and rng.random() < 0.3:
                    yield W(f"pv_done{x}", g - 1)
                    yield ("read", f"O{x}", u)   # the rescale of O_X, in place
                    yield ("write", f"O{x}", u)
                yield ("arrive", f"p_full{x}", 32)
                g += 1
            yield W(f"pv_done{x}", g - 1)        # the unit's last P_X V done
            yield ("read", f"O{x}", u)           # the epilogue
            yield ("arrive", f"o_empty{x}", 32)

    u_of = [u for u in range(units) for _ in range(nkv)]
    return {"prod": prod(), "mma": mma(),
            **{f"sm{x}{i}": softmax(x) for x in "AB" for i in range(4)}}


def run(units, nkv, kvst, seed, roles=None, ordered_writes=False, **kw):
    """Random schedule; "ok", "deadlock" or the first hazard found.

    An MMA is in flight from its issue until a later commit of the issuing
    thread completes (a commit arrives once every earlier MMA of the thread
    is done); in-flight MMAs may execute in any order, so two in flight that
    touch the same TMEM region, one of them writing, are a hazard, and so is
    a softmax or epilogue access to a region an in-flight MMA writes.
    ``ordered_writes``: two in-flight MMAs that both accumulate into one
    region are not a hazard (the tensor core applies one thread's MMAs to an
    accumulator in issue order -- the way every K loop accumulates)."""
    rng = random.Random(seed)
    bars = {}

    def bar(name):
        if name not in bars:
            bars[name] = Bar(128 if name.startswith(("p_full", "o_empty", "s_free", "tok")) else 1)
        return bars[name]

    gens = (roles or _roles)(units, nkv, kvst, rng, **kw)
    cur = {r: next(g) for r, g in gens.items()}
    tma = []
    commits = []          # (issuer, barrier, number of its MMAs issued before it)
    flight = []           # (issuer, issue number, kind, region, value)
    issued: dict = {}     # MMAs issued so far, per issuing role ("mma...")
    state: dict = {}              # TMEM region -> the value last written
    while cur or tma or commits:
        ready = [r for r, op in cur.items()
                 if op[0] != "wait" or bar(op[1]).passes(op[2])]
        choices = ready + (["TMA"] if tma else []) + (["COMMIT"] if commits else [])
        if not choices:
            return "deadlock"
        c = rng.choice(choices)
        if c == "TMA":
            bar(tma.pop(rng.randrange(len(tma)))).arrive(1)
            continue
        if c == "COMMIT":
            # one issuer's commits complete in its order; issuers are independent
            who = rng.choice(sorted({cm[0] for cm in commits}))
            i = next(n for n, cm in enumerate(commits) if cm[0] == who)
            _, name, upto = commits.pop(i)
            for f in [f for f in flight if f[0] == who and f[1] < upto]:
                if f[2] == "write":
                    state[f[3]] = f[4]
                flight.remove(f)
            bar(name).arrive(1)
            continue
        op = cur[c]
        if op[0] == "wait":
            b, meant = bar(op[1]), op[3]
            if meant >= 0 and b.phase != meant + 1:
                return f"alias: {c} waited {op[1]} phase {meant}, barrier at {b.phase}"
        elif op[0] == "tma":
            tma.append(op[1])
        elif op[0] == "commit":
            commits.append((c, op[1], issued.get(c, 0)))
        elif op[0] in ("read", "write") and c.startswith("mma"):
            for f in flight:
                if ordered_writes and f[0] == c and f[2] == op[0] == "write":
                    continue
                if f[3] == op[1] and "write" in (f[2], op[0]):
                    return f"hazard: MMA {op[0]} of {op[1]} while an MMA {f[2]} is in flight"
            if op[0] == "read" and op[1].startswith("S") and state.get(op[1]) != op[2]:
                if not any(f[2] == "write" and f[3] == op[1] for f in flight):
                    return f"hazard: P.V read {op[1]} for block {op[2]}, it holds {state.get(op[1])}"
            flight.append((c, issued.get(c, 0), op[0], op[1], op[2]))
            issued[c] = issued.get(c, 0) + 1
        elif op[0] in ("read", "write"):
            if any(f[3] == op[1] for f in flight if f[2] == "write" or op[0] == "write"):
                return f"hazard: {c} {op[0]} of {op[1]} while an MMA touches it"
            if op[0] == "read" and state.get(op[1]) != op[2]:
                return f"hazard: {c} read {op[1]} wanting {op[2]}, it holds {state.get(op[1])}"
            if op[0] == "write":
                state[op[1]] = op[2]
        else:
            bar(op[1]).arrive(op[2])
        try:
            cur[c] = next(gens[c])
        except StopIteration:
            del cur[c]
    return "ok"


SHAPES = [(1, 1), (1, 2), (2, 1), (3, 3), (2, 5), (4, 4), (3, 7)]


@pytest.mark.parametrize("kvst", [1, 2])
def test_two_tile_protocol_has_no_deadlock_or_aliasing(kvst):
    for units, nkv in SHAPES:
        for seed in range(200):
            r = run(units, nkv, kvst, seed)
            assert r == "ok", (units, nkv, seed, r)


def test_model_finds_a_missing_pv_wait():
    """Without the pv_done wait before S_X = Q_X K^T, the next block's scores
    could overwrite P_X before P_X V has read it."""
    found = any(run(u, n, 2, seed, qk_waits_pv=False) != "ok"
                for u, n in SHAPES for seed in range(200))
    assert found


def test_o_empty_barrier_would_add_nothing():
    """With an explicit O_X-released barrier the protocol is no safer: it was
    already hazard-free without it."""
    for units, nkv in SHAPES:
        for seed in range(100):
            assert run(units, nkv, 2, seed, o_empty=True) == "ok"
