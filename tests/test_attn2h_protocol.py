"""A CPU model of the barrier protocol of the two-tile bf16 attention on
64-key blocks (``ptxgen/tmpl_attn2h.py``), run with the random scheduler,
TMA and commit rules of ``tests/test_attn2q_protocol.py``.

Each query tile X keeps two S buffers in TMEM (S_X0, S_X1): block g uses
buffer g % 2, so S_X = Q_X K_{g+2}^T can be issued as soon as P_X V_g has
read buffer g % 2, while the softmax still works on block g + 1.  Per
block g the MMA thread issues PV_A(g), PV_B(g), then QK_A(g+2), QK_B(g+2);
a unit starts with QK_A, QK_B of its first two blocks.  Barriers per tile
and buffer: s_full, p_full (128 arrivals), pv_done; per K/V stage full and
empty; per unit q_full / q_empty.  Checked: no deadlock, no TMEM hazard and
no wait that could pass on the wrong phase, for 2 to 4 stages; and that
dropping the pv_done wait before a QK is caught.  P V of consecutive blocks
may both be in flight on O_X: one thread's MMAs accumulate in issue
order."""

import pytest

from tests.test_attn2q_protocol import run


def _roles(units, nkv, kvst, rng, qk_waits_pv=True, split=False, p_smem=False,
           pingpong=False, tok_wait=True):
    W = lambda name, n: ("wait", name, n & 1, n)                  # noqa: E731
    Wi = lambda name, n: ("wait", name, (n & 1) ^ 1, n - 1)       # noqa: E731

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
        def qk(x, g, last_b):
            st, h = g % kvst, g % 2
            yield W(f"k_full{st}", g // kvst)
            if g >= 2 and qk_waits_pv:
                if p_smem:      # S of block g - 2 read by the softmax
                    yield W(f"s_free{x}{h}", (g - 2) >> 1)
                else:           # P of block g - 2 (over S) read by P V
                    yield W(f"pv_done{x}{h}", (g - 2) >> 1)
            yield ("write", f"S{x}{h}", g)
            yield ("commit", f"s_full{x}{h}")
            if x == "B":
                yield ("commit", f"k_empty{st}")
                if last_b:
                    yield ("commit", "q_empty")

        def pv(x, g, u):
            st, h = g % kvst, g % 2
            yield W(f"p_full{x}{h}", g >> 1)
            yield W(f"v_full{st}", g // kvst)
            yield ("read", f"P{x}{h}" if p_smem else f"S{x}{h}", g)
            yield ("write", f"O{x}", u)
            yield ("commit", f"pv_done{x}{h}")
            if x == "B":
                yield ("commit", f"v_empty{st}")

        def one_thread():
            g0 = 0
            for u in range(units):
                yield W("q_full", u)
                for j in range(min(2, nkv)):
                    yield from qk("A", g0 + j, False)
                    yield from qk("B", g0 + j, j == nkv - 1)
                for j in range(nkv):
                    g = g0 + j
                    yield from pv("A", g, u)
                    yield from pv("B", g, u)
                    if j + 2 < nkv:
                        yield from qk("A", g + 2, False)
                        yield from qk("B", g + 2, j + 2 == nkv - 1)
                g0 += nkv

        def qk_thread():
            g = 0
            for u in range(units):
                yield W("q_full", u)
                for j in range(nkv):
                    yield from qk("A", g, False)
                    yield from qk("B", g, j == nkv - 1)
                    g += 1

        def pv_thread():
            g = 0
            for u in range(units):
                for _ in range(nkv):
                    yield from pv("A", g, u)
                    yield from pv("B", g, u)
                    g += 1

        return (qk_thread(), pv_thread()) if split else (one_thread(),)

    def softmax(x):                        # one warp of four; 32 arrivals each
        g = 0
        for u in range(units):
            for j in range(nkv):
                h = g % 2
                yield W(f"s_full{x}{h}", g >> 1)
                yield ("read", f"S{x}{h}", g)
                if p_smem:
                    yield ("arrive", f"s_free{x}{h}", 32)
                if j and rng.random() < 0.3:
                    yield W(f"pv_done{x}{(g - 1) % 2}", (g - 1) >> 1)
                    yield ("read", f"O{x}", u)
                    yield ("write", f"O{x}", u)
                if pingpong:
                    # the exp2 loops take turns: A(g) after B(g - 1), B(g)
                    # after A(g); "MUFU" holds whose loop runs, and a loop
                    # that finds another tile's mark at its end overlapped it
                    if tok_wait:
                        if x == "B":
                            yield W("tokA", g)
                        elif g:
                            yield W("tokB", g - 1)
                    yield ("write", "MUFU", (x, g))
                if p_smem:
                    # the P buffer of block g - 2 must have been read by its P V
                    if g >= 2:
                        yield W(f"pv_done{x}{h}", (g - 2) >> 1)
                    yield ("write", f"P{x}{h}", g)
                else:
                    yield ("write", f"S{x}{h}", g)  # P of block g over its scores
                if pingpong:
                    yield ("read", "MUFU", (x, g))
                    yield ("arrive", f"tok{x}", 32)
                yield ("arrive", f"p_full{x}{h}", 32)
                g += 1
            yield W(f"pv_done{x}{(g - 1) % 2}", (g - 1) >> 1)
            yield ("read", f"O{x}", u)           # the epilogue

    issuers = mma()
    return {"prod": prod(), **{f"mma{i}": t for i, t in enumerate(issuers)},
            **{f"sm{x}{i}": softmax(x) for x in "AB" for i in range(4)}}


SHAPES = [(1, 1), (1, 2), (2, 1), (1, 3), (3, 3), (2, 5), (4, 4), (3, 8)]


@pytest.mark.parametrize("form", ["one issuer", "two issuers", "P in shared memory",
                                  "exp2 loops in turn"])
@pytest.mark.parametrize("kvst", [2, 3, 4])
def test_half_block_protocol_has_no_deadlock_or_aliasing(kvst, form):
    """One issuing thread; S = Q K^T and O += P V issued by two threads
    (each thread's commits cover only its own MMAs); and the same with P in
    shared memory, where an S buffer is free once the softmax has read it
    (``s_free``) and the softmax waits for the P V two blocks back before
    overwriting that block's P buffer; and the two-issuer form with the two
    tiles' exp2 loops taking turns (``tok`` barriers).  The kernel ships the
    two-issuer form; the other two are measured alternatives (correct and
    slower) kept modelled so a future variant starts from a checked
    protocol."""
    kw = {"one issuer": {}, "two issuers": {"split": True},
          "P in shared memory": {"split": True, "p_smem": True},
          "exp2 loops in turn": {"split": True, "pingpong": True}}[form]
    for units, nkv in SHAPES:
        for seed in range(150):
            r = run(units, nkv, kvst, seed, roles=_roles, ordered_writes=True, **kw)
            assert r == "ok", (units, nkv, seed, r)


def test_model_finds_a_missing_pv_wait():
    """Without the wait for P V of block g - 2, S = Q K^T of block g could
    overwrite P of block g - 2 before it is read."""
    for split in (False, True):
        found = any(run(u, n, 4, seed, roles=_roles, ordered_writes=True,
                        qk_waits_pv=False, split=split) != "ok"
                    for u, n in SHAPES for seed in range(150))
        assert found
    # with P in shared memory: S of block g overwritten before the softmax
    # has read it, once QK stops waiting for s_free
    found = any(run(u, n, 4, seed, roles=_roles, ordered_writes=True, qk_waits_pv=False,
                    split=True, p_smem=True) != "ok"
                for u, n in SHAPES for seed in range(150))
    assert found


def test_model_finds_overlapping_exp2_loops():
    """Without the token waits the two tiles' exp2 loops overlap."""
    found = any(run(u, n, 4, seed, roles=_roles, ordered_writes=True, split=True,
                    pingpong=True, tok_wait=False) != "ok"
                for u, n in SHAPES for seed in range(50))
    assert found
