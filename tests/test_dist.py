"""Multi-process host logic on CPU (gloo, world size 2): sharding, the
global mean from per-rank partials, the unique-id broadcast, and failure
detection -- a rank that dies before the rendezvous makes the other fail on
the host within its timeout, with nothing enqueued on any GPU."""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

from ptxgen.dist import shard_range

WORKER = Path(__file__).parent / "dist_worker.py"


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _launch(mode, world=2, timeout=120, extra_env=None):
    port = _port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        env.update(extra_env or {})
        procs.append(subprocess.Popen([sys.executable, str(WORKER), mode], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
    outs = []
    for p in procs:
        try:
            o, e = p.communicate(timeout=timeout)
        except subprocess.TimeoutExpired:
            p.kill()
            o, e = p.communicate()
        outs.append((p.returncode, o, e))
    return outs


@pytest.mark.parametrize("n,world", [(1000, 1), (1 << 20, 2), (1 << 20 | 12, 8), (37, 3)])
def test_shard_range_covers_exactly(n, world):
    spans = [shard_range(n, world, r, align=4) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a, b), (c, d) in zip(spans, spans[1:]):
        assert b == c and (b % 4 == 0)


def test_global_mean_from_rank_partials():
    outs = _launch("mean")
    assert all(rc == 0 for rc, _, _ in outs), outs
    res = json.loads(outs[0][1].strip().splitlines()[-1])
    assert abs(res["mean"] - res["ref"]) <= 1e-5 * abs(res["ref"])


def test_unique_id_broadcast():
    outs = _launch("bcast")
    assert all(rc == 0 for rc, _, _ in outs)
    assert all(json.loads(o.strip().splitlines()[-1])["ok"] for _, o, _ in outs)


def test_missing_rank_fails_on_the_host():
    outs = _launch("die", timeout=90, extra_env={"RDV_TIMEOUT": "5"})
    assert outs[1][0] == 3
    assert outs[0][0] != 0, "the surviving rank must fail, not hang or succeed"


def test_allgather_for_peer_inboxes():
    """The IPC-handle exchange of ``PeerInbox`` and its one-GPU-per-rank check
    (run on gloo ranks: no GPU is touched)."""
    outs = _launch("gather")
    assert len(outs) == 2
    for rc, out, err in outs:
        assert rc == 0, err
        o = json.loads(out.strip().splitlines()[-1])
        assert o["ok"] and o["distinct"] and o["shared_detected"]
        assert o["names"] == ["3", "5"]
