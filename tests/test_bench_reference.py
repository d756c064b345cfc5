"""bench.py's reference arm (the oracle port on every host core, no GPU):
one JSON line with the contract's keys, ``cores`` the workers it used.  For
the default configuration it runs the whole workload (same_config), for
another workload a bounded sample."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--workload", "pointwise", "--steps", "1", "--warmup", "3"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "GB/s"
    for key in ("metric", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]


def test_reference_arm_under_torchrun_prints_once():
    """Launched as the driver launches it for N > 1 (torchrun, two ranks,
    gloo rendezvous on 127.0.0.1): rank 0 alone runs and prints one line,
    the other rank exits 0 without work."""
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
                        "--master-port", "29631", str(ROOT / "bench.py"), "--gpus", "2",
                        "--impl", "reference", "--workload", "pointwise", "--steps", "1",
                        "--warmup", "3"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["value"] > 0


def test_reference_arm_full_default_configuration():
    """The driver's reference arm: the full configs[1] workload split over
    the host cores, its folded result checked against float64 in-run."""
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "3"],
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["config"]["same_config"] is True
    assert "2^26" in line["config"]["workload"] and line["cpu_baseline"]["kind"] == "port"
