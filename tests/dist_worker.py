"""One rank of the multi-process CPU tests (run by tests/test_dist.py).

Modes:
  mean  -- each rank runs the mean IR (global count) on its shard with the
           CPU oracle, the partial results are summed over gloo, rank 0
           prints the global mean as JSON;
  bcast -- rank 0 broadcasts 128 bytes (the NCCL unique id path);
  die   -- rank 1 exits before the rendezvous; rank 0 must fail on the host;
  gather -- every rank all-gathers a 64-byte token (the IPC handle exchange of
           the peer inboxes) and the physical GPU names of two layouts: one
           GPU per rank, and two ranks on one GPU (which peer inboxes refuse).
"""

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "emmy-ptx_b200"))
sys.path.insert(0, ROOT)


def main():
    mode = sys.argv[1]
    rank = int(os.environ["RANK"])
    import numpy as np
    from ptxgen.dist import Rendezvous, shard_range
    if mode == "die" and rank == 1:
        sys.exit(3)
    try:
        rdv = Rendezvous(timeout_s=float(os.environ.get("RDV_TIMEOUT", "60")))
    except Exception as exc:  # noqa: BLE001
        print(json.dumps({"rank": rank, "error": type(exc).__name__}), flush=True)
        sys.exit(4)
    if mode == "bcast":
        b = bytes(range(128)) if rank == 0 else None
        got = rdv.bcast_bytes(b)
        print(json.dumps({"rank": rank, "ok": got == bytes(range(128))}), flush=True)
    elif mode == "gather":
        from ptxgen.dist import physical_gpu
        tok = bytes([rank]) * 64
        got = rdv.allgather_bytes(tok)
        os.environ["CUDA_VISIBLE_DEVICES"] = "3,5"
        distinct = rdv.allgather_bytes(physical_gpu(rank).encode())
        shared = rdv.allgather_bytes(physical_gpu(0).encode())
        print(json.dumps({"rank": rank, "ok": got == [bytes([r]) * 64 for r in range(rdv.world)],
                          "distinct": len(set(distinct)) == len(distinct),
                          "shared_detected": len(set(shared)) < len(shared),
                          "names": [d.decode().split(":")[-1] for d in distinct]}), flush=True)
    elif mode == "mean":
        from oracle.interp import interpret
        from ptxgen import irgen
        from ptxgen.loader import load_kernel_data
        n_total = 1 << 16
        x = np.random.default_rng(0).random(n_total, dtype=np.float32)
        lo, hi = shard_range(n_total, rdv.world, rank, align=4)
        g, m = irgen.reduce_full(hi - lo, mean=True)
        spec = load_kernel_data(g, m, "mean")
        spec.args["mean_keepdim_count"].data = [float(n_total)]
        out = interpret(spec, {"x": x[lo:hi],
                               "mean_keepdim_count": np.array([n_total], np.float32)})
        total = rdv.sum(float(out["mean"][0]))
        if rank == 0:
            print(json.dumps({"mean": total, "ref": float(x.astype(np.float64).mean())}),
                  flush=True)
    rdv.close()


if __name__ == "__main__":
    main()
