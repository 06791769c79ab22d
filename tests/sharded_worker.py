"""One rank of the 2-GPU sharded mul_mat check (launched by tests/test_sharded_mgpu.py
through torchrun; not a test module itself).  Every rank builds the same full weights
from a seed, keeps its M/G rows, runs mlzc_mul_mat_sharded_dev through NCCL, and compares
the gathered Y with the single-GPU mul_mat of the full weights and with the oracle on
sampled rows.  Writes one JSON result per rank to argv[1]."""
import datetime
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main(out_path: str) -> None:
    import torch
    import torch.distributed as dist
    import mlz_b200
    import oracle
    from mlz_b200 import synth
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    obj = [mlz_b200.Comm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    comm = mlz_b200.Comm(world, rank, local, obj[0], timeout_ms=30000)
    res = {"rank": rank, "cases": []}
    try:
        for (kind, M, K, N) in [("f16", 1024, 512, 1), ("f16", 2048, 1024, 4), ("f16", 512, 768, 33),
                                ("f16", 1024, 256, 256), ("f16", 516, 256, 5), ("q4k", 1024, 1024, 1),
                                ("q4k", 512, 512, 16)]:
            g = synth.rng(5000 + M + K + N)
            if kind == "f16":
                w = synth.f16_weights(g, M, K)
            else:
                w = synth.q4k_blocks(g, M, K)
            x = synth.f32_acts(g, N, K)
            m_loc = M // world
            wd = torch.from_numpy(np.ascontiguousarray(w[rank * m_loc:(rank + 1) * m_loc])).to(dev)
            xd = torch.from_numpy(x).to(dev)
            y = comm.mul_mat_sharded(wd, xd, M)
            full = mlz_b200.mul_mat(torch.from_numpy(w).to(dev), xd)
            torch.cuda.synchronize()
            yh, fh = y.cpu().numpy(), full.cpu().numpy()
            rows = np.sort(g.choice(M, size=16, replace=False))
            if kind == "f16":
                want = oracle.mul_mat_f16(np.ascontiguousarray(w[rows]).view(np.uint16), x)
            else:
                want = oracle.mul_mat_q4k(np.ascontiguousarray(w[rows]), x)
            res["cases"].append({"kind": kind, "M": M, "K": K, "N": N,
                                 "vs_single": float(np.max(np.abs(yh - fh)) / max(np.max(np.abs(fh)), 1e-30)),
                                 "vs_oracle": float(oracle.rel_err(yh[:, rows], want)),
                                 "finite": bool(np.isfinite(yh).all())})
        res["device_errors"] = mlz_b200.device_errors(local)
    finally:
        comm.destroy()
        dist.destroy_process_group()
    with open(f"{out_path}.{rank}", "w") as f:
        json.dump(res, f)


if __name__ == "__main__":
    main(sys.argv[1])
