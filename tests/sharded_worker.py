"""One rank of the multi-GPU sharded mul_mat check (launched by tests/test_sharded_mgpu.py
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
        # small shapes (host-generated), then the Llama-3-70B FFN shapes at full size
        # (gate/up 28672x8192 at N = 1, down 8192x28672 at N = 1 and 256; generated on the
        # device from one seed on every rank, so every rank holds the same full W)
        for (kind, M, K, N) in [("f16", 1024, 512, 1), ("f16", 2048, 1024, 4), ("f16", 512, 768, 33),
                                ("f16", 1024, 256, 256), ("f16", 520, 256, 5), ("q4k", 1024, 1024, 1),
                                ("q4k", 512, 512, 16), ("f16", 28672, 8192, 1), ("f16", 8192, 28672, 1),
                                ("f16", 8192, 28672, 256)]:
            g = synth.rng(5000 + M + K + N)
            m_loc = M // world
            if M * K > (1 << 26):
                gen = torch.Generator(device=dev).manual_seed(5000 + M + K + N)
                wfull = synth.f16_weights_dev(gen, M, K, dev)
                xd = torch.randn((N, K), generator=gen, device=dev)
                x = xd.cpu().numpy()
                wd = wfull[rank * m_loc:(rank + 1) * m_loc].contiguous()
            else:
                w = synth.f16_weights(g, M, K) if kind == "f16" else synth.q4k_blocks(g, M, K)
                x = synth.f32_acts(g, N, K)
                wfull = torch.from_numpy(w).to(dev)
                wd = torch.from_numpy(np.ascontiguousarray(w[rank * m_loc:(rank + 1) * m_loc])).to(dev)
                xd = torch.from_numpy(x).to(dev)
            y = comm.mul_mat_sharded(wd, xd, M)
            full = mlz_b200.mul_mat(wfull, xd)
            torch.cuda.synchronize()
            yh, fh = y.cpu().numpy(), full.cpu().numpy()
            rows = np.sort(np.concatenate([g.choice(M, size=14, replace=False), [0, M - 1]]))
            w_rows = wfull.index_select(0, torch.from_numpy(rows).to(dev)).cpu().numpy()
            if kind == "f16":
                want = oracle.mul_mat_f16(w_rows.view(np.uint16), x)
            else:
                want = oracle.mul_mat_q4k(w_rows, x)
            del wfull, full
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
