"""Host logic of the multi-GPU path, as world-size-2 `gloo` process groups on CPU.

The row-sharded mul_mat (config c5) gives every rank M/G weight rows, all-gathers the
[N][M/G] output slices as [G][N][M/G] and permutes them to ggml's [N][M].  These tests check
that decomposition against the unsharded oracle, the rendezvous of the NCCL unique id over
a torch.distributed group, the bench's max-over-ranks reduction, and that the reference arm
under torchrun prints exactly one line (rank 0)."""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(fn, world: int = 2):
    import torch.multiprocessing as mp
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    results = {}
    while not q.empty():
        r, out = q.get()
        results[r] = out
    for p in procs:
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    assert sorted(results) == list(range(world)), results
    return results


def _entry(fn, rank, world, port, q):
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, fn(rank, world)))
    finally:
        dist.destroy_process_group()


def _sharded_rows(rank, world):
    import torch
    import torch.distributed as dist
    import oracle
    from mlz_b200 import synth
    M, K, N = 96, 136, 5
    g = synth.rng(4242)
    w = synth.f16_weights(g, M, K)
    x = synth.f32_acts(g, N, K)
    m_loc = M // world
    mine = oracle.mul_mat_f16(np.ascontiguousarray(w[rank * m_loc:(rank + 1) * m_loc]).view(np.uint16), x)  # [N][m_loc]
    parts = [torch.empty((N, m_loc), dtype=torch.float64) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(mine, dtype=np.float64)))
    gathered = torch.stack(parts)                               # [G][N][m_loc]
    y = gathered.permute(1, 0, 2).reshape(N, M).numpy()         # [N][M]
    full = oracle.mul_mat_f16(w.view(np.uint16), x)
    return bool(np.array_equal(y, full))


def test_row_shards_gathered_and_permuted_equal_unsharded():
    assert all(_run_ranks(_sharded_rows).values())


def _uid(rank, world):
    import torch.distributed as dist
    import mlz_b200
    obj = [mlz_b200.Comm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0].hex()


def test_nccl_unique_id_rendezvous():
    try:
        import mlz_b200
        mlz_b200.Comm.unique_id()
    except Exception as exc:  # NCCL not loadable here: nothing to rendezvous
        pytest.skip(f"NCCL unique id unavailable: {exc}")
    res = _run_ranks(_uid)
    assert res[0] == res[1] and len(bytes.fromhex(res[0])) == 128 and any(bytes.fromhex(res[0]))


def _max(rank, world):
    import bench
    return bench.max_over_ranks(1.5 + rank, world)


def test_bench_max_over_ranks():
    assert _run_ranks(_max) == {0: 2.5, 1: 2.5}


def test_reference_arm_under_torchrun_prints_one_line():
    port = _free_port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus",
           "2", "--config", "c1", "--steps", "1", "--warmup", "1", "--cpu-seconds", "0.3"]
    out = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["kind"] == "port"
