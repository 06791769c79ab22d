"""GPU, one rank: the row-sharded mul_mat through its peer-memory all-gather (exchange
region, push and wait kernels, device-side epochs) with a communicator of one rank, against
the unsharded mul_mat bit for bit; consecutive calls of alternating shapes (the two
epoch-parity slots), and the calls captured in a CUDA graph and replayed (epochs advance
on the device, not in the captured arguments)."""
import numpy as np
import pytest

import mlz_b200
from mlz_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def comm(dev):
    c = mlz_b200.Comm(1, 0, 0, mlz_b200.Comm.unique_id(), timeout_ms=20000)
    yield c
    c.destroy()


# (3584 x 8192 and 2050 x 28672 at one column take the fused decode GEMV's 4-row launch
# shapes, with 4 and 8 warps splitting K, as the 70B FFN's row shards on 8 and 4 GPUs do)
CASES = [(4096, 1024, 1), (1024, 512, 33), (2048, 1024, 256), (516, 256, 5), (3584, 8192, 1), (2050, 28672, 1)]


def test_single_rank_equals_unsharded(dev, comm):
    import torch
    for rep in range(2):
        for i, (M, K, N) in enumerate(CASES):
            gen = torch.Generator(device=dev).manual_seed(600 + i)
            w = synth.f16_weights_dev(gen, M, K, dev)
            x = torch.randn((N, K), generator=gen, device=dev)
            y = comm.mul_mat_sharded(w, x, M)
            ref = mlz_b200.mul_mat(w, x)
            torch.cuda.synchronize()
            assert torch.equal(y, ref), (rep, M, K, N)


@pytest.mark.parametrize("N", [1, 4, 64])
def test_single_rank_graph_replay(dev, comm, N):
    """N = 1 takes the fused decode GEMV (outputs stored straight into the exchange slots),
    N = 4 the slice + push kernels, N = 64 the tcgen05 GEMM that stores its tiles into its
    rows of Y and into the other ranks' slots (none here) before the wait kernel."""
    import torch
    M, K = 2048, 1024
    gen = torch.Generator(device=dev).manual_seed(700)
    ws_ = [synth.f16_weights_dev(gen, M, K, dev) for _ in range(3)]
    x = torch.randn((N, K), generator=gen, device=dev)
    ys = [torch.full((N, M), float("nan"), device=dev) for _ in range(3)]
    wsb = comm.workspace_bytes(mlz_b200.TYPE_F16, M, K, N)
    work = torch.empty(wsb, dtype=torch.uint8, device=dev)
    for j in range(3):                       # warm-up outside capture
        comm.mul_mat_sharded(ws_[j], x, M, out=ys[j], workspace=work)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for j in range(3):
            comm.mul_mat_sharded(ws_[j], x, M, out=ys[j], workspace=work, stream=s)
    refs = [mlz_b200.mul_mat(w, x) for w in ws_]
    for _ in range(3):
        for y in ys:
            y.fill_(float("nan"))
        with torch.cuda.stream(s):
            g.replay()
        torch.cuda.synchronize()
        for y, r in zip(ys, refs):
            assert torch.equal(y, r)
    del g
