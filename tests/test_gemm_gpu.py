"""GPU parity of the tcgen05 tensor-core GEMM (F16 weights, N > 16 activation columns, or
N >= 8 when the skinny path does not apply) and of the skinny mma.sync path (N <= 16).

Gate: max |y - y_oracle| / max |y_oracle| <= 1e-3 against the fp64 oracle with activations
narrowed to f16 (the reference's F16 path).  Full-size shapes are checked on a random
subset of weight rows (every column), where the fp64 oracle finishes in seconds."""
import numpy as np
import pytest

import mlz_b200
import oracle
from mlz_b200 import synth

TOL = 1e-3
pytestmark = pytest.mark.gpu


def _gemm(dev, w, x, y_pad=0):
    import torch
    wd = torch.from_numpy(w).to(dev)
    xd = torch.from_numpy(x).to(dev)
    M, N = w.shape[0], x.shape[0]
    yb = torch.full((N, M + y_pad), float("nan"), dtype=torch.float32, device=dev)
    n0 = mlz_b200.launch_count()
    mlz_b200.mul_mat(wd, xd, out=yb[:, :M])
    launched = mlz_b200.launch_count() - n0
    torch.cuda.synchronize()
    yh = yb.cpu().numpy()
    if y_pad:
        assert np.isnan(yh[:, M:]).all(), "wrote outside the output columns"
    return yh[:, :M], launched


@pytest.mark.parametrize("tokens", [512, 2048])
@pytest.mark.parametrize("proj", [("q", 3072, 3072), ("k", 1024, 3072), ("gate", 8192, 3072), ("down", 3072, 8192)])
def test_llama32_3b_layer_projections(dev, tokens, proj):
    name, M, K = proj
    g = synth.rng(synth.seed_for(2, tokens) + M + K)
    w = synth.f16_weights(g, M, K)
    x = synth.f32_acts(g, tokens, K)
    y, launched = _gemm(dev, w, x)
    assert launched == 2, "expected the narrow + tensor-core GEMM launches"
    rows = np.sort(g.choice(M, size=48, replace=False))
    want = oracle.mul_mat_f16(np.ascontiguousarray(w[rows]).view(np.uint16), x)
    assert oracle.rel_err(y[:, rows], want) <= TOL
    assert np.isfinite(y).all()


@pytest.mark.parametrize("M,K,N", [(128, 64, 8), (129, 72, 9), (1, 8, 16), (300, 520, 17), (127, 3072, 31),
                                   (256, 256, 33), (64, 1024, 100), (200, 136, 255), (130, 512, 256),
                                   (384, 320, 257), (8192, 3072, 32), (1000, 2000, 300),
                                   (256, 64, 128), (257, 136, 129), (600, 8, 500), (512, 4096, 160),
                                   (1024, 200, 2048)])
def test_edge_shapes(dev, M, K, N):
    g = synth.rng(700 + M + K + N)
    w = synth.f16_weights(g, M, K)
    x = synth.f32_acts(g, N, K)
    y, launched = _gemm(dev, w, x, y_pad=5)
    # N <= 16 with 16-byte-aligned operands and K % 8 == 0 takes the skinny mma.sync kernel
    skinny = N <= 16 and K % 8 == 0
    assert launched == (1 if skinny else 2)
    assert oracle.rel_err(y, oracle.mul_mat_f16(w.view(np.uint16), x)) <= TOL


def test_unaligned_rows_take_exact_fallback(dev):
    g = synth.rng(710)
    w = synth.f16_weights(g, 96, 100)          # 200-byte rows: not a TMA-legal stride
    x = synth.f32_acts(g, 40, 100)
    y, launched = _gemm(dev, w, x)
    assert oracle.rel_err(y, oracle.mul_mat_f16(w.view(np.uint16), x)) <= TOL


def test_power_of_two_scaling_full_layer(dev):
    """Size-independent property at the benchmark size (M = 2048 tokens)."""
    import torch
    gen = torch.Generator(device=dev).manual_seed(9)
    for (M, K) in [(3072, 3072), (8192, 3072), (3072, 8192)]:
        w = synth.f16_weights_dev(gen, M, K, dev)
        x = torch.randn((2048, K), generator=gen, device=dev)
        x = torch.where(x.abs() < 1e-3, torch.zeros_like(x), x)  # keep 4x out of f16 subnormals
        y = mlz_b200.mul_mat(w, x)
        y4 = mlz_b200.mul_mat(w, 4.0 * x)
        torch.cuda.synchronize()
        assert torch.isfinite(y).all()
        assert torch.equal(y4, 4.0 * y)


def test_repeat_is_deterministic(dev):
    import torch
    gen = torch.Generator(device=dev).manual_seed(10)
    w = synth.f16_weights_dev(gen, 3072, 3072, dev)
    x = torch.randn((512, 3072), generator=gen, device=dev)
    y1 = mlz_b200.mul_mat(w, x)
    y2 = mlz_b200.mul_mat(w, x)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
