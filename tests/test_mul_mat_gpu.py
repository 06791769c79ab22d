"""GPU parity of mul_mat (F16 and F32 weights) against the fp64 oracle.

Gate: max |y - y_oracle| / max |y_oracle| <= 1e-3 (F16/F32, fp32 accumulation); the
oracle narrows activations to f16 for F16 weights, as the reference's F16 path does."""
import numpy as np
import pytest

import mlz_b200
import oracle
from mlz_b200 import synth

TOL = 1e-3
pytestmark = pytest.mark.gpu


def _run(dev, w_np, x_np, x_pad=0, y_pad=0):
    import torch
    w = torch.from_numpy(w_np).to(dev)
    N, K = x_np.shape
    xb = torch.zeros((N, K + x_pad), dtype=torch.float32, device=dev)
    xb[:, :K] = torch.from_numpy(x_np).to(dev)
    x = xb[:, :K]
    M = w_np.shape[0]
    yb = torch.full((N, M + y_pad), float("nan"), dtype=torch.float32, device=dev)
    y = yb[:, :M]
    mlz_b200.mul_mat(w, x, out=y)
    torch.cuda.synchronize()
    yh = yb.cpu().numpy()
    if y_pad:
        assert np.isnan(yh[:, M:]).all(), "wrote outside the output columns"
    return yh[:, :M]


@pytest.mark.parametrize("N", [1, 8, 32])
def test_f16_llama32_3b_up_proj(dev, N):
    """W 8192x3072 f16 ~ N(0, 0.02), X 3072xN f32 ~ N(0, 1)."""
    g = synth.rng(synth.seed_for(1, N))
    w = synth.f16_weights(g, 8192, 3072)
    x = synth.f32_acts(g, N, 3072)
    y = _run(dev, w, x)
    want = oracle.mul_mat_f16(w.view(np.uint16), x)
    assert oracle.rel_err(y, want) <= TOL


@pytest.mark.parametrize("M,K,N", [(1, 64, 1), (5, 3080, 2), (33, 256, 3), (130, 520, 31), (64, 1024, 33),
                                   (17, 100, 4), (9, 7, 5), (3, 2056, 9)])
def test_f16_edge_shapes(dev, M, K, N):
    g = synth.rng(100 + M + K + N)
    w = synth.f16_weights(g, M, K)
    x = synth.f32_acts(g, N, K)
    y = _run(dev, w, x, x_pad=4, y_pad=3)
    assert oracle.rel_err(y, oracle.mul_mat_f16(w.view(np.uint16), x)) <= TOL


@pytest.mark.parametrize("M,K,N", [(256, 512, 1), (100, 36, 3), (64, 4096, 8), (7, 5, 2)])
def test_f32_weights(dev, M, K, N):
    g = synth.rng(200 + M + N)
    w = g.standard_normal((M, K), dtype=np.float32) * 0.02
    x = synth.f32_acts(g, N, K)
    y = _run(dev, w, x, y_pad=1)
    assert oracle.rel_err(y, oracle.mul_mat_f32(w, x)) <= TOL


def test_empty_and_degenerate(dev):
    import torch
    w = torch.zeros((8, 0), dtype=torch.float16, device=dev)
    x = torch.zeros((2, 0), dtype=torch.float32, device=dev)
    y = mlz_b200.mul_mat(w, x)
    torch.cuda.synchronize()
    assert (y.cpu() == 0).all()
    w = torch.zeros((0, 16), dtype=torch.float16, device=dev)
    x = torch.zeros((2, 16), dtype=torch.float32, device=dev)
    assert mlz_b200.mul_mat(w, x).shape == (2, 0)


@pytest.mark.parametrize("N", [1, 4, 32])
def test_power_of_two_scaling_is_exact_full_size(dev, N):
    """Size-independent property at the benchmark size: scaling X by 4 scales Y by exactly
    4 (power-of-two scaling commutes with every f16 / f32 rounding on the path)."""
    import torch
    gen = torch.Generator(device=dev).manual_seed(5)
    w = synth.f16_weights_dev(gen, 8192, 3072, dev)
    x = torch.randn((N, 3072), generator=gen, device=dev)
    x = torch.where(x.abs() < 1e-3, torch.zeros_like(x), x)  # keep 4x out of f16 subnormals
    y = mlz_b200.mul_mat(w, x)
    y4 = mlz_b200.mul_mat(w, 4.0 * x)
    torch.cuda.synchronize()
    assert torch.equal(y4, 4.0 * y)
    assert torch.isfinite(y).all()
