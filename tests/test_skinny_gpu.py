"""GPU parity of the skinny F16 mul_mat on the tensor cores (mma.sync, 2 <= N <= 16).

Gate: max |y - y_oracle| / max |y_oracle| <= 1e-3 against the fp64 oracle with the
activations narrowed to f16 (the reference's F16 path); one launch per call."""
import numpy as np
import pytest

import mlz_b200
import oracle
from mlz_b200 import synth

TOL = 1e-3
pytestmark = pytest.mark.gpu


def _run(dev, w, x, x_pad=0, y_pad=0):
    import torch
    wd = torch.from_numpy(w).to(dev)
    N, K = x.shape
    xb = torch.zeros((N, K + x_pad), dtype=torch.float32, device=dev)
    xb[:, :K] = torch.from_numpy(x).to(dev)
    M = w.shape[0]
    yb = torch.full((N, M + y_pad), float("nan"), dtype=torch.float32, device=dev)
    n0 = mlz_b200.launch_count()
    mlz_b200.mul_mat(wd, xb[:, :K], out=yb[:, :M])
    launched = mlz_b200.launch_count() - n0
    torch.cuda.synchronize()
    yh = yb.cpu().numpy()
    if y_pad:
        assert np.isnan(yh[:, M:]).all(), "wrote outside the output columns"
    return yh[:, :M], launched


@pytest.mark.parametrize("M,K,N", [(31, 8, 2), (100, 24, 3), (257, 520, 5), (64, 3072, 8), (33, 1000, 9),
                                   (500, 72, 16), (129, 2056, 12), (16, 4096, 15), (300, 136, 7),
                                   (47, 256, 16), (8192, 3072, 4), (1, 64, 2)])
def test_edge_shapes(dev, M, K, N):
    g = synth.rng(1700 + M + K + N)
    w = synth.f16_weights(g, M, K)
    x = synth.f32_acts(g, N, K)
    y, launched = _run(dev, w, x, x_pad=4, y_pad=3)
    assert launched == 1
    assert oracle.rel_err(y, oracle.mul_mat_f16(w.view(np.uint16), x)) <= TOL


@pytest.mark.parametrize("N", [2, 8, 13, 16])
def test_full_size_sampled_rows(dev, N):
    """W 8192x3072 (the decode projection): every column, 64 sampled rows against the oracle."""
    g = synth.rng(synth.seed_for(1, 100 + N))
    w = synth.f16_weights(g, 8192, 3072)
    x = synth.f32_acts(g, N, 3072)
    y, launched = _run(dev, w, x)
    assert launched == 1
    rows = np.sort(g.choice(8192, size=64, replace=False))
    want = oracle.mul_mat_f16(np.ascontiguousarray(w[rows]).view(np.uint16), x)
    assert oracle.rel_err(y[:, rows], want) <= TOL
    assert np.isfinite(y).all()


@pytest.mark.parametrize("N", [2, 9, 16])
def test_power_of_two_scaling_and_repeat_full_size(dev, N):
    import torch
    gen = torch.Generator(device=dev).manual_seed(40 + N)
    w = synth.f16_weights_dev(gen, 28672, 8192, dev)
    x = torch.randn((N, 8192), generator=gen, device=dev)
    x = torch.where(x.abs() < 1e-3, torch.zeros_like(x), x)  # keep 4x out of f16 subnormals
    y = mlz_b200.mul_mat(w, x)
    y4 = mlz_b200.mul_mat(w, 4.0 * x)
    y2 = mlz_b200.mul_mat(w, x)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    assert torch.equal(y4, 4.0 * y)
    assert torch.equal(y2, y)
