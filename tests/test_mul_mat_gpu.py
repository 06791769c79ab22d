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
                                   (17, 100, 4), (9, 7, 5), (3, 2056, 9),
                                   # few rows over a long K: the warps of a CTA split K
                                   (1024, 28672, 1), (37, 16384, 2), (3584, 8192, 1), (515, 8200, 3)])
def test_f16_edge_shapes(dev, M, K, N):
    g = synth.rng(100 + M + K + N)
    w = synth.f16_weights(g, M, K)
    x = synth.f32_acts(g, N, K)
    y = _run(dev, w, x, x_pad=4, y_pad=3)
    assert oracle.rel_err(y, oracle.mul_mat_f16(w.view(np.uint16), x)) <= TOL


@pytest.mark.parametrize("M,K", [(16576, 512), (8192, 3072), (3584, 8192), (2048, 28672), (2050, 28672),
                                 (1024, 28672)])
def test_f16_decode_gemv_launch_shapes(dev, M, K):
    """One activation column through every launch shape of the decode GEMV: 4 rows per warp
    group with 1, 2, 4 and 8 warps splitting K (the shapes whose grid would be small:
    16576 x 512, C1's 8192 x 3072, the 8- and 4-GPU shards of the 70B FFN), a row count
    that is not a multiple of 4, and the 2-row shape (1024 x 28672); NaN guard columns
    around Y must stay NaN."""
    g = synth.rng(900 + M % 97 + K % 89)
    w = synth.f16_weights(g, M, K)
    x = synth.f32_acts(g, 1, K)
    y = _run(dev, w, x, x_pad=4, y_pad=8)
    assert oracle.rel_err(y, oracle.mul_mat_f16(w.view(np.uint16), x)) <= TOL


@pytest.mark.parametrize("M,K,N", [(256, 512, 1), (100, 36, 3), (64, 4096, 8), (7, 5, 2), (100, 8192, 3)])
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


def test_f16_matches_reference_simd_matmul_f16(dev, golden):
    """GPU F16 mul_mat against the reference's own F16 GEMM, simd_matmul_f16
    (src/simd/simd_matmul.cpp:428-480, f16 operands, fp32 accumulation, f16 result), on
    the committed fixture: the GPU's f32 result rounded to f16 is within 1 ulp of the
    reference's f16 result.  The cases reach the GEMV (N = 1), skinny tensor-core
    (N = 4, 8), tcgen05 GEMM (N >= 17) and unaligned kernels."""
    f = golden("matmul_f16_reference.npz")
    n = len([k for k in f.files if k.startswith("a")])
    for i in range(n):
        a, b, c = f[f"a{i}"], f[f"b{i}"], f[f"c{i}"]
        x = np.ascontiguousarray(b.T.view(np.float16).astype(np.float32))
        y = _run(dev, a.view(np.float16), x, y_pad=1)
        got = y.astype(np.float16).view(np.int16).astype(np.int32)
        want = c.T.view(np.int16).astype(np.int32)
        # ulp distance on the sign-magnitude f16 encoding
        to_ord = lambda v: np.where(v < 0, -(v & 0x7FFF), v)
        assert np.abs(to_ord(got) - to_ord(want)).max() <= 1, f"case {i}: {a.shape} x {b.shape}"


C5_MATS = [("gate", 28672, 8192), ("down", 8192, 28672)]


@pytest.mark.parametrize("N", [1, 256])
@pytest.mark.parametrize("name,M,K", C5_MATS)
def test_f16_llama3_70b_ffn_full_shape(dev, name, M, K, N):
    """Llama-3-70B FFN shapes at full size (gate/up 28672x8192, down 8192x28672) for
    N = 1 (GEMV) and N = 256 (tcgen05 GEMM): every column of 48 rows spread over all of M
    (both ends included) against the fp64 oracle."""
    import torch
    gen = torch.Generator(device=dev).manual_seed(7000 + M + N)
    w = synth.f16_weights_dev(gen, M, K, dev)
    x = torch.randn((N, K), generator=gen, device=dev)
    y = mlz_b200.mul_mat(w, x)
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([np.linspace(0, M - 1, 46).astype(np.int64), [1, M - 2]]))
    rows_t = torch.from_numpy(rows).to(dev)
    w_rows = w.index_select(0, rows_t).cpu().numpy()
    want = oracle.mul_mat_f16(w_rows.view(np.uint16), x.cpu().numpy())
    got = y.index_select(1, rows_t).cpu().numpy()
    assert np.isfinite(got).all()
    assert oracle.rel_err(got, want) <= TOL
