"""GPU parity of the Q6_K dequant-dot (ggml type 14; the reference hook routes it with
Q4_K, src/simd/ggml_simd_hook.cpp:282-288) against the oracle's dequantised-F32 product.

Gate: max |y - y_oracle| / max |y_oracle| <= 2e-3, with the oracle dequantising the same
blocks with GGUF semantics (pinned bit for bit to the gguf decoder) and accumulating in
fp64.  With one-hot activations the kernel's output is the dequantised weight itself,
which must equal the gguf decoder's value bit for bit."""
import numpy as np
import pytest

import mlz_b200
import oracle
from mlz_b200 import synth

TOL = 2e-3
pytestmark = pytest.mark.gpu
Q6 = mlz_b200.TYPE_Q6_K


def _run(dev, blocks, x, y_pad=0):
    import torch
    w = torch.from_numpy(blocks).to(dev)
    xd = torch.from_numpy(x).to(dev)
    M, N = blocks.shape[0], x.shape[0]
    yb = torch.full((N, M + y_pad), float("nan"), dtype=torch.float32, device=dev)
    mlz_b200.mul_mat(w, xd, out=yb[:, :M], w_type=Q6)
    torch.cuda.synchronize()
    yh = yb.cpu().numpy()
    if y_pad:
        assert np.isnan(yh[:, M:]).all()
    return yh[:, :M]


def test_dequant_bit_identical_to_gguf(dev, golden):
    f = golden("q6k_gguf.npz")
    blocks, K = f["blocks"], int(f["K"])
    eye = np.eye(K, dtype=np.float32)                # column n = one-hot at k = n
    want = f["dequant"].T
    # decode-sized calls (32 columns at a time): the weights enter the MMAs exactly, so
    # y[n, m] = w[m, n] bit for bit (a zero weight may come out as +0 where the decoder gives -0)
    for n0 in range(0, K, 32):
        y = _run(dev, blocks, eye[n0:n0 + 32], y_pad=1)
        assert (y == want[n0:n0 + 32]).all()


def _f16_row_image(dq, d_bound):
    """What the prefill path stores for one row: f16(RNE) of w 2^-e, times 2^e, with e the
    smallest exponent that brings the row's bound within 65504."""
    import math
    e = 0
    if d_bound > 65504.0:
        f, e = math.frexp(d_bound / 65504.0)
        e = e - 1 if f == 0.5 else e
    return (np.ldexp(dq, -e).astype(np.float16).astype(np.float32) * np.float32(2.0 ** e)).astype(np.float32)


def test_prefill_dequant_is_f16_rounding_of_gguf(dev, golden):
    """Prefill sizes (N = K = 512 here) dequantise to f16 once: with a one-hot X the GEMM
    returns the stored f16 weights, which must be the RNE roundings of the decoder's f32
    weights -- after a power-of-two row scale where |d| 4096 exceeds the f16 range (the
    golden blocks include d = 65504)."""
    f = golden("q6k_gguf.npz")
    blocks, K = f["blocks"], int(f["K"])
    rep = 1366   # the golden rows tiled to 8196 x 512: over the 4 M weights the path needs
    y = _run(dev, np.tile(blocks, (rep, 1)), np.eye(K, dtype=np.float32), y_pad=1)
    dq = f["dequant"].astype(np.float32)
    nb = K // 256
    for m in range(blocks.shape[0]):
        assert all((y[:, m + 6 * i] == y[:, m]).all() for i in (1, rep // 2, rep - 1))
        d = blocks[m].reshape(nb, 210)[:, 208:210].copy().view(np.float16).astype(np.float32).ravel()
        want = _f16_row_image(dq[m], float(np.abs(d).max()) * 4096.0)
        assert (y[:, m] == want).all(), m


@pytest.mark.parametrize("MK", [(4096, 4096), (14336, 4096), (4096, 14336)])
@pytest.mark.parametrize("B", [1, 4, 16])
def test_llama31_8b_shapes(dev, MK, B):
    """Llama-3.1-8B projection shapes, every column of 64 rows spread over M."""
    import torch
    M, K = MK
    gen = torch.Generator(device=dev).manual_seed(9000 + M + K + B)
    w = synth.q6k_blocks_dev(gen, M, K, dev)
    x = torch.randn((B, K), generator=gen, device=dev)
    y = mlz_b200.mul_mat(w, x, w_type=Q6)
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([np.linspace(0, M - 1, 62).astype(np.int64), [1, M - 2]]))
    rt = torch.from_numpy(rows).to(dev)
    want = oracle.mul_mat_q6k(w.index_select(0, rt).cpu().numpy(), x.cpu().numpy())
    got = y.index_select(1, rt).cpu().numpy()
    assert np.isfinite(got).all()
    assert oracle.rel_err(got, want) <= TOL


@pytest.mark.parametrize("M,K,N", [(1, 256, 1), (3, 512, 2), (37, 768, 5), (300, 256, 17), (8, 1024, 33),
                                   (17, 2304, 3), (2053, 4352, 7), (64, 14336, 4), (33, 11520, 9), (16, 256, 8),
                                   (8197, 4096, 1), (100, 1024, 2), (37, 3072, 3), (16, 8192, 4), (5, 2048, 1),
                                   (1000, 5120, 2)])
def test_edge_shapes(dev, M, K, N):
    """Odd block counts (odd row strides: rows alternate between 4- and 2-byte alignment),
    ragged row tiles, 1 .. 33 columns; K a multiple of 1024 with N <= 4 takes the int8 path
    (partial last unit at K = 1024, 3072, 5120)."""
    g = synth.rng(9300 + M + K + N)
    blocks = synth.q6k_blocks(g, M, K)
    x = synth.f32_acts(g, N, K)
    y = _run(dev, blocks, x, y_pad=1)
    assert oracle.rel_err(y, oracle.mul_mat_q6k(blocks, x)) <= TOL


def test_repeat_and_linearity_full_size(dev):
    import torch
    M, K, B = 14336, 4096, 4
    gen = torch.Generator(device=dev).manual_seed(9400)
    w = synth.q6k_blocks_dev(gen, M, K, dev)
    x = torch.randn((B, K), generator=gen, device=dev)
    x = torch.where(x.abs() < 1e-3, torch.zeros_like(x), x)   # keep 4x out of f16 subnormals
    y = mlz_b200.mul_mat(w, x, w_type=Q6)
    y4 = mlz_b200.mul_mat(w, 4.0 * x, w_type=Q6)
    y2 = mlz_b200.mul_mat(w, x, w_type=Q6)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    # powers of two commute with every rounding except where an f16 part of an activation
    # group sum is subnormal (the int8 path for N <= 4): 1e-6 of max |y|
    assert ((y4 - 4.0 * y).abs().max() / (4.0 * y).abs().max()).item() <= 1e-6
    assert torch.equal(y2, y)


def test_q6k_through_hook(dev):
    g = synth.rng(9500)
    M, K, N = 96, 1024, 3
    w = synth.q6k_blocks(g, M, K)
    x = synth.f32_acts(g, N, K)
    y = np.full((N, M), np.nan, dtype=np.float32)
    s0 = mlz_b200.tensor_view(w, Q6, ne0=K)
    s1 = mlz_b200.tensor_view(x, mlz_b200.TYPE_F32)
    d = mlz_b200.tensor_view(y, mlz_b200.TYPE_F32)
    assert mlz_b200.ggml_simd_try_mul_mat(s0, s1, d, 0, 1) == 1
    assert oracle.rel_err(y, oracle.mul_mat_q6k(w, x)) <= TOL


@pytest.mark.parametrize("M,K,N", [(4096, 4096, 64), (14336, 4096, 256), (1001, 2304, 100), (37, 768, 65), (1001, 4352, 100)])
def test_prefill_sizes_dequant_then_gemm(dev, M, K, N):
    """64 columns and more: dequantised to f16 once (odd block counts: rows 2-byte aligned),
    then the tcgen05 GEMM.  Oracle on sampled rows, every column."""
    g = synth.rng(9700 + M + K + N)
    blocks = synth.q6k_blocks(g, M, K)
    x = synth.f32_acts(g, N, K)
    y = _run(dev, blocks, x, y_pad=1)
    rows = np.unique(np.concatenate([g.choice(M, size=min(M, 40), replace=False), [0, M - 1]]))
    assert np.isfinite(y).all()
    assert oracle.rel_err(y[:, rows], oracle.mul_mat_q6k(np.ascontiguousarray(blocks[rows]), x)) <= TOL
