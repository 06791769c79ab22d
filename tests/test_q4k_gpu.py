"""GPU parity of the Q4_K dequant-dot against the oracle's dequantised-F32 product.

Gate: max |y - y_oracle| / max |y_oracle| <= 2e-3, with the oracle dequantising the same
blocks with GGUF semantics (pinned to the gguf decoder) and accumulating in fp64."""
import numpy as np
import pytest

import mlz_b200
import oracle
from mlz_b200 import synth

TOL = 2e-3
pytestmark = pytest.mark.gpu


def _run(dev, blocks, x, y_pad=0):
    import torch
    w = torch.from_numpy(blocks).to(dev)
    xd = torch.from_numpy(x).to(dev)
    M, N = blocks.shape[0], x.shape[0]
    yb = torch.full((N, M + y_pad), float("nan"), dtype=torch.float32, device=dev)
    mlz_b200.mul_mat(w, xd, out=yb[:, :M])
    torch.cuda.synchronize()
    yh = yb.cpu().numpy()
    if y_pad:
        assert np.isnan(yh[:, M:]).all()
    return yh[:, :M]


@pytest.mark.parametrize("MK", [(4096, 4096), (14336, 4096), (4096, 14336)])
@pytest.mark.parametrize("B", [1, 4, 16])
def test_llama31_8b_shapes(dev, MK, B):
    M, K = MK
    g = synth.rng(synth.seed_for(3, B) + M + K)
    blocks = synth.q4k_blocks(g, M, K)
    x = synth.f32_acts(g, B, K)
    y = _run(dev, blocks, x)
    assert oracle.rel_err(y, oracle.mul_mat_q4k(blocks, x)) <= TOL


def test_gguf_golden_blocks(dev, golden):
    f = golden("q4k_gguf.npz")
    blocks, K = f["blocks"], int(f["K"])
    x = synth.f32_acts(synth.rng(3), 3, K)
    y = _run(dev, blocks, x, y_pad=2)
    want = x.astype(np.float64) @ f["dequant"].astype(np.float64).T
    # the golden blocks include d = 65504: compare per row against each row's magnitude
    den = np.maximum(np.abs(want).max(axis=0, keepdims=True), 1e-30)
    assert (np.abs(y - want) / den).max() <= TOL


def test_prefill_dequant_is_f16_rounding_of_gguf(dev, golden):
    """Prefill sizes (N = K = 512 here) dequantise to f16 once: with a one-hot X the GEMM
    returns the stored f16 weights, which must be the RNE roundings of the decoder's f32
    weights -- after a power-of-two row scale where |d| 945 + |dmin| 63 exceeds the f16
    range (the golden blocks include d = 65504)."""
    import math
    f = golden("q4k_gguf.npz")
    blocks, K = f["blocks"], int(f["K"])
    rep = 1366   # the golden rows tiled to 8196 x 512: over the 4 M weights the path needs
    y = _run(dev, np.tile(blocks, (rep, 1)), np.eye(K, dtype=np.float32), y_pad=1)
    dq = f["dequant"].astype(np.float32)
    nb = K // 256
    for m in range(blocks.shape[0]):
        assert all((y[:, m + 6 * i] == y[:, m]).all() for i in (1, rep // 2, rep - 1))
        hdr = blocks[m].reshape(nb, 144)[:, 0:4].copy().view(np.float16).astype(np.float32)
        bound = float((np.abs(hdr[:, 0]) * 945.0 + np.abs(hdr[:, 1]) * 63.0).max())
        e = 0
        if bound > 65504.0:
            fr, e = math.frexp(bound / 65504.0)
            e = e - 1 if fr == 0.5 else e
        want = np.ldexp(dq[m], -e).astype(np.float16).astype(np.float32) * np.float32(2.0 ** e)
        assert (y[:, m] == want).all(), m


def test_known_answer_block(dev):
    K = 512
    blk = np.zeros((1, 2, 144), dtype=np.uint8)
    blk[0, :, 0:2] = np.array([0.5], dtype=np.float16).view(np.uint8)
    blk[0, :, 2:4] = np.array([0.25], dtype=np.float16).view(np.uint8)
    blk[0, :, 4:8] = 1
    blk[0, :, 12:16] = 0x01
    blk[0, :, 16:] = 0x11
    blk = blk.reshape(1, -1)
    x = synth.f32_acts(synth.rng(8), 5, K)
    y = _run(dev, blk, x)
    # every weight is d * sc * q - dmin * m = 0.5 * 1 * 1 - 0.25 * 0; the kernel rounds the
    # activations to f16 once, so the exact answer is 0.5 * sum(f16(x))
    want = 0.5 * x.astype(np.float16).astype(np.float64).sum(axis=1)
    np.testing.assert_allclose(y[:, 0], want, rtol=1e-5, atol=1e-5)


def _int8_model(x):
    """The activations as the N <= 4 path carries them: per 256-value block one scale
    s = max|x| / 127 and two int8 vectors, x ~= s (hi + lo / 254)."""
    xb = x.astype(np.float32).reshape(x.shape[0], -1, 256)
    amax = np.abs(xb).max(axis=2, keepdims=True)
    s = (amax / np.float32(127.0)).astype(np.float32)
    inv = np.where(amax > 0, np.float32(127.0) / np.where(amax > 0, amax, 1), 0).astype(np.float32)
    hi = np.rint((xb * inv).astype(np.float32))
    r = (xb.astype(np.float64) - s.astype(np.float64) * hi).astype(np.float32)
    lo = np.clip(np.rint(((r * inv).astype(np.float32) * np.float32(254.0)).astype(np.float32)), -127, 127)
    return s.astype(np.float64), hi.astype(np.float64), lo.astype(np.float64)


@pytest.mark.parametrize("N", [1, 2, 4])
def test_known_answer_block_int8_path(dev, N):
    """Every weight 0.5 (as in the test above) with N <= 4 columns, where the activations
    are carried as int8 hi + lo per block: the exact answer is 0.5 sum_b s_b (sum hi + sum lo / 254)."""
    K = 512
    blk = np.zeros((1, 2, 144), dtype=np.uint8)
    blk[0, :, 0:2] = np.array([0.5], dtype=np.float16).view(np.uint8)
    blk[0, :, 2:4] = np.array([0.25], dtype=np.float16).view(np.uint8)
    blk[0, :, 4:8] = 1
    blk[0, :, 12:16] = 0x01
    blk[0, :, 16:] = 0x11
    blk = blk.reshape(1, -1)
    x = synth.f32_acts(synth.rng(9 + N), N, K)
    y = _run(dev, blk, x)
    s, hi, lo = _int8_model(x)
    want = 0.5 * (s[:, :, 0] * (hi.sum(axis=2) + lo.sum(axis=2) / 254.0)).sum(axis=1)
    np.testing.assert_allclose(y[:, 0], want, rtol=1e-5, atol=1e-6)
    # and the quantisation error itself is far inside the parity tolerance
    assert np.abs(y[:, 0] - 0.5 * x.sum(axis=1)).max() <= 1e-3 * np.abs(0.5 * x.sum(axis=1)).max() + 1e-4


@pytest.mark.parametrize("M,K,N", [(1, 256, 1), (3, 512, 2), (37, 768, 5), (300, 256, 17), (8, 1024, 33),
                                   (17, 2304, 3), (2053, 4352, 7), (64, 14336, 4), (40, 14336, 8), (16, 256, 8),
                                   (8200, 512, 3), (8197, 4096, 8), (100, 11520, 3), (33, 11520, 6),
                                   (8197, 4096, 1), (8197, 4096, 2), (5000, 2048, 4), (20, 18432, 1),
                                   (129, 6144, 2), (7, 256, 4)])
def test_edge_shapes(dev, M, K, N):
    g = synth.rng(300 + M + K + N)
    blocks = synth.q4k_blocks(g, M, K)
    x = synth.f32_acts(g, N, K)
    y = _run(dev, blocks, x, y_pad=1)
    assert oracle.rel_err(y, oracle.mul_mat_q4k(blocks, x)) <= TOL


@pytest.mark.parametrize("MK", [(14336, 4096), (4096, 14336)])
@pytest.mark.parametrize("B", [1, 16])
def test_power_of_two_scaling_is_exact_full_size(dev, MK, B):
    """Size-independent properties at the benchmark size: linearity (scaling the activations
    by 4 scales y by 4, to 1e-6 of max |y|: the f16 low part of a sub-block sum may be
    subnormal, where rounding does not commute with scaling) and bitwise repeatability."""
    import torch
    M, K = MK
    gen = torch.Generator(device=dev).manual_seed(11 + B)
    w = synth.q4k_blocks_dev(gen, M, K, dev)
    x = torch.randn((B, K), generator=gen, device=dev)
    x = torch.where(x.abs() < 1e-3, torch.zeros_like(x), x)  # keep 4x out of f16 subnormals
    y = mlz_b200.mul_mat(w, x)
    y4 = mlz_b200.mul_mat(w, 4.0 * x)
    y2 = mlz_b200.mul_mat(w, x)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    assert ((y4 - 4.0 * y).abs().max() / (4.0 * y).abs().max()).item() <= 1e-6
    assert torch.equal(y2, y), "repeat is bitwise identical"


@pytest.mark.parametrize("M,K,N", [(4096, 4096, 64), (14336, 4096, 256), (1000, 2304, 100), (37, 768, 65), (1001, 4352, 100),
                                   (4096, 14336, 128)])
def test_prefill_sizes_dequant_then_gemm(dev, M, K, N):
    """64 columns and more: the blocks are dequantised to f16 once and the tcgen05 GEMM runs
    (one pass over W instead of one per 16 columns).  Oracle on sampled rows, every column."""
    g = synth.rng(700 + M + K + N)
    blocks = synth.q4k_blocks(g, M, K)
    x = synth.f32_acts(g, N, K)
    y = _run(dev, blocks, x, y_pad=1)
    rows = np.unique(np.concatenate([g.choice(M, size=min(M, 40), replace=False), [0, M - 1]]))
    assert np.isfinite(y).all()
    assert oracle.rel_err(y[:, rows], oracle.mul_mat_q4k(np.ascontiguousarray(blocks[rows]), x)) <= TOL
