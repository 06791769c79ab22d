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
    np.testing.assert_allclose(y[:, 0], 0.5 * x.astype(np.float64).sum(axis=1), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("M,K,N", [(1, 256, 1), (3, 512, 2), (37, 768, 5), (300, 256, 17), (8, 1024, 33)])
def test_edge_shapes(dev, M, K, N):
    g = synth.rng(300 + M + K + N)
    blocks = synth.q4k_blocks(g, M, K)
    x = synth.f32_acts(g, N, K)
    y = _run(dev, blocks, x, y_pad=1)
    assert oracle.rel_err(y, oracle.mul_mat_q4k(blocks, x)) <= TOL
