"""GPU: F32 -> Q8_K activation quantisation (mlzc_quantize_q8k_dev) against the oracle's
restatement of the reference's quantize_row_q8_k_reference
(src/simd/ggml_simd_hook.cpp:109-148): bit-identical blocks (d, quants, group sums)."""
import numpy as np
import pytest

import mlz_b200
import oracle
from mlz_b200 import synth

pytestmark = pytest.mark.gpu


def _oracle_blocks(x):
    return np.stack([oracle.quantize_q8k(x[n]) for n in range(x.shape[0])])


@pytest.mark.parametrize("N,K", [(1, 256), (3, 4096), (16, 14336), (5, 768)])
def test_q8k_bit_identical(dev, N, K):
    import torch
    g = synth.rng(8000 + N + K)
    x = synth.f32_acts(g, N, K)
    x[0, :256] = 0.0                                  # an all-zero block: d = 0, q = 0
    if N > 1:
        x[1, 256:512] *= 1e-30                        # tiny values
        x[1, :256] = np.where(np.arange(256) % 2, 1e20, -3e19).astype(np.float32)
    if K >= 768:
        x[-1, 512:768] = np.round(x[-1, 512:768] * 4) / 4   # exact halves after scaling (ties)
    got = mlz_b200.quantize_q8k(torch.from_numpy(x).to(dev)).cpu().numpy()
    want = _oracle_blocks(x)
    assert got.shape == want.shape
    assert np.array_equal(got, want)


def test_q8k_strided_and_unaligned_columns(dev):
    import torch
    g = synth.rng(8100)
    N, K = 4, 512
    base = torch.from_numpy(synth.f32_acts(g, N, K + 3)).to(dev)
    x = base[:, 1:K + 1]                              # 4-byte aligned, not 16-byte aligned
    out = torch.full((N, 2 * 292 + 8), 0xAB, dtype=torch.uint8, device=dev)
    mlz_b200.quantize_q8k(x, out=out[:, :2 * 292])
    o = out.cpu().numpy()
    assert (o[:, 2 * 292:] == 0xAB).all(), "wrote past the blocks"
    assert np.array_equal(o[:, :2 * 292], _oracle_blocks(x.cpu().numpy()))


def test_q8k_rejects_ragged_k(dev):
    import torch
    x = torch.zeros((1, 300), device=dev)
    with pytest.raises(mlz_b200.MlzcError):
        mlz_b200.quantize_q8k(x, out=torch.zeros((1, 292), dtype=torch.uint8, device=dev))


def test_q8k_matches_reference_quantiser_fixture(dev, golden):
    """The GPU quantiser against blocks produced by the reference's own
    quantize_row_q8_k_reference (ggml_simd_hook.cpp:109-148): bit-identical."""
    import torch
    f = golden("q8k_reference.npz")
    got = mlz_b200.quantize_q8k(torch.from_numpy(f["x"]).to(dev)).cpu().numpy()
    assert np.array_equal(got.view(np.uint8).reshape(f["q8k"].shape), f["q8k"])
