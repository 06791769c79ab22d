"""GPU: the ggml-hook-level entry point with host tensors, as the patched
ggml_compute_forward_mul_mat would call it from every threadpool thread."""
import threading

import numpy as np
import pytest

import mlz_b200
import oracle
from mlz_b200 import synth

pytestmark = pytest.mark.gpu


def _views(w, x, y, wtype, K=None):
    return (mlz_b200.tensor_view(w, wtype, ne0=K), mlz_b200.tensor_view(x, mlz_b200.TYPE_F32),
            mlz_b200.tensor_view(y, mlz_b200.TYPE_F32))


@pytest.mark.parametrize("nth", [1, 4, 16])
def test_f16_all_threads_handled(dev, nth):
    mlz_b200.lib().mlzc_weight_cache_clear()
    g = synth.rng(600 + nth)
    w = synth.f16_weights(g, 1000, 768)
    x = synth.f32_acts(g, 3, 768)
    y = np.full((3, 1000), np.nan, dtype=np.float32)
    s0, s1, d = _views(w, x, y, mlz_b200.TYPE_F16)
    res = [None] * nth

    def run(i):
        res[i] = mlz_b200.ggml_simd_try_mul_mat(s0, s1, d, i, nth)

    ts = [threading.Thread(target=run, args=(i,)) for i in range(nth)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=60)
    assert res == [1] * nth
    assert oracle.rel_err(y, oracle.mul_mat_f16(w.view(np.uint16), x)) <= 1e-3


def test_q4k_and_f32_through_hook(dev):
    g = synth.rng(610)
    K = 1024
    wq = synth.q4k_blocks(g, 96, K)
    x = synth.f32_acts(g, 2, K)
    y = np.zeros((2, 96), dtype=np.float32)
    assert mlz_b200.ggml_simd_try_mul_mat(*_views(wq, x, y, mlz_b200.TYPE_Q4_K, K=K)) == 1
    assert oracle.rel_err(y, oracle.mul_mat_q4k(wq, x)) <= 2e-3
    wf = g.standard_normal((50, K), dtype=np.float32)
    y2 = np.zeros((2, 50), dtype=np.float32)
    assert mlz_b200.ggml_simd_try_mul_mat(*_views(wf, x, y2, mlz_b200.TYPE_F32)) == 1
    assert oracle.rel_err(y2, oracle.mul_mat_f32(wf, x)) <= 1e-3


def test_reused_host_buffer_is_reuploaded(dev):
    """A host buffer refilled with other weights at the same address is detected by the
    cache's content fingerprint and uploaded again."""
    g = synth.rng(615)
    w = synth.f16_weights(g, 128, 256)
    x = synth.f32_acts(g, 2, 256)
    y = np.zeros((2, 128), dtype=np.float32)
    views = _views(w, x, y, mlz_b200.TYPE_F16)
    assert mlz_b200.ggml_simd_try_mul_mat(*views) == 1
    w[:] = synth.f16_weights(g, 128, 256)      # same address, new contents
    assert mlz_b200.ggml_simd_try_mul_mat(*views) == 1
    assert oracle.rel_err(y, oracle.mul_mat_f16(w.view(np.uint16), x)) <= 1e-3


def test_weight_cache_reuse_and_strided_dst(dev):
    g = synth.rng(620)
    w = synth.f16_weights(g, 64, 256)
    big_y = np.full((4, 80), np.nan, dtype=np.float32)   # dst rows 80 floats apart
    y = big_y[:, :64]
    for rep in range(3):
        x = synth.f32_acts(g, 4, 256)
        s0 = mlz_b200.tensor_view(w, mlz_b200.TYPE_F16)
        s1 = mlz_b200.tensor_view(x, mlz_b200.TYPE_F32)
        d = mlz_b200.tensor_view(y, mlz_b200.TYPE_F32)
        assert mlz_b200.ggml_simd_try_mul_mat(s0, s1, d) == 1
        assert oracle.rel_err(y, oracle.mul_mat_f16(w.view(np.uint16), x)) <= 1e-3
        assert np.isnan(big_y[:, 64:]).all()
    mlz_b200.lib().mlzc_weight_cache_clear()


def test_weight_handle_host_call(dev):
    g = synth.rng(630)
    w = synth.f16_weights(g, 300, 512)
    h = mlz_b200.Weight(w.view(np.uint16), mlz_b200.TYPE_F16, 512)
    x = synth.f32_acts(g, 9, 512)
    y = h.mul_mat(x)
    h.free()
    assert oracle.rel_err(y, oracle.mul_mat_f16(w.view(np.uint16), x)) <= 1e-3


@pytest.mark.parametrize("nth", [1, 3])
def test_f32_node_matches_reference_hook(dev, golden, nth):
    """The same one-column F32 nodes the reference's own ggml_simd_try_mul_mat computed
    (its F32 branch, compiled from source): this hook returns 1 on every thread and the
    same values to fp32 rounding."""
    f = golden("hook_reference.npz")
    for i in range(3):
        w, x = f[f"f32_{i}__w"], f[f"f32_{i}__x"]
        y = np.full((1, w.shape[0]), np.nan, dtype=np.float32)
        s0, s1, d = _views(w, x, y, mlz_b200.TYPE_F32)
        assert [mlz_b200.ggml_simd_try_mul_mat(s0, s1, d, t, nth) for t in range(nth)] == [1] * nth
        assert oracle.rel_err(y, f[f"f32_{i}_nth{nth}__y"]) < 1e-5
