"""GPU: the allocation-free flash-attention entry point (mlzc_flash_attn_dev_noalloc).

It exists for callers that cannot allocate device memory per call; it must give the same
results as mlzc_flash_attn_dev (which takes a caller workspace) through the C ABI, on
consecutive calls that share its fixed scratch.  This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

import mlz_b200
from mlz_b200 import synth
from mlz_b200.ops import _nb

pytestmark = pytest.mark.gpu


def _desc(q, k, v, out, kv_len, scale):
    B, Hq, NQ, D = q.shape
    _, Hkv, L, _ = k.shape
    return mlz_b200.make_fa_desc(q.data_ptr(), _nb(q, 4), k.data_ptr(), _nb(k, 2), v.data_ptr(), _nb(v, 2),
                                 out.data_ptr(), _nb(out, 4), (B, Hq, NQ, Hkv, L, D), scale,
                                 kv_len_ptr=kv_len.data_ptr())


def _inputs(dev, seed, B, Hq, Hkv, L, D):
    import torch
    g = synth.rng(seed)
    q, k, v = synth.fa_inputs(g, B, Hq, Hkv, L, D)
    kl = synth.kv_lengths(g, B, 1, L)
    return (torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev),
            torch.from_numpy(kl).to(dev))


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(dev):
    import torch
    L = mlz_b200.lib()
    shapes = [(16, 32, 8, 8192, 128), (5, 8, 2, 3000, 64)]   # the second call reuses the scratch
    for i, (B, Hq, Hkv, Lmax, D) in enumerate(shapes):
        q, k, v, kl = _inputs(dev, 900 + i, B, Hq, Hkv, Lmax, D)
        scale = 1.0 / np.sqrt(D)
        out_ws = torch.full((B, Hq, 1, D), float("nan"), device=dev)
        out_na = torch.full((B, Hq, 1, D), float("nan"), device=dev)
        d_ws = _desc(q, k, v, out_ws, kl, scale)
        d_na = _desc(q, k, v, out_na, kl, scale)
        wsb = C.c_size_t(0)
        mlz_b200.check(L.mlzc_flash_attn_workspace_bytes(C.byref(d_ws), C.byref(wsb)))
        assert wsb.value > 0, "the case must exercise the split scratch"
        ws = torch.empty(wsb.value, dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream().cuda_stream
        mlz_b200.check(L.mlzc_flash_attn_dev(C.byref(d_ws), ws.data_ptr(), wsb.value, stream))
        mlz_b200.check(L.mlzc_flash_attn_dev_noalloc(C.byref(d_na), stream))
        torch.cuda.synchronize()
        a, b = out_ws.cpu().numpy(), out_na.cpu().numpy()
        assert np.isfinite(b).all()
        assert np.max(np.abs(a - b)) / max(np.max(np.abs(a)), 1e-30) <= 1e-3


def test_noalloc_batch_slices_reuse_the_scratch(dev):
    """More than 1024 sequences: one call launches its batch in slices of 1024, each slice's
    decode kernel rewriting the prefix table and partial records in the shared scratch
    that the previous slice's combine kernel read.  Kept small enough to fit the scratch
    (one kv head, D = 64, short sequences)."""
    import torch
    L = mlz_b200.lib()
    B, Hq, Hkv, Lmax, D = 1100, 4, 1, 40, 64
    q, k, v, kl = _inputs(dev, 950, B, Hq, Hkv, Lmax, D)
    scale = 1.0 / np.sqrt(D)
    out_ws = torch.full((B, Hq, 1, D), float("nan"), device=dev)
    out_na = torch.full((B, Hq, 1, D), float("nan"), device=dev)
    d_ws = _desc(q, k, v, out_ws, kl, scale)
    d_na = _desc(q, k, v, out_na, kl, scale)
    wsb = C.c_size_t(0)
    mlz_b200.check(L.mlzc_flash_attn_workspace_bytes(C.byref(d_ws), C.byref(wsb)))
    assert 0 < wsb.value <= 16 << 20
    ws = torch.empty(wsb.value, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        mlz_b200.check(L.mlzc_flash_attn_dev(C.byref(d_ws), ws.data_ptr(), wsb.value, stream))
        mlz_b200.check(L.mlzc_flash_attn_dev_noalloc(C.byref(d_na), stream))
        torch.cuda.synchronize()
        a, b = out_ws.cpu().numpy(), out_na.cpu().numpy()
        assert np.isfinite(b).all()
        assert np.max(np.abs(a - b)) / max(np.max(np.abs(a)), 1e-30) <= 1e-3


def test_noalloc_rejects_calls_beyond_its_scratch(dev):
    import torch
    # 2048 sequences (launched 1024 at a time) x 8 kv heads: 1024 x 8 segment records of
    # 8 rows x 130 floats plus one record per CTA is ~35 MB > 16 MiB.  Every declared
    # extent lies inside real memory (K/V broadcast over the batch), so nothing would read
    # out of bounds even if the call were not refused.
    B, Hq, Hkv, L, D = 2048, 32, 8, 16, 128
    q = torch.zeros((B, Hq, 1, D), device=dev)
    k = torch.zeros((1, Hkv, L, D), dtype=torch.float16, device=dev)
    out = torch.zeros((B, Hq, 1, D), device=dev)
    d = mlz_b200.make_fa_desc(q.data_ptr(), _nb(q, 4), k.data_ptr(), (2, 2 * D, 2 * D * L, 0), k.data_ptr(),
                              (2, 2 * D, 2 * D * L, 0), out.data_ptr(), _nb(out, 4), (B, Hq, 1, Hkv, L, D),
                              0.088)
    st = mlz_b200.lib().mlzc_flash_attn_dev_noalloc(C.byref(d), None)
    assert st == -4  # MLZC_ERR_NOMEM, before anything is launched
    assert "fixed scratch" in mlz_b200.last_error()


@pytest.mark.parametrize("kv_type", [mlz_b200.TYPE_Q8_0, mlz_b200.TYPE_Q5_1, mlz_b200.TYPE_F32])
def test_noalloc_quantised_and_f32_caches(dev, kv_type):
    """Quantised (Q8_0, Q5_1) and F32 KV caches take the same scratch for their split
    records: two consecutive calls of each equal the workspace entry point's result."""
    import torch
    L = mlz_b200.lib()
    B, Hq, Hkv, Lmax, D = 4, 8, 2, 1500, 128
    g = synth.rng(960 + kv_type)
    q = torch.from_numpy(synth.fa_inputs(g, B, Hq, Hkv, 1, D)[0]).to(dev)
    k = torch.from_numpy(synth.kv_quant_rows(g, (B, Hkv, Lmax), D, kv_type)).to(dev)
    v = torch.from_numpy(synth.kv_quant_rows(g, (B, Hkv, Lmax), D, kv_type)).to(dev)
    kl = torch.from_numpy(synth.kv_lengths(g, B, 1, Lmax)).to(dev)
    bb = mlz_b200.ops.KV_BLOCK_BYTES[kv_type]
    outs = [torch.full((B, Hq, 1, D), float("nan"), device=dev) for _ in range(2)]
    descs = [mlz_b200.make_fa_desc(q.data_ptr(), _nb(q, 4), k.data_ptr(), (bb,) + _nb(k, 1)[1:], v.data_ptr(),
                                   (bb,) + _nb(v, 1)[1:], o.data_ptr(), _nb(o, 4), (B, Hq, 1, Hkv, Lmax, D),
                                   1.0 / np.sqrt(D), kv_len_ptr=kl.data_ptr(), kv_type=kv_type) for o in outs]
    wsb = C.c_size_t(0)
    mlz_b200.check(L.mlzc_flash_attn_workspace_bytes(C.byref(descs[0]), C.byref(wsb)))
    assert 0 < wsb.value <= 16 << 20
    ws = torch.empty(wsb.value, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        mlz_b200.check(L.mlzc_flash_attn_dev(C.byref(descs[0]), ws.data_ptr(), wsb.value, stream))
        mlz_b200.check(L.mlzc_flash_attn_dev_noalloc(C.byref(descs[1]), stream))
        torch.cuda.synchronize()
        a, b = outs[0].cpu().numpy(), outs[1].cpu().numpy()
        assert np.isfinite(b).all()
        assert np.max(np.abs(a - b)) / max(np.max(np.abs(a)), 1e-30) <= 1e-3
