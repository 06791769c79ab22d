"""GPU parity of flash-attention decode against the fp64 oracle (itself pinned to the
reference's own flash_attn_quantized).  Gate: max abs error / max |o| <= 1e-3."""
import numpy as np
import pytest

import mlz_b200
import oracle
from mlz_b200 import synth

TOL = 1e-3
pytestmark = pytest.mark.gpu


def _run(dev, q, k, v, scale, kv_len=None, mask=None, softcap=0.0, alibi=False, layout="bhld"):
    import torch
    qd = torch.from_numpy(q).to(dev)
    if layout == "blhd":  # llama.cpp cache layout: token rows of all heads interleaved
        kd = torch.from_numpy(np.ascontiguousarray(k.transpose(0, 2, 1, 3))).to(dev).transpose(1, 2)
        vd = torch.from_numpy(np.ascontiguousarray(v.transpose(0, 2, 1, 3))).to(dev).transpose(1, 2)
    else:
        kd = torch.from_numpy(k).to(dev)
        vd = torch.from_numpy(v).to(dev)
    kl = torch.from_numpy(kv_len).to(dev) if kv_len is not None else None
    md = torch.from_numpy(mask).to(dev) if mask is not None else None
    out = mlz_b200.flash_attn_dispatch(qd, kd, vd, scale, kv_len=kl, mask=md, softcap=softcap, alibi=alibi)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_gqa_decode_ragged_batch(dev):
    """32 query heads, 8 KV heads, D = 128, F16 KV, 16 sequences, L ~ U{512..8192}."""
    g = synth.rng(synth.seed_for(4, 16))
    B, Hq, Hkv, D = 16, 32, 8, 128
    kv_len = synth.kv_lengths(g, B, 512, 8192)
    L = int(kv_len.max())
    q, k, v = synth.fa_inputs(g, B, Hq, Hkv, L, D)
    scale = 1.0 / np.sqrt(D)
    got = _run(dev, q, k, v, scale, kv_len=kv_len)
    want = oracle.flash_attn(q, k.view(np.uint16), v.view(np.uint16), scale, kv_len=kv_len)
    assert oracle.rel_err(got, want) <= TOL


@pytest.mark.parametrize("L", [1, 63, 64, 65, 255, 256, 257, 1000])
def test_kv_lengths(dev, L):
    g = synth.rng(400 + L)
    q, k, v = synth.fa_inputs(g, 2, 8, 2, L, 128)
    q *= 8.0  # sharper softmax than the benchmark's
    got = _run(dev, q, k, v, 0.0883883)
    want = oracle.flash_attn(q, k.view(np.uint16), v.view(np.uint16), 0.0883883)
    assert oracle.rel_err(got, want) <= TOL


def test_zero_length_rows_are_zero(dev):
    g = synth.rng(41)
    q, k, v = synth.fa_inputs(g, 3, 4, 1, 300, 64)
    kv_len = np.array([0, 300, 1], dtype=np.int32)
    got = _run(dev, q, k, v, 0.125, kv_len=kv_len)
    assert (got[0] == 0).all()
    want = oracle.flash_attn(q, k.view(np.uint16), v.view(np.uint16), 0.125, kv_len=kv_len)
    assert oracle.rel_err(got, want) <= TOL


@pytest.mark.parametrize("case", ["gqa4_l70_d64", "mha_l1_d128", "gqa4_l65_d128_mask",
                                  "gqa2_l64_d64_softcap", "gqa4_l63_d64_alibi", "gqa4_nq3_l40_d64"])
def test_reference_fixtures(dev, golden, case):
    """The reference's own flash_attn_quantized outputs (mask, softcap, ALiBi, n_q > 1)."""
    f = golden("fa_reference.npz")
    q, k, v = f[case + "__q"], f[case + "__k"], f[case + "__v"]
    softcap, alibi, scale = f[case + "__meta"]
    mask = f[case + "__mask"] if (case + "__mask") in f.files else None
    got = _run(dev, q, k.view(np.float16), v.view(np.float16), float(scale), mask=mask,
               softcap=float(softcap), alibi=bool(alibi))
    assert oracle.rel_err(got, f[case + "__out"]) <= TOL


@pytest.mark.parametrize("D,Hq,Hkv,NQ", [(64, 4, 4, 1), (256, 8, 2, 1), (128, 6, 4, 1), (128, 16, 2, 2), (64, 3, 1, 5)])
def test_head_layouts(dev, D, Hq, Hkv, NQ):
    g = synth.rng(500 + D + Hq + Hkv + NQ)
    q, k, v = synth.fa_inputs(g, 2, Hq, Hkv, 700, D, NQ=NQ)
    kv_len = np.array([700, 333], dtype=np.int32)
    got = _run(dev, q, k, v, 1.0 / np.sqrt(D), kv_len=kv_len)
    want = oracle.flash_attn(q, k.view(np.uint16), v.view(np.uint16), 1.0 / np.sqrt(D), kv_len=kv_len)
    assert oracle.rel_err(got, want) <= TOL


def test_llama_cpp_cache_layout(dev):
    """K/V with token rows of all heads interleaved ([B, L, Hkv, D] memory order)."""
    g = synth.rng(77)
    q, k, v = synth.fa_inputs(g, 2, 8, 2, 600, 128)
    got = _run(dev, q, k, v, 0.0883883, layout="blhd")
    want = oracle.flash_attn(q, k.view(np.uint16), v.view(np.uint16), 0.0883883)
    assert oracle.rel_err(got, want) <= TOL


def test_hook_flash_attn_host_buffers(dev):
    g = synth.rng(88)
    q, k, v = synth.fa_inputs(g, 2, 8, 2, 300, 64)
    out = np.full((2, 8, 1, 64), np.nan, dtype=np.float32)
    kb, vb = k.view(np.uint16), v.view(np.uint16)
    nb = lambda a: tuple(a.strides[::-1])
    desc = mlz_b200.make_fa_desc(q.ctypes.data, nb(q), kb.ctypes.data, nb(kb), vb.ctypes.data, nb(vb),
                                 out.ctypes.data, nb(out), (2, 8, 1, 2, 300, 64), 0.125)
    assert mlz_b200.ggml_simd_try_flash_attn(desc, 0, 1) == 1
    want = oracle.flash_attn(q, kb, vb, 0.125)
    assert oracle.rel_err(out, want) <= TOL


def test_kv_shared_across_sequences(dev):
    """One K/V (batch stride 0) serves every sequence, each with its own length."""
    import torch
    from mlz_b200.ops import _nb
    g = synth.rng(91)
    B, Hq, Hkv, L, D = 6, 16, 4, 900, 128
    q, k1, v1 = synth.fa_inputs(g, B, Hq, Hkv, L, D)
    k1, v1 = k1[:1], v1[:1]
    kv_len = synth.kv_lengths(g, B, 1, L)
    qd = torch.from_numpy(q).to(dev)
    kd = torch.from_numpy(k1).to(dev)
    vd = torch.from_numpy(v1).to(dev)
    kl = torch.from_numpy(kv_len).to(dev)
    out = torch.full((B, Hq, 1, D), float("nan"), device=dev)
    knb = (2, 2 * D, 2 * D * L, 0)
    desc = mlz_b200.make_fa_desc(qd.data_ptr(), _nb(qd, 4), kd.data_ptr(), knb, vd.data_ptr(), knb,
                                 out.data_ptr(), _nb(out, 4), (B, Hq, 1, Hkv, L, D), 0.088,
                                 kv_len_ptr=kl.data_ptr())
    import ctypes as C
    wsb = mlz_b200.ops.flash_attn_workspace_bytes(desc)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    mlz_b200.check(mlz_b200.lib().mlzc_flash_attn_dev(C.byref(desc), ws.data_ptr(), wsb,
                                                      torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    kb = np.broadcast_to(k1, (B, Hkv, L, D))
    vb = np.broadcast_to(v1, (B, Hkv, L, D))
    want = oracle.flash_attn(q, np.ascontiguousarray(kb).view(np.uint16), np.ascontiguousarray(vb).view(np.uint16),
                             0.088, kv_len=kv_len)
    assert oracle.rel_err(out.cpu().numpy(), want) <= TOL


def test_cache_rows_past_kv_len_may_hold_nan(dev):
    """Unused cache rows (past each sequence's length) hold NaN bit patterns; they must not
    reach the output (P = 0 there, and 0 * NaN would)."""
    g = synth.rng(92)
    B, Hq, Hkv, L, D = 3, 8, 2, 700, 64
    q, k, v = synth.fa_inputs(g, B, Hq, Hkv, L, D)
    kv_len = np.array([1, 333, 650], dtype=np.int32)
    kn, vn = k.copy(), v.copy()
    for b, n in enumerate(kv_len):
        kn[b, :, n:, :] = np.float16(np.nan)
        vn[b, :, n:, :] = np.float16(np.nan)
    got = _run(dev, q, kn, vn, 0.125, kv_len=kv_len)
    want = oracle.flash_attn(q, k.view(np.uint16), v.view(np.uint16), 0.125, kv_len=kv_len)
    assert np.isfinite(got).all()
    assert oracle.rel_err(got, want) <= TOL
