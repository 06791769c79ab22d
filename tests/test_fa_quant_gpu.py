"""GPU: flash-attention decode over a quantised KV cache (Q8_0, Q4_0, Q4_1, Q5_0, Q5_1 and
IQ4_NL K/V) and over an F32 one, the branches of flash_attn_dispatch at
src/simd/flash_attention.cpp:112-248, against the oracle, which dequantises every element
with the GGUF rule (pinned to the gguf decoder) and runs the attention in fp64.
Gate: max |o - o_oracle| / max |o_oracle| <= 1e-3."""
import ctypes as C

import numpy as np
import pytest

import mlz_b200
import oracle
from mlz_b200 import synth

TOL = 1e-3
pytestmark = pytest.mark.gpu
TYPES = [(mlz_b200.TYPE_Q8_0, "q8_0"), (mlz_b200.TYPE_Q4_0, "q4_0"), (mlz_b200.TYPE_Q4_1, "q4_1"),
         (mlz_b200.TYPE_Q5_0, "q5_0"), (mlz_b200.TYPE_Q5_1, "q5_1"), (mlz_b200.TYPE_IQ4_NL, "iq4_nl"),
         (mlz_b200.TYPE_F32, "f32")]


def _case(dev, seed, B, Hq, Hkv, L, D, kv_type, NQ=1, ragged=True):
    import torch
    g = synth.rng(seed)
    q = synth.fa_inputs(g, B, Hq, Hkv, 1, D, NQ=NQ)[0]
    k = synth.kv_quant_rows(g, (B, Hkv, L), D, kv_type)
    v = synth.kv_quant_rows(g, (B, Hkv, L), D, kv_type)
    kl = synth.kv_lengths(g, B, 1, L) if ragged else None
    return q, k, v, kl


@pytest.mark.parametrize("kv_type,name", TYPES)
@pytest.mark.parametrize("B,Hq,Hkv,L,D", [(3, 8, 2, 300, 128), (2, 4, 4, 129, 64), (2, 8, 1, 700, 256),
                                          (16, 32, 8, 1100, 128)])
def test_decode_parity(dev, kv_type, name, B, Hq, Hkv, L, D):
    import torch
    if kv_type == mlz_b200.TYPE_F32 and D == 256:
        pytest.skip("F32 K/V rows of 256 dims are declined (test_f32_head_dim_256_declined)")
    q, k, v, kl = _case(dev, 700 + B + L + D + kv_type, B, Hq, Hkv, L, D, kv_type)
    o = mlz_b200.flash_attn_dispatch_quant(torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev),
                                           torch.from_numpy(v).to(dev), 1 / np.sqrt(D), kv_type,
                                           kv_len=torch.from_numpy(kl).to(dev))
    torch.cuda.synchronize()
    want = oracle.flash_attn_q(q, k, v, 1 / np.sqrt(D), kv_type, kv_len=kl)
    got = o.cpu().numpy()
    assert np.isfinite(got).all()
    assert oracle.rel_err(got, want) <= TOL


@pytest.mark.parametrize("kv_type,name", TYPES)
def test_mask_softcap_alibi_rows_and_groups(dev, kv_type, name):
    """3 query positions x 16 heads per KV head = 48 rows (6 row groups), a mask with -inf
    entries, softcap and ALiBi together."""
    import torch
    B, Hq, Hkv, L, D, NQ = 2, 32, 2, 150, 64, 3
    q, k, v, _ = _case(dev, 777 + kv_type, B, Hq, Hkv, L, D, kv_type, NQ=NQ, ragged=False)
    q = q * 4
    g = synth.rng(778)
    mask = (g.standard_normal((NQ, L)) * 0.5).astype(np.float32)
    mask[:, ::7] = -np.inf
    o = mlz_b200.flash_attn_dispatch_quant(torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev),
                                           torch.from_numpy(v).to(dev), 0.125, kv_type,
                                           mask=torch.from_numpy(mask).to(dev), softcap=20.0, alibi=True)
    torch.cuda.synchronize()
    want = oracle.flash_attn_q(q, k, v, 0.125, kv_type, mask=mask, softcap=20.0,
                               mode=oracle.FA_MODE_SOFTCAP | oracle.FA_MODE_ALIBI)
    assert oracle.rel_err(o.cpu().numpy(), want) <= TOL


@pytest.mark.parametrize("kv_type,name", TYPES)
def test_llama_cpp_layout_ungrouped_heads_and_empty_sequence(dev, kv_type, name):
    """K/V in llama.cpp's [B][L][Hkv][row] order (strided rows), 6 query heads over 4 KV
    heads (not a multiple: one segment per query head), and a sequence with no keys."""
    import torch
    B, Hq, Hkv, L, D = 3, 6, 4, 90, 128
    q, k, v, kl = _case(dev, 790 + kv_type, B, Hq, Hkv, L, D, kv_type)
    kl[1] = 0
    kt = torch.from_numpy(np.ascontiguousarray(k.transpose(0, 2, 1, 3))).to(dev).permute(0, 2, 1, 3)
    vt = torch.from_numpy(np.ascontiguousarray(v.transpose(0, 2, 1, 3))).to(dev).permute(0, 2, 1, 3)
    o = mlz_b200.flash_attn_dispatch_quant(torch.from_numpy(q).to(dev), kt, vt, 1 / np.sqrt(D), kv_type,
                                           kv_len=torch.from_numpy(kl).to(dev))
    torch.cuda.synchronize()
    want = oracle.flash_attn_q(q, k, v, 1 / np.sqrt(D), kv_type, kv_len=kl)
    got = o.cpu().numpy()
    assert (got[1] == 0).all()
    assert oracle.rel_err(got, want) <= TOL


def test_q8_0_through_hook_with_host_buffers(dev):
    B, Hq, Hkv, L, D = 2, 8, 2, 200, 128
    q, k, v, kl = _case(dev, 800, B, Hq, Hkv, L, D, mlz_b200.TYPE_Q8_0)
    out = np.zeros((B, Hq, 1, D), dtype=np.float32)
    from mlz_b200.ops import _nb
    desc = mlz_b200.make_fa_desc(q.ctypes.data, _nb(q, 4), k.ctypes.data, (34,) + _nb(k, 1)[1:], v.ctypes.data,
                                 (34,) + _nb(v, 1)[1:], out.ctypes.data, _nb(out, 4), (B, Hq, 1, Hkv, L, D),
                                 1 / np.sqrt(D), kv_len_ptr=kl.ctypes.data, kv_type=mlz_b200.TYPE_Q8_0)
    assert mlz_b200.ggml_simd_try_flash_attn(desc, 0, 1) == 1
    want = oracle.flash_attn_q(q, k, v, 1 / np.sqrt(D), mlz_b200.TYPE_Q8_0, kv_len=kl)
    assert oracle.rel_err(out, want) <= TOL


def test_quant_gate_rejects_mixed_types_and_misaligned_rows(dev):
    B, Hq, Hkv, L, D = 1, 4, 1, 16, 64
    d = mlz_b200.make_fa_desc(16, (4, 256, 256, 1024), 16, (34, 68, 68 * L, 68 * L), 16, (34, 68, 68 * L, 68 * L),
                              16, (4, 256, 256, 1024), (B, Hq, 1, Hkv, L, D), 0.1, kv_type=mlz_b200.TYPE_Q8_0)
    out = C.c_size_t(0)
    d.v_type = mlz_b200.TYPE_Q4_0
    assert mlz_b200.lib().mlzc_flash_attn_workspace_bytes(C.byref(d), C.byref(out)) == -2   # mixed K/V types
    d.v_type = mlz_b200.TYPE_Q8_0
    d.k_nb[1] = 70
    assert mlz_b200.lib().mlzc_flash_attn_workspace_bytes(C.byref(d), C.byref(out)) == -1   # row stride % 4


@pytest.mark.parametrize("kv_type,name", TYPES[2:])
def test_new_types_through_hook_with_host_buffers(dev, kv_type, name):
    """Q4_1 / Q5_0 / Q5_1 / IQ4_NL / F32 caches through the hook body (host buffers, block
    (or element) size nb[0]), GQA 4:1 with ragged lengths."""
    B, Hq, Hkv, L, D = 2, 8, 2, 333, 128
    q, k, v, kl = _case(dev, 810 + kv_type, B, Hq, Hkv, L, D, kv_type)
    bb = mlz_b200.ops.KV_BLOCK_BYTES[kv_type]
    out = np.zeros((B, Hq, 1, D), dtype=np.float32)
    from mlz_b200.ops import _nb
    desc = mlz_b200.make_fa_desc(q.ctypes.data, _nb(q, 4), k.ctypes.data, (bb,) + _nb(k, 1)[1:], v.ctypes.data,
                                 (bb,) + _nb(v, 1)[1:], out.ctypes.data, _nb(out, 4), (B, Hq, 1, Hkv, L, D),
                                 1 / np.sqrt(D), kv_len_ptr=kl.ctypes.data, kv_type=kv_type)
    assert mlz_b200.ggml_simd_try_flash_attn(desc, 0, 1) == 1
    want = oracle.flash_attn_q(q, k, v, 1 / np.sqrt(D), kv_type, kv_len=kl)
    assert oracle.rel_err(out, want) <= TOL


@pytest.mark.parametrize("kv_type,name", TYPES[2:6])
def test_new_types_large_minimum_and_all_fifth_bits(dev, kv_type, name):
    """Blocks whose minimum m dominates the values (Q4_1 / Q5_1: m = -40 d), every fifth bit
    set (Q5_x: qh = 0xFFFFFFFF) and every code-book entry (IQ4_NL): the minimum, fifth-bit
    and table paths of both the score and the value side."""
    import torch
    B, Hq, Hkv, L, D = 2, 4, 1, 200, 64
    q, k, v, kl = _case(dev, 830 + kv_type, B, Hq, Hkv, L, D, kv_type)
    bb = oracle.KV_BLOCK[kv_type][0]
    for rows in (k, v):
        r = rows.reshape(B, Hkv, L, D // 32, bb)
        d = r[..., 0:2].copy().view(np.float16).astype(np.float32)
        if kv_type in (mlz_b200.TYPE_Q4_1, mlz_b200.TYPE_Q5_1):
            r[..., 2:4] = (-40.0 * d).astype(np.float16).view(np.uint8)
        if kv_type in (mlz_b200.TYPE_Q5_0, mlz_b200.TYPE_Q5_1):
            off = 2 if kv_type == mlz_b200.TYPE_Q5_0 else 4
            r[..., off:off + 4] = 0xFF
        if kv_type == mlz_b200.TYPE_IQ4_NL:
            r[..., 2:] = (np.arange(16, dtype=np.uint8) * 17)[None, None, None, None, :]   # byte i = (i, i)
    o = mlz_b200.flash_attn_dispatch_quant(torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev),
                                           torch.from_numpy(v).to(dev), 1 / np.sqrt(D), kv_type,
                                           kv_len=torch.from_numpy(kl).to(dev))
    torch.cuda.synchronize()
    want = oracle.flash_attn_q(q, k, v, 1 / np.sqrt(D), kv_type, kv_len=kl)
    assert oracle.rel_err(o.cpu().numpy(), want) <= TOL


def test_f32_head_dim_256_declined(dev):
    """F32 rows of 256 dims do not fit the kernel's two-stage ring: the gate refuses them
    (MLZC_ERR_UNSUPPORTED) and the hook returns 0, so upstream computes them."""
    B, Hq, Hkv, L, D = 1, 4, 1, 16, 256
    d = mlz_b200.make_fa_desc(16, (4, 1024, 1024, 4096), 16, (4, 1024, 1024 * L, 1024 * L), 16,
                              (4, 1024, 1024 * L, 1024 * L), 16, (4, 1024, 1024, 4096), (B, Hq, 1, Hkv, L, D), 0.1,
                              kv_type=mlz_b200.TYPE_F32)
    out = C.c_size_t(0)
    assert mlz_b200.lib().mlzc_flash_attn_workspace_bytes(C.byref(d), C.byref(out)) == -2


def test_f32_large_values_keep_fp32_accuracy(dev):
    """F32 keys and values with a wide dynamic range (|k| up to ~300, values carrying bits
    below f16's precision): the hi + lo split keeps the scores and the output far below f16
    rounding error against the fp64 oracle (1e-4, ten times inside the gate; f16-rounded K
    and V alone would miss it)."""
    import torch
    B, Hq, Hkv, L, D = 2, 8, 2, 257, 128
    g = synth.rng(850)
    q = synth.fa_inputs(g, B, Hq, Hkv, 1, D)[0]
    kf = (g.standard_normal((B, Hkv, L, D)) * np.exp(g.uniform(-4, 4, (B, Hkv, L, 1))) / np.sqrt(D)).astype(np.float32)
    vf = (g.standard_normal((B, Hkv, L, D)) * (1 + 1e-4 * g.standard_normal((B, Hkv, L, D)))).astype(np.float32)
    k, v = kf.view(np.uint8), vf.view(np.uint8)
    kl = np.array([257, 100], dtype=np.int32)
    o = mlz_b200.flash_attn_dispatch_quant(torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev),
                                           torch.from_numpy(v).to(dev), 1 / np.sqrt(D), mlz_b200.TYPE_F32,
                                           kv_len=torch.from_numpy(kl).to(dev))
    torch.cuda.synchronize()
    want = oracle.flash_attn_q(q, k, v, 1 / np.sqrt(D), mlz_b200.TYPE_F32, kv_len=kl)
    assert oracle.rel_err(o.cpu().numpy(), want) <= 1e-4


@pytest.mark.parametrize("case", ["gqa4_l70_d64", "gqa4_l65_d128_mask", "gqa2_l64_d64_softcap",
                                  "gqa4_l33_d128_alibi", "gqa4_nq3_l40_d64"])
def test_f32_reference_fixtures(dev, golden, case):
    """F32 K/V against the reference's own flash_attn_quantized outputs (its F32 value
    branch; mask, softcap, ALiBi, n_q > 1), within 1e-4."""
    import torch
    f = golden("fa_f32_reference.npz")
    q, k, v = f[case + "__q"], f[case + "__k"], f[case + "__v"]
    softcap, alibi, scale = f[case + "__meta"]
    mask = f[case + "__mask"] if (case + "__mask") in f.files else None
    o = mlz_b200.flash_attn_dispatch_quant(torch.from_numpy(q).to(dev), torch.from_numpy(k.view(np.uint8)).to(dev),
                                           torch.from_numpy(v.view(np.uint8)).to(dev), float(scale),
                                           mlz_b200.TYPE_F32,
                                           mask=torch.from_numpy(mask).to(dev) if mask is not None else None,
                                           softcap=float(softcap), alibi=bool(alibi))
    torch.cuda.synchronize()
    assert oracle.rel_err(o.cpu().numpy(), f[case + "__out"]) <= 1e-4
