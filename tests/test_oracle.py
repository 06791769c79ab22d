"""CPU: the oracle pinned against the golden fixtures and the reference's own code."""
import numpy as np
import pytest

import oracle
from mlz_b200 import synth


def test_f16_widening_all_patterns():
    h = np.arange(65536, dtype=np.uint16)
    got = oracle.f16_bits_to_f32(h)
    want = h.view(np.float16).astype(np.float32)
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    assert same.all()


def test_f16_narrowing_matches_ieee_rne():
    g = np.random.default_rng(0)
    x = np.concatenate([g.standard_normal(1 << 16).astype(np.float32) * s
                        for s in (1e-8, 3e-6, 1e-3, 1.0, 300.0, 6e4)])
    edge = np.array([65504, 65519.99, 65520, -65520, np.inf, -np.inf, 2 ** -24, 2 ** -25,
                     2 ** -25 * 1.0001, 3 * 2 ** -26, 0.0, -0.0], dtype=np.float32)
    x = np.concatenate([x, edge])
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert (oracle.f32_to_f16_bits(x) == want).all()


def test_f16_mul_mat_matches_reference_simd_matmul_f16(golden):
    """The oracle's F16 product (f16 weights x activations rounded to f16, accumulated in
    fp64), rounded to f16, equals bit for bit the reference's own F16 GEMM
    simd_matmul_f16 (src/simd/simd_matmul.cpp:428-480: f16 operands, fp32 accumulation,
    f16 result) on every fixture case."""
    f = golden("matmul_f16_reference.npz")
    n = len([k for k in f.files if k.startswith("a")])
    assert n >= 12
    for i in range(n):
        a, b, c = f[f"a{i}"], f[f"b{i}"], f[f"c{i}"]
        x = b.T.view(np.float16).astype(np.float32)            # (N, K): ggml columns of X
        y = oracle.mul_mat_f16(a, x)                           # (N, M), fp64
        got = np.asarray(y, dtype=np.float64).astype(np.float16).view(np.uint16)
        assert np.array_equal(got, c.T), f"case {i}: {a.shape} x {b.shape}"


def test_q4k_dequant_matches_gguf_decoder(golden):
    f = golden("q4k_gguf.npz")
    got = oracle.q4k_dequant(f["blocks"], int(f["K"]))
    want = f["dequant"]
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    assert same.all()


def test_q6k_dequant_matches_gguf_decoder(golden):
    f = golden("q6k_gguf.npz")
    got = oracle.q6k_dequant(f["blocks"], int(f["K"]))
    want = f["dequant"]
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    assert same.all()


def test_q6k_known_answer():
    # ql low nibbles 5, high nibbles 1, qh all 2 (bits 10 per element), every scale 3,
    # d = 0.25: low-nibble elements q = 5 + 32 - 32 = 5, high-nibble q = 1 -> known row dot
    K = 256
    blk = np.zeros((1, 210), dtype=np.uint8)
    blk[0, :128] = 0x15
    blk[0, 128:192] = 0xAA
    blk[0, 192:208] = 3
    blk[0, 208:210] = np.array([0.25], dtype=np.float16).view(np.uint8)
    w = oracle.q6k_dequant(blk, K)[0]
    p = np.arange(256)
    low = ((p % 128) // 32) < 2          # elements k = 0, 1 read the low nibble
    assert np.all(w[low] == 0.75 * 5) and np.all(w[~low] == 0.75 * 1)
    x = np.random.default_rng(2).standard_normal((1, K)).astype(np.float32)
    np.testing.assert_allclose(oracle.mul_mat_q6k(blk, x)[0, 0], float(np.dot(w.astype(np.float64), x[0])),
                               rtol=1e-12)


@pytest.mark.parametrize("name,kv_type", [("q8_0", 8), ("q4_0", 2), ("q4_1", 3), ("q5_0", 6), ("q5_1", 7),
                                           ("iq4_nl", 20)])
def test_kv_dequant_matches_gguf_decoder(golden, name, kv_type):
    """The quantised KV-cache element rule of the oracle (Q8_0, Q4_0, Q4_1, Q5_0, Q5_1,
    IQ4_NL) equals the gguf decoder bit for bit on blocks with edge scales (and, for Q4_1 /
    Q5_1, edge block minima)."""
    f = golden("kv_gguf.npz")
    got = oracle.kv_dequant(f[name + "_rows"], 128, kv_type)
    want = f[name + "_dequant"]
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    assert same.all()


def test_fa_quant_oracle_equals_f16_oracle_on_exact_values():
    """Q8_0 blocks whose values are exact in f16 (d a power of two, small q): the quantised
    attention oracle equals the F16 one on the same values."""
    g = synth.rng(44)
    B, Hq, Hkv, L, D = 2, 8, 2, 70, 64
    q = synth.fa_inputs(g, B, Hq, Hkv, L, D)[0]
    kq = synth.kv_quant_rows(g, (B, Hkv, L), D, 8)
    vq = synth.kv_quant_rows(g, (B, Hkv, L), D, 8)
    for rows in (kq, vq):
        r = rows.reshape(B, Hkv, L, D // 32, 34)
        r[..., 0:2] = np.array([2.0 ** -7], dtype=np.float16).view(np.uint8)
        r[..., 2:] = (r[..., 2:].view(np.int8) // 16).view(np.uint8)
    kf = oracle.kv_dequant(kq, D, 8).astype(np.float16)
    vf = oracle.kv_dequant(vq, D, 8).astype(np.float16)
    kl = np.array([70, 33], dtype=np.int32)
    a = oracle.flash_attn_q(q, kq, vq, 0.125, 8, kv_len=kl)
    b = oracle.flash_attn(q, kf.view(np.uint16), vf.view(np.uint16), 0.125, kv_len=kl)
    assert np.array_equal(a, b)


def test_q4k_known_answer():
    # every nibble 1, sc = 1, m = 0, d = 0.5, dmin arbitrary: row dot = d * sum(x)
    K = 512
    blk = np.zeros((1, 2, 144), dtype=np.uint8)
    blk[0, :, 0:2] = np.array([0.5], dtype=np.float16).view(np.uint8)
    blk[0, :, 2:4] = np.array([0.25], dtype=np.float16).view(np.uint8)
    blk[0, :, 4:8] = 1        # sc of sub-blocks 0..3
    blk[0, :, 8:12] = 0       # m of sub-blocks 0..3
    blk[0, :, 12:16] = 0x01   # sub-blocks 4..7: sc low nibble 1, m high nibble 0
    blk[0, :, 16:] = 0x11
    blk = blk.reshape(1, -1)
    x = np.random.default_rng(1).standard_normal((2, K)).astype(np.float32)
    y = oracle.mul_mat_q4k(blk, x)
    np.testing.assert_allclose(y[:, 0], 0.5 * x.astype(np.float64).sum(axis=1), rtol=1e-12)
    w = oracle.q4k_dequant(blk, K)
    assert np.all(w == 0.5)


def test_q4k_q8k_dot_tracks_dequant_product():
    """The reference's Q8_K-activation dot (integer sub-block dots) stays within the
    activation-quantisation error of the dequantised-F32 product."""
    g = synth.rng(5)
    K = 1024
    w = synth.q4k_blocks(g, 8, K)
    x = synth.f32_acts(g, 1, K)
    exact = oracle.mul_mat_q4k(w, x)[0]
    q8 = oracle.quantize_q8k(x[0])
    approx = np.array([oracle.vec_dot_q4k_q8k(w[m], q8, K) for m in range(8)])
    assert oracle.rel_err(approx, exact) < 2e-2


def test_q8k_quantize_layout():
    x = np.linspace(-3, 3, 256, dtype=np.float32)
    q = oracle.quantize_q8k(x)
    d = q[:4].view(np.float32)[0]
    assert abs(d - 3.0 / 127.0) < 1e-7
    qs = q[4:260].view(np.int8)
    assert qs[0] == -127 and qs[-1] == 127
    bs = q[260:292].view(np.int16)
    assert (bs == qs.reshape(16, 16).astype(np.int32).sum(axis=1)).all()


@pytest.mark.parametrize("case", ["gqa4_l70_d64", "mha_l1_d128", "gqa4_l65_d128_mask",
                                  "gqa2_l64_d64_softcap", "gqa4_l63_d64_alibi", "gqa4_nq3_l40_d64"])
def test_fa_oracle_matches_reference_outputs(golden, case):
    f = golden("fa_reference.npz")
    q, k, v = f[case + "__q"], f[case + "__k"], f[case + "__v"]
    softcap, alibi, scale = f[case + "__meta"]
    mask = f[case + "__mask"] if (case + "__mask") in f.files else None
    mode = (oracle.FA_MODE_SOFTCAP if softcap else 0) | (oracle.FA_MODE_ALIBI if alibi else 0)
    got = oracle.flash_attn(q, k, v, float(scale), mask=mask, softcap=float(softcap), mode=mode)
    assert oracle.rel_err(f[case + "__out"], got) < 2e-5


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")
def test_reference_library_untouched_stubs():
    g = np.random.default_rng(3)
    q = g.standard_normal((1, 4, 1, 64)).astype(np.float32)
    k = g.standard_normal((1, 2, 10, 64)).astype(np.float16).view(np.uint16)
    out = oracle.ref_flash_attn(q, k, k, 0.125)
    assert np.isfinite(out).all()
    assert oracle.ref_stub_hits() == 0


def test_matmul_oracle_matches_reference_scalar_path(golden):
    f = golden("matmul_reference.npz")
    i = 0
    while f"a{i}" in f.files:
        a, b, c = f[f"a{i}"], f[f"b{i}"], f[f"c{i}"]
        # row-major C = A.B is ggml's mul_mat with W = A, X = B^T, Y = C^T
        y = oracle.mul_mat_f32(a, np.ascontiguousarray(b.T))
        assert oracle.rel_err(c, y.T) < 1e-6
        i += 1


def test_mul_mat_f16_rounds_activations():
    g = synth.rng(2)
    w = synth.f16_weights(g, 16, 96)
    x = synth.f32_acts(g, 3, 96)
    yr = oracle.mul_mat_f16(w.view(np.uint16), x, round_x=True)
    xr = x.astype(np.float16).astype(np.float64)
    np.testing.assert_allclose(yr, xr @ w.astype(np.float64).T, rtol=1e-12, atol=1e-15)


def test_cpu_baselines_agree_with_oracle():
    g = synth.rng(9)
    w = synth.f16_weights(g, 70, 256)
    x = synth.f32_acts(g, 5, 256)
    want = oracle.mul_mat_f16(w.view(np.uint16), x)
    got = oracle.base_mul_mat_f16(w, x, nth=3)
    assert oracle.rel_err(got, want) < 1e-5
    wq = synth.q4k_blocks(g, 33, 512)
    xq = synth.f32_acts(g, 2, 512)
    got = oracle.base_mul_mat_q4k(wq, xq, nth=4)
    assert oracle.rel_err(got, oracle.mul_mat_q4k(wq, xq)) < 2e-2
    q, k, v = synth.fa_inputs(g, 2, 8, 2, 150, 64)
    kl = np.array([150, 37], dtype=np.int32)
    got = oracle.base_flash_attn(q, k, v, 0.125, kv_len=kl, nth=3)
    want = oracle.flash_attn(q, k, v, 0.125, kv_len=kl)
    assert oracle.rel_err(got, want) < 1e-5


@pytest.mark.parametrize("kv_type", [8, 2, 3, 6, 7, 20, 0])
def test_fa_quant_oracle_equals_numpy_attention_on_decoded_rows(kv_type):
    """The quantised-KV attention oracle equals a plain numpy fp64 attention over the rows
    decoded by kv_dequant (the gguf-pinned rule), for every KV-cache type (and F32 rows),
    GQA and ragged."""
    g = synth.rng(45 + kv_type)
    B, Hq, Hkv, L, D = 2, 4, 2, 37, 64
    q = synth.fa_inputs(g, B, Hq, Hkv, L, D)[0]
    k = synth.kv_quant_rows(g, (B, Hkv, L), D, kv_type)
    v = synth.kv_quant_rows(g, (B, Hkv, L), D, kv_type)
    kl = np.array([37, 20], dtype=np.int32)
    got = oracle.flash_attn_q(q, k, v, 0.125, kv_type, kv_len=kl)
    kf = oracle.kv_dequant(k, D, kv_type).astype(np.float64)
    vf = oracle.kv_dequant(v, D, kv_type).astype(np.float64)
    for b in range(B):
        for h in range(Hq):
            hk = h * Hkv // Hq
            s = kf[b, hk, :kl[b]] @ q[b, h, 0].astype(np.float64) * 0.125
            p = np.exp(s - s.max())
            want = (p @ vf[b, hk, :kl[b]]) / p.sum()
            np.testing.assert_allclose(got[b, h, 0], want, rtol=1e-6, atol=1e-9)


@pytest.mark.parametrize("case", ["gqa4_l70_d64", "gqa4_l65_d128_mask", "gqa2_l64_d64_softcap",
                                  "gqa4_l33_d128_alibi", "gqa4_nq3_l40_d64"])
def test_fa_oracle_f32_kv_matches_reference_outputs(golden, case):
    """F32 K/V: the oracle's attention (kv_type 0) equals the reference's own
    flash_attn_quantized run on the same f32 rows (its F32 value branch), to f32 rounding."""
    f = golden("fa_f32_reference.npz")
    q, k, v = f[case + "__q"], f[case + "__k"], f[case + "__v"]
    softcap, alibi, scale = f[case + "__meta"]
    mask = f[case + "__mask"] if (case + "__mask") in f.files else None
    mode = (oracle.FA_MODE_SOFTCAP if softcap else 0) | (oracle.FA_MODE_ALIBI if alibi else 0)
    got = oracle.flash_attn_q(q, k.view(np.uint8), v.view(np.uint8), float(scale), 0, mask=mask,
                              softcap=float(softcap), mode=mode)
    assert oracle.rel_err(f[case + "__out"], got) < 2e-5


def test_q8k_oracle_matches_reference_quantiser(golden):
    """The oracle's Q8_K restatement equals the reference's own quantize_row_q8_k_reference
    (src/simd/ggml_simd_hook.cpp:109-148, compiled from the reference tree) bit for bit,
    edge blocks included (zeros, tiny and huge values, rounding ties)."""
    f = golden("q8k_reference.npz")
    got = np.stack([oracle.quantize_q8k(r) for r in f["x"]]).view(np.uint8).reshape(f["q8k"].shape)
    assert np.array_equal(got, f["q8k"])


def test_f32_oracle_matches_reference_hook(golden):
    """One-column F32-weight nodes through the reference's own ggml_simd_try_mul_mat (with 1
    and 3 thread indices): the oracle's F32 product agrees to fp32 rounding; the reference
    declines F16 weights (returns 0) -- this library's hook takes them (a superset)."""
    f = golden("hook_reference.npz")
    for i in range(3):
        w, x = f[f"f32_{i}__w"], f[f"f32_{i}__x"]
        want = oracle.mul_mat_f32(w, x)
        for nth in (1, 3):
            assert oracle.rel_err(f[f"f32_{i}_nth{nth}__y"], want) < 1e-6
    assert int(f["f16__handled"][0]) == 0
