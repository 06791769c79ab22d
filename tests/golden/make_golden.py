"""Generates the golden fixtures of tests/golden/ (run in a checkout that has the
reference tree and the gguf package; the fixtures are committed, this script is how
they were made).

* q4k_gguf.npz      -- Q4_K super-blocks and their dequantisation by the gguf 0.19.0
                       Python decoder (gguf.quants.dequantize), the published GGUF
                       algorithm the reference's Q4_K kernels implement.
* q6k_gguf.npz      -- Q6_K super-blocks and their dequantisation by the same gguf decoder.
* kv_gguf.npz       -- Q8_0, Q4_0, Q4_1, Q5_0, Q5_1 and IQ4_NL blocks (the quantised
                       KV-cache formats) and their dequantisation by the same gguf decoder.
* fa_reference.npz  -- flash-attention decode cases and the outputs of the reference's
                       own flash_attn_quantized (src/simd/flash_attention.cpp:291-410),
                       compiled from source into oracle/_ref, fed F16 K/V and an f32 query.
* fa_f32_reference.npz -- the same for F32 K/V (the reference's F32 value branch, fed
                       through an f32 x f32 dot).
* q8k_reference.npz  -- F32 rows and their Q8_K blocks from the reference's own
                       quantize_row_q8_k_reference (src/simd/ggml_simd_hook.cpp:109-148),
                       the hook compiled in place against minimal ggml declarations.
* hook_reference.npz -- one-column MUL_MAT nodes through the reference's own hook,
                       ggml_simd_try_mul_mat (its F32 branch; F16 weights are declined).
* matmul_reference.npz -- tiny row-major matmuls through the reference's simd_matmul_f32
                       scalar path (src/simd/simd_matmul.cpp:196-223).
* matmul_f16_reference.npz -- tiny F16 matmuls through the reference's own F16 GEMM,
                       simd_matmul_f16 (src/simd/simd_matmul.cpp:428-480): f16 operands,
                       fp32 accumulation, f16 result.  A is an F16 weight block (M x K),
                       B the activations already rounded to f16 (K x N).

Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402


def q4k_fixture() -> None:
    from gguf import GGMLQuantizationType, quants
    g = np.random.Generator(np.random.PCG64(7))
    M, K = 6, 512
    nb = K // 256
    blk = g.integers(0, 256, size=(M, nb, 144), dtype=np.uint8)
    d = np.abs(g.standard_normal((M, nb, 2)) * 0.01).astype(np.float16)
    # edge values for d/dmin: zero, a subnormal, the largest finite half, negative
    d[0, 0, 0] = np.float16(0.0)
    d[1, 0, 1] = np.float16(6e-8)
    d[2, 1, 0] = np.float16(65504.0)
    d[3, 1, 1] = np.float16(-0.5)
    blk[:, :, 0:4] = d.view(np.uint8).reshape(M, nb, 4)
    blk[4, 0, 4:16] = 0xFF   # all scale/min bits set
    blk[5, 1, 4:16] = 0x00   # all zero scales
    blk = blk.reshape(M, nb * 144)
    deq = quants.dequantize(blk, GGMLQuantizationType.Q4_K).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "q4k_gguf.npz"), blocks=blk, dequant=deq, K=K)


def q6k_fixture() -> None:
    from gguf import GGMLQuantizationType, quants
    g = np.random.Generator(np.random.PCG64(9))
    M, K = 6, 512
    nb = K // 256
    blk = g.integers(0, 256, size=(M, nb, 210), dtype=np.uint8)
    d = np.abs(g.standard_normal((M, nb)) * 0.001).astype(np.float16)
    # edge values for d: zero, a subnormal, the largest finite half, negative
    d[0, 0] = np.float16(0.0)
    d[1, 1] = np.float16(6e-8)
    d[2, 0] = np.float16(65504.0)
    d[3, 1] = np.float16(-0.5)
    blk[:, :, 208:210] = d.view(np.uint8).reshape(M, nb, 2)
    blk[4, 0, 192:208] = np.array([-128, 127] * 8, dtype=np.int8).view(np.uint8)   # extreme scales
    blk[4, 1, :192] = 0xFF                                                        # q = 31 everywhere
    blk[5, 0, :192] = 0x00                                                        # q = -32 everywhere
    blk = blk.reshape(M, nb * 210)
    deq = quants.dequantize(blk, GGMLQuantizationType.Q6_K).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "q6k_gguf.npz"), blocks=blk, dequant=deq, K=K)


def kv_fixture() -> None:
    from gguf import GGMLQuantizationType, quants
    g = np.random.Generator(np.random.PCG64(21))
    out = {}
    for name, qt, bb in (("q8_0", GGMLQuantizationType.Q8_0, 34), ("q4_0", GGMLQuantizationType.Q4_0, 18),
                         ("q4_1", GGMLQuantizationType.Q4_1, 20), ("q5_0", GGMLQuantizationType.Q5_0, 22),
                         ("q5_1", GGMLQuantizationType.Q5_1, 24), ("iq4_nl", GGMLQuantizationType.IQ4_NL, 18)):
        rows = g.integers(0, 256, size=(6, 4, bb), dtype=np.uint8)
        d = (np.abs(g.standard_normal((6, 4))) * 0.02).astype(np.float16)
        d[0, 0] = np.float16(0.0)
        d[1, 1] = np.float16(6e-8)
        d[2, 2] = np.float16(65504.0)
        d[3, 3] = np.float16(-0.5)
        rows[:, :, 0:2] = d.view(np.uint8).reshape(6, 4, 2)
        if name in ("q4_1", "q5_1"):
            # block minimum m: the usual -c * d, plus edge values
            with np.errstate(over="ignore"):   # the 65504 scale gives an infinite m: kept as an edge case
                m = (-8.0 * d.astype(np.float32) * (1 + 0.1 * g.standard_normal((6, 4)))).astype(np.float16)
            m[0, 1] = np.float16(0.0)
            m[4, 0] = np.float16(-65504.0)
            m[5, 2] = np.float16(3e-8)
            rows[:, :, 2:4] = m.view(np.uint8).reshape(6, 4, 2)
        rows = rows.reshape(6, 4 * bb)
        out[name + "_rows"] = rows
        out[name + "_dequant"] = quants.dequantize(rows, qt).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "kv_gguf.npz"), **out)


def fa_fixture() -> None:
    g = np.random.Generator(np.random.PCG64(11))
    cases = {}
    # (B, Hq, Hkv, L, D, NQ, mask, softcap, alibi)
    specs = [
        ("gqa4_l70_d64", 2, 8, 2, 70, 64, 1, False, 0.0, False),
        ("mha_l1_d128", 1, 4, 4, 1, 128, 1, False, 0.0, False),
        ("gqa4_l65_d128_mask", 2, 8, 2, 65, 128, 1, True, 0.0, False),
        ("gqa2_l64_d64_softcap", 1, 4, 2, 64, 64, 1, False, 30.0, False),
        ("gqa4_l63_d64_alibi", 1, 8, 2, 63, 64, 1, False, 0.0, True),
        ("gqa4_nq3_l40_d64", 1, 8, 2, 40, 64, 3, True, 0.0, False),
    ]
    for name, B, Hq, Hkv, L, D, NQ, use_mask, softcap, alibi in specs:
        s = 1.0 / np.sqrt(D)
        q = (g.standard_normal((B, Hq, NQ, D)) * s * 4).astype(np.float32)
        k = (g.standard_normal((B, Hkv, L, D)) * s * 4).astype(np.float16)
        v = (g.standard_normal((B, Hkv, L, D)) * s).astype(np.float16)
        mask = None
        if use_mask:
            mask = (g.standard_normal((NQ, L)) * 0.5).astype(np.float32)
            mask[:, ::7] = -np.inf
        mode = (oracle.FA_MODE_SOFTCAP if softcap else 0) | (oracle.FA_MODE_ALIBI if alibi else 0)
        out = oracle.ref_flash_attn(q, k.view(np.uint16), v.view(np.uint16), float(s), mask=mask,
                                    softcap=softcap, mode=mode)
        assert oracle.ref_stub_hits() == 0
        cases[name + "__q"] = q
        cases[name + "__k"] = k.view(np.uint16)
        cases[name + "__v"] = v.view(np.uint16)
        if mask is not None:
            cases[name + "__mask"] = mask
        cases[name + "__meta"] = np.array([softcap, 1.0 if alibi else 0.0, s], dtype=np.float64)
        cases[name + "__out"] = out
    np.savez_compressed(os.path.join(HERE, "fa_reference.npz"), **cases)


def fa_f32_fixture() -> None:
    """F32 K/V cases through the reference's flash_attn_quantized (its F32 value branch)."""
    g = np.random.Generator(np.random.PCG64(12))
    cases = {}
    specs = [
        ("gqa4_l70_d64", 1, 8, 2, 70, 64, 1, False, 0.0, False),
        ("gqa4_l65_d128_mask", 1, 8, 2, 65, 128, 1, True, 0.0, False),
        ("gqa2_l64_d64_softcap", 1, 4, 2, 64, 64, 1, False, 30.0, False),
        ("gqa4_l33_d128_alibi", 1, 8, 2, 33, 128, 1, False, 0.0, True),
        ("gqa4_nq3_l40_d64", 1, 8, 2, 40, 64, 3, True, 0.0, False),
    ]
    for name, B, Hq, Hkv, L, D, NQ, use_mask, softcap, alibi in specs:
        s = 1.0 / np.sqrt(D)
        q = (g.standard_normal((B, Hq, NQ, D)) * s * 4).astype(np.float32)
        k = (g.standard_normal((B, Hkv, L, D)) * s * 4).astype(np.float32)
        v = (g.standard_normal((B, Hkv, L, D)) * s).astype(np.float32)
        mask = None
        if use_mask:
            mask = (g.standard_normal((NQ, L)) * 0.5).astype(np.float32)
            mask[:, ::7] = -np.inf
        mode = (oracle.FA_MODE_SOFTCAP if softcap else 0) | (oracle.FA_MODE_ALIBI if alibi else 0)
        out = oracle.ref_flash_attn(q, k, v, float(s), mask=mask, softcap=softcap, mode=mode, f32_kv=True)
        assert oracle.ref_stub_hits() == 0
        cases[name + "__q"], cases[name + "__k"], cases[name + "__v"] = q, k, v
        if mask is not None:
            cases[name + "__mask"] = mask
        cases[name + "__meta"] = np.array([softcap, 1.0 if alibi else 0.0, s], dtype=np.float64)
        cases[name + "__out"] = out
    np.savez_compressed(os.path.join(HERE, "fa_f32_reference.npz"), **cases)


def q8k_fixture() -> None:
    """Rows quantised by the reference's own quantize_row_q8_k_reference (ggml_simd_hook.cpp
    :109-148) through oracle/_ref, with edge blocks: all zero, tiny values, huge values of
    both signs, exact halves after scaling (ties of the rounding) and a lone extreme."""
    g = np.random.Generator(np.random.PCG64(31))
    K = 2048
    rows = g.standard_normal((6, K)).astype(np.float32)
    rows[0, :256] = 0.0
    rows[1, :256] *= np.float32(1e-30)
    rows[1, 256:512] = np.where(np.arange(256) % 2, 1e20, -3e19).astype(np.float32)
    rows[2, :256] = (np.round(rows[2, :256] * 4) / 4).astype(np.float32)
    rows[2, 256:512] = np.float32(0.5) * (np.arange(256) % 7 - 3).astype(np.float32)
    rows[3, 512:768] = 0.0
    rows[3, 700] = np.float32(-7.0)
    rows[4] *= np.float32(1000.0)
    out = np.stack([oracle.ref_quantize_q8k(r) for r in rows])
    assert oracle.ref_stub_hits() == 0
    np.savez_compressed(os.path.join(HERE, "q8k_reference.npz"), x=rows, q8k=out)


def hook_fixture() -> None:
    """One-column MUL_MAT nodes through the reference's own hook, ggml_simd_try_mul_mat
    (src/simd/ggml_simd_hook.cpp:153-315, compiled in place), for F32 weights (handled: its
    F32 branch, simd_matmul_f32 on the scalar path below M*N*K = 512) with 1 and 3 thread
    indices, and F16 weights (declined: 0, upstream computes them)."""
    g = np.random.Generator(np.random.PCG64(41))
    out = {}
    for i, (M, K) in enumerate([(8, 32), (12, 40), (3, 160)]):
        w = g.standard_normal((M, K)).astype(np.float32)
        x = g.standard_normal((1, K)).astype(np.float32)
        for nth in (1, 3):
            r, y = oracle.ref_try_mul_mat(w, x, 0, nth)
            assert r == 1 and oracle.ref_stub_hits() == 0
            out[f"f32_{i}_nth{nth}__y"] = y
        out[f"f32_{i}__w"], out[f"f32_{i}__x"] = w, x
    w16 = g.standard_normal((8, 32)).astype(np.float16)
    x16 = g.standard_normal((1, 32)).astype(np.float32)
    r, _ = oracle.ref_try_mul_mat(w16.view(np.uint16), x16, 1, 1)
    out["f16__handled"] = np.array([r], dtype=np.int32)
    np.savez_compressed(os.path.join(HERE, "hook_reference.npz"), **out)


def matmul_fixture() -> None:
    g = np.random.Generator(np.random.PCG64(13))
    cases = {}
    for i, (M, N, K) in enumerate([(4, 3, 8), (1, 1, 511), (7, 5, 14), (3, 1, 100)]):
        a = g.standard_normal((M, K)).astype(np.float32)
        b = g.standard_normal((K, N)).astype(np.float32)
        cases[f"a{i}"] = a
        cases[f"b{i}"] = b
        cases[f"c{i}"] = oracle.ref_matmul_f32_small(a, b)
    assert oracle.ref_stub_hits() == 0
    np.savez_compressed(os.path.join(HERE, "matmul_reference.npz"), **cases)


def matmul_f16_fixture() -> None:
    g = np.random.Generator(np.random.PCG64(17))
    cases = {}
    # (M, N, K), all with M*N*K < 512 (the scalar path) and M*N % 8 == 0 (the F16C
    # rounding of the result).  K = 56 / 16 / 24 keep 16-byte rows, so the GPU takes its
    # vectorised GEMV (N = 1), skinny tensor-core (N = 4, 8) and tcgen05 GEMM (N >= 17)
    # kernels on them; K = 63 / 31 / 15 / 7 take the unaligned paths.
    shapes = [(8, 1, 56), (1, 8, 56), (2, 4, 56), (1, 24, 16), (1, 32, 15), (4, 2, 63),
              (8, 1, 63), (2, 4, 63), (8, 2, 31), (2, 8, 31), (4, 8, 15), (8, 8, 7)]
    for i, (M, N, K) in enumerate(shapes):
        a = (g.standard_normal((M, K)) * 0.5).astype(np.float16)
        b = g.standard_normal((K, N)).astype(np.float16)
        if i == 0:  # zeros, signed zeros, a subnormal and large finite values
            a[0, :4] = np.array([0.0, -0.0, 6e-8, 1000.0], dtype=np.float16)
            b[:4, 0] = np.array([-0.0, 5.0, 3000.0, -0.25], dtype=np.float16)
        c = oracle.ref_matmul_f16_small(a.view(np.uint16), b.view(np.uint16))
        cases[f"a{i}"] = a.view(np.uint16)
        cases[f"b{i}"] = b.view(np.uint16)
        cases[f"c{i}"] = c
    assert oracle.ref_stub_hits() == 0
    np.savez_compressed(os.path.join(HERE, "matmul_f16_reference.npz"), **cases)


if __name__ == "__main__":
    oracle.build()
    if not oracle.ref_available():
        sys.exit("oracle/_ref/libmlzref.so is missing: run `make -C oracle` where the reference tree exists")
    q4k_fixture()
    q6k_fixture()
    kv_fixture()
    fa_fixture()
    fa_f32_fixture()
    q8k_fixture()
    hook_fixture()
    matmul_fixture()
    matmul_f16_fixture()
    print("fixtures written to", HERE)
