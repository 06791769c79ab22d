"""CPU oracle for the MLz src/simd hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of bench.py may
import this package.  It is the checker, never the thing measured or shipped: the
product (``mlz_b200``) has no CPU fallback and never imports it.

Wraps two shared libraries built by ``oracle/Makefile``:

* ``liboracle.so`` -- ``oracle.c``: fp64 restatements (``ora_*``) and the timed
  AVX-512/AVX2 restatements of the reference kernels (``base_*``).
* ``_ref/libmlzref.so`` -- the reference's own ``src/simd/flash_attention.cpp`` and
  ``src/simd/simd_matmul.cpp`` built from source, used to pin the restatement.

Array conventions follow ggml (ne[0] is the fastest axis), so a numpy array has the
ggml dims reversed: W is (M, K), X is (N, K), Y is (N, M); attention tensors are
(B, H, n, D).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(_HERE, "liboracle.so")
_REF = os.path.join(_HERE, "_ref", "libmlzref.so")

QK_K = 256
Q4K_BYTES = 144
Q8K_BYTES = 292
Q6K_BYTES = 210
FA_MODE_ALIBI = 0x08
FA_MODE_SOFTCAP = 0x10
FA_MODE_GQA_BATCH = 0x04


# The reference checkout this recipe compiles oracle/_ref from (read in place, never
# copied); MLZ_REF_SIMD overrides it.  Where it is absent the prebuilt _ref is used.
_REF_SIMD = os.environ.get("MLZ_REF_SIMD", "/root/reference/src/simd")


def build(quiet: bool = True) -> None:
    """Compile liboracle.so (and oracle/_ref when the reference tree exists)."""
    args = ["make", "-C", _HERE]
    if os.path.isdir(_REF_SIMD):
        args.append("REF_SIMD=" + _REF_SIMD)
    out = subprocess.run(args, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


_lib = None
_ref = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB):
            build()
        _lib = C.CDLL(_LIB)
        _declare(_lib)
    return _lib


def ref_available() -> bool:
    return os.path.exists(_REF)


def ref() -> C.CDLL:
    global _ref
    if _ref is None:
        _ref = C.CDLL(_REF)
        _ref.mlzref_config_size.restype = C.c_size_t
        _ref.mlzref_flash_attn_f16.argtypes = [C.c_void_p]
        _ref.mlzref_flash_attn_f32.argtypes = [C.c_void_p]
        _ref.mlzref_quantize_row_q8k.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
        _ref.mlzref_try_mul_mat.argtypes = [C.c_int, C.c_void_p, C.c_size_t, C.c_int64, C.c_int64, C.c_void_p,
                                            C.c_int64, C.c_void_p, C.c_int]
        _ref.simd_matmul_f32.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                         C.c_size_t, C.c_size_t, C.c_int, C.c_int]
        _ref.simd_matmul_f16.argtypes = _ref.simd_matmul_f32.argtypes
    return _ref


def ref_stub_hits() -> int:
    return C.c_int.in_dll(ref(), "mlzref_stub_hits").value


class OraFA(C.Structure):
    """Mirror of ``ora_fa_t`` in oracle.c."""
    _fields_ = [
        ("head_dim_k", C.c_int64), ("head_dim_v", C.c_int64), ("n_queries", C.c_int64),
        ("n_kv", C.c_int64), ("n_head_q", C.c_int64), ("n_head_kv", C.c_int64),
        ("batch_size", C.c_int64),
        ("scale", C.c_float), ("logit_softcap", C.c_float), ("max_bias", C.c_float),
        ("mode", C.c_uint32),
        ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("mask", C.c_void_p),
        ("dst", C.c_void_p),
        ("q_nb", C.c_size_t * 4), ("k_nb", C.c_size_t * 4), ("v_nb", C.c_size_t * 4),
        ("mask_nb", C.c_size_t * 4), ("dst_nb", C.c_size_t * 4),
        ("kv_len", C.c_void_p),
        ("kv_type", C.c_int32),
    ]


class RefFAConfig(C.Structure):
    """Mirror of the reference's ``flash_attn_config_t`` (src/simd/flash_attention.h:65-114)."""
    _fields_ = [
        ("head_dim_k", C.c_int64), ("head_dim_v", C.c_int64), ("n_queries", C.c_int64),
        ("n_kv", C.c_int64), ("n_head_q", C.c_int64), ("n_head_kv", C.c_int64),
        ("batch_size", C.c_int64),
        ("scale", C.c_float), ("logit_softcap", C.c_float), ("max_bias", C.c_float),
        ("mode", C.c_uint32), ("window_size", C.c_int64),
        ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("mask", C.c_void_p),
        ("dst", C.c_void_p),
        ("q_nb", C.c_size_t * 4), ("k_nb", C.c_size_t * 4), ("v_nb", C.c_size_t * 4),
        ("mask_nb", C.c_size_t * 4), ("dst_nb", C.c_size_t * 4),
        ("k_type", C.c_int), ("v_type", C.c_int),
        ("page_size", C.c_int), ("page_table", C.c_void_p), ("n_pages_logical", C.c_int),
        ("k_pages", C.c_void_p), ("v_pages", C.c_void_p),
        ("ith", C.c_int), ("nth", C.c_int),
    ]


def _declare(L: C.CDLL) -> None:
    vp, i64, sz, i32 = C.c_void_p, C.c_int64, C.c_size_t, C.c_int
    L.ora_f16_to_f32.argtypes = [C.c_uint16]
    L.ora_f16_to_f32.restype = C.c_float
    L.ora_f32_to_f16.argtypes = [C.c_float]
    L.ora_f32_to_f16.restype = C.c_uint16
    L.ora_f32_to_f16_array.argtypes = [vp, vp, i64]
    L.ora_f16_to_f32_array.argtypes = [vp, vp, i64]
    L.ora_mul_mat_f16.argtypes = [vp, sz, i64, i64, vp, sz, i64, vp, i32]
    L.ora_mul_mat_f32.argtypes = [vp, sz, i64, i64, vp, sz, i64, vp]
    L.ora_q4k_dequant_row.argtypes = [vp, i64, vp]
    L.ora_kv_row.argtypes = [vp, i64, i32, vp]
    L.ora_mul_mat_q4k.argtypes = [vp, sz, i64, i64, vp, sz, i64, vp]
    L.ora_q6k_dequant_row.argtypes = [vp, i64, vp]
    L.ora_mul_mat_q6k.argtypes = [vp, sz, i64, i64, vp, sz, i64, vp]
    L.base_mul_mat_q6k.argtypes = [vp, sz, i64, i64, vp, sz, i64, vp, i32]
    L.ora_quantize_row_q8k.argtypes = [vp, i64, vp]
    L.ora_vec_dot_q4k_q8k.argtypes = [i64, vp, vp]
    L.ora_vec_dot_q4k_q8k.restype = C.c_float
    L.ora_flash_attn.argtypes = [C.POINTER(OraFA)]
    L.base_mul_mat_f16.argtypes = [vp, sz, i64, i64, vp, sz, i64, vp, i32]
    L.base_mul_mat_q4k.argtypes = [vp, sz, i64, i64, vp, sz, i64, vp, i32]
    L.base_flash_attn.argtypes = [C.POINTER(OraFA), i32]
    L.base_has_avx512.restype = i32
    L.base_has_avx2.restype = i32


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle expects C-contiguous arrays"
    return a.ctypes.data


# ---------------------------------------------------------------------------
# f16 helpers
# ---------------------------------------------------------------------------

def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().ora_f32_to_f16_array(_p(x), _p(out), x.size)
    return out


def f16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().ora_f16_to_f32_array(_p(h), _p(out), h.size)
    return out


# ---------------------------------------------------------------------------
# exact mul_mat checkers (fp64 accumulation)
# ---------------------------------------------------------------------------

def mul_mat_f16(w_bits: np.ndarray, x: np.ndarray, round_x: bool = True) -> np.ndarray:
    """y[n, m] = sum_k f16(W[m, k]) * X[n, k] (X narrowed to f16 when round_x)."""
    w_bits = np.ascontiguousarray(w_bits.view(np.uint16))
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = w_bits.shape
    N = x.shape[0]
    assert x.shape[1] == K
    y = np.empty((N, M), dtype=np.float64)
    lib().ora_mul_mat_f16(_p(w_bits), K * 2, M, K, _p(x), K * 4, N, _p(y), int(round_x))
    return y


def mul_mat_f32(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = w.shape
    N = x.shape[0]
    y = np.empty((N, M), dtype=np.float64)
    lib().ora_mul_mat_f32(_p(w), K * 4, M, K, _p(x), K * 4, N, _p(y))
    return y


def q4k_dequant(blocks: np.ndarray, K: int) -> np.ndarray:
    """Dequantise Q4_K rows: blocks is (M, K/256*144) uint8 -> (M, K) f32."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    M = blocks.shape[0]
    out = np.empty((M, K), dtype=np.float32)
    for m in range(M):
        lib().ora_q4k_dequant_row(blocks[m].ctypes.data, K, out[m].ctypes.data)
    return out


def mul_mat_q4k(blocks: np.ndarray, x: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, row_bytes = blocks.shape
    K = row_bytes // Q4K_BYTES * QK_K
    N = x.shape[0]
    y = np.empty((N, M), dtype=np.float64)
    lib().ora_mul_mat_q4k(_p(blocks), row_bytes, M, K, _p(x), K * 4, N, _p(y))
    return y


def q6k_dequant(blocks: np.ndarray, K: int) -> np.ndarray:
    """Dequantise Q6_K rows: blocks is (M, K/256*210) uint8 -> (M, K) f32."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    M = blocks.shape[0]
    out = np.empty((M, K), dtype=np.float32)
    for m in range(M):
        lib().ora_q6k_dequant_row(blocks[m].ctypes.data, K, out[m].ctypes.data)
    return out


def mul_mat_q6k(blocks: np.ndarray, x: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, row_bytes = blocks.shape
    K = row_bytes // Q6K_BYTES * QK_K
    N = x.shape[0]
    y = np.empty((N, M), dtype=np.float64)
    lib().ora_mul_mat_q6k(_p(blocks), row_bytes, M, K, _p(x), K * 4, N, _p(y))
    return y


def quantize_q8k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    K = x.shape[-1]
    out = np.empty(K // QK_K * Q8K_BYTES, dtype=np.uint8)
    lib().ora_quantize_row_q8k(_p(x), K, _p(out))
    return out


def vec_dot_q4k_q8k(w_row: np.ndarray, y_q8: np.ndarray, K: int) -> float:
    w_row = np.ascontiguousarray(w_row, dtype=np.uint8)
    y_q8 = np.ascontiguousarray(y_q8, dtype=np.uint8)
    return float(lib().ora_vec_dot_q4k_q8k(K, _p(w_row), _p(y_q8)))


# ---------------------------------------------------------------------------
# flash-attention decode
# ---------------------------------------------------------------------------

def _nb(a: np.ndarray) -> tuple:
    """ggml byte strides nb[0..3] of a numpy array with dims (d3, d2, d1, d0)."""
    s = a.strides[::-1]
    return tuple(s) + (0,) * (4 - len(s))


def _fa_struct(q, k_bits, v_bits, out, scale, mask=None, kv_len=None,
               softcap=0.0, max_bias=0.0, mode=0, kv_type=1) -> OraFA:
    B, Hq, NQ, D = q.shape
    Hkv, NKV = v_bits.shape[1], v_bits.shape[2]
    DV = out.shape[-1]
    c = OraFA()
    c.head_dim_k, c.head_dim_v, c.n_queries, c.n_kv = D, DV, NQ, NKV
    c.n_head_q, c.n_head_kv, c.batch_size = Hq, Hkv, B
    c.scale, c.logit_softcap, c.max_bias, c.mode = scale, softcap, max_bias, mode
    c.q, c.k, c.v, c.dst = _p(q), _p(k_bits), _p(v_bits), _p(out)
    c.mask = _p(mask) if mask is not None else None
    c.q_nb[:] = _nb(q)
    c.k_nb[:] = _nb(k_bits)
    c.v_nb[:] = _nb(v_bits)
    c.dst_nb[:] = _nb(out)
    if mask is not None:
        c.mask_nb[:] = _nb(mask)
    c.kv_len = _p(kv_len) if kv_len is not None else None
    c.kv_type = kv_type
    return c


def flash_attn(q, k_bits, v_bits, scale, mask=None, kv_len=None, softcap=0.0,
               max_bias=0.0, mode=0) -> np.ndarray:
    """Exact decode attention. q: (B, Hq, NQ, D) f32; k/v: (B, Hkv, NKV, D) f16 bits;
    mask: (NQ, NKV) f32 or None; kv_len: (B,) int32 or None. Returns (B, Hq, NQ, DV)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k_bits = np.ascontiguousarray(k_bits.view(np.uint16))
    v_bits = np.ascontiguousarray(v_bits.view(np.uint16))
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.float32)
    if kv_len is not None:
        kv_len = np.ascontiguousarray(kv_len, dtype=np.int32)
    B, Hq, NQ, _ = q.shape
    out = np.zeros((B, Hq, NQ, v_bits.shape[-1]), dtype=np.float32)
    c = _fa_struct(q, k_bits, v_bits, out, scale, mask, kv_len, softcap, max_bias, mode)
    lib().ora_flash_attn(C.byref(c))
    return out


# ggml type id -> (bytes, values) per block: Q8_0, Q4_0, Q4_1, Q5_0, Q5_1, IQ4_NL
KV_BLOCK = {8: (34, 32), 2: (18, 32), 3: (20, 32), 6: (22, 32), 7: (24, 32), 20: (18, 32)}


def flash_attn_q(q, k_blocks, v_blocks, scale, kv_type, mask=None, kv_len=None, softcap=0.0,
                 max_bias=0.0, mode=0) -> np.ndarray:
    """Exact decode attention over a quantised KV cache (kv_type 8 = Q8_0, 2 = Q4_0, 3 = Q4_1,
    6 = Q5_0, 7 = Q5_1, 20 = IQ4_NL) or an F32 one (kv_type 0): k/v_blocks: (B, Hkv, NKV,
    row_bytes) uint8 rows (blocks, or D f32 values); every row is decoded with GGUF's rule
    (ora_kv_row) and the attention runs in fp64."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k_blocks = np.ascontiguousarray(k_blocks, dtype=np.uint8)
    v_blocks = np.ascontiguousarray(v_blocks, dtype=np.uint8)
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.float32)
    if kv_len is not None:
        kv_len = np.ascontiguousarray(kv_len, dtype=np.int32)
    B, Hq, NQ, D = q.shape
    out = np.zeros((B, Hq, NQ, D), dtype=np.float32)
    c = _fa_struct(q, k_blocks, v_blocks, out, scale, mask, kv_len, softcap, max_bias, mode, kv_type)
    c.head_dim_k = c.head_dim_v = D
    lib().ora_flash_attn(C.byref(c))
    return out


def kv_dequant(rows: np.ndarray, D: int, kv_type: int) -> np.ndarray:
    """Dequantise (..., D/32*block_bytes) uint8 K/V rows of kv_type to (..., D) f32."""
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    lead = rows.shape[:-1]
    flat = rows.reshape(-1, rows.shape[-1])
    out = np.empty((flat.shape[0], D), dtype=np.float32)
    for i in range(flat.shape[0]):
        lib().ora_kv_row(flat[i].ctypes.data, D, kv_type, out[i].ctypes.data)
    return out.reshape(*lead, D)


def base_flash_attn_q(q, k_blocks, v_blocks, scale, kv_type, kv_len=None, nth: int = 1) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    k_blocks = np.ascontiguousarray(k_blocks, dtype=np.uint8)
    v_blocks = np.ascontiguousarray(v_blocks, dtype=np.uint8)
    if kv_len is not None:
        kv_len = np.ascontiguousarray(kv_len, dtype=np.int32)
    B, Hq, NQ, D = q.shape
    out = np.zeros((B, Hq, NQ, D), dtype=np.float32)
    c = _fa_struct(q, k_blocks, v_blocks, out, scale, None, kv_len, kv_type=kv_type)
    c.head_dim_k = c.head_dim_v = D
    lib().base_flash_attn(C.byref(c), nth)
    return out


def ref_flash_attn(q, k_bits, v_bits, scale, mask=None, softcap=0.0, max_bias=0.0,
                   mode=0, f32_kv: bool = False) -> np.ndarray:
    """Run the reference's own flash_attn_quantized (oracle/_ref) on F16 K/V (f16 bit
    patterns), or on F32 K/V arrays with f32_kv=True."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    if f32_kv:
        k_bits = np.ascontiguousarray(k_bits, dtype=np.float32)
        v_bits = np.ascontiguousarray(v_bits, dtype=np.float32)
    else:
        k_bits = np.ascontiguousarray(k_bits.view(np.uint16))
        v_bits = np.ascontiguousarray(v_bits.view(np.uint16))
    B, Hq, NQ, D = q.shape
    _, Hkv, NKV, DV = v_bits.shape
    out = np.zeros((B, Hq, NQ, DV), dtype=np.float32)
    c = RefFAConfig()
    c.head_dim_k, c.head_dim_v, c.n_queries, c.n_kv = D, DV, NQ, NKV
    c.n_head_q, c.n_head_kv, c.batch_size = Hq, Hkv, B
    c.scale, c.logit_softcap, c.max_bias, c.mode = scale, softcap, max_bias, mode
    c.q, c.k, c.v, c.dst = _p(q), _p(k_bits), _p(v_bits), _p(out)
    c.q_nb[:] = _nb(q)
    c.k_nb[:] = _nb(k_bits)
    c.v_nb[:] = _nb(v_bits)
    c.dst_nb[:] = _nb(out)
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.float32)
        c.mask = _p(mask)
        nb = _nb(mask)
        # flash_attn_quantized reads mask(iq, j) at iq*nb[0] + j*nb[1]
        # (src/simd/flash_attention.cpp:352); hand it the transposed strides so that
        # it reads the same element the skeleton's iq*nb1 + j*nb0 does.
        c.mask_nb[0], c.mask_nb[1] = nb[1], nb[0]
    c.k_type = c.v_type = 0 if f32_kv else 1
    c.ith, c.nth = 0, 1
    assert C.sizeof(RefFAConfig) == ref().mlzref_config_size()
    if f32_kv:
        ref().mlzref_flash_attn_f32(C.byref(c))
    else:
        ref().mlzref_flash_attn_f16(C.byref(c))
    return out


def ref_quantize_q8k(x: np.ndarray) -> np.ndarray:
    """The reference's own quantize_row_q8_k_reference (src/simd/ggml_simd_hook.cpp:109-148,
    compiled into oracle/_ref) on one row of K f32 values: (K/256 * 292,) uint8."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.shape[0] // QK_K * Q8K_BYTES, dtype=np.uint8)
    ref().mlzref_quantize_row_q8k(_p(x), _p(out), int(x.shape[0]))
    return out


def ref_try_mul_mat(w: np.ndarray, x: np.ndarray, w_type: int, nth: int = 1):
    """The reference's own hook, ggml_simd_try_mul_mat (src/simd/ggml_simd_hook.cpp:153-315,
    compiled into oracle/_ref), on W (M, K) of w_type (0 = F32, 1 = F16 bit patterns) and X
    (N, K) f32, for thread indices 0..nth-1 in turn.  Returns (handled, Y (N, M))."""
    w = np.ascontiguousarray(w)
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = w.shape
    N = x.shape[0]
    y = np.zeros((N, M), dtype=np.float32)
    r = ref().mlzref_try_mul_mat(w_type, _p(w), w.strides[0], M, K, _p(x), N, _p(y), nth)
    return int(r), y


def ref_matmul_f32_small(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """The reference's simd_matmul_f32 (row-major C = A.B) below its scalar
    threshold M*N*K < 512 (src/simd/simd_matmul.cpp:217-223)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    M, K = a.shape
    N = b.shape[1]
    assert M * N * K < 512
    c = np.full((M, N), np.nan, dtype=np.float32)
    ref().simd_matmul_f32(_p(a), _p(b), _p(c), M, N, K, 0, 1)
    return c


def ref_matmul_f16_small(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """The reference's simd_matmul_f16 (src/simd/simd_matmul.cpp:428-480): f16 A (M x K)
    and B (K x N) widened to f32, simd_matmul_f32's scalar i-k-j loop (fp32, k ascending,
    below M*N*K < 512: :217-223), C rounded to f16 (F16C round-to-nearest-even in chunks
    of 8, :378-384; the scalar tail loop :387-406 truncates, so callers keep M*N a
    multiple of 8).  Returns C's f16 bits (M x N)."""
    a_bits = np.ascontiguousarray(a_bits, dtype=np.uint16)
    b_bits = np.ascontiguousarray(b_bits, dtype=np.uint16)
    M, K = a_bits.shape
    N = b_bits.shape[1]
    assert M * N * K < 512 and (M * N) % 8 == 0
    c = np.full((M, N), 0x7E00, dtype=np.uint16)
    ref().simd_matmul_f16(_p(a_bits), _p(b_bits), _p(c), M, N, K, 0, 1)
    return c


# ---------------------------------------------------------------------------
# timed CPU baselines (the reference's loop structure on the host cores)
# ---------------------------------------------------------------------------

def base_mul_mat_f16(w_bits, x, nth: int) -> np.ndarray:
    w_bits = np.ascontiguousarray(w_bits.view(np.uint16))
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = w_bits.shape
    N = x.shape[0]
    y = np.empty((N, M), dtype=np.float32)
    lib().base_mul_mat_f16(_p(w_bits), K * 2, M, K, _p(x), K * 4, N, _p(y), nth)
    return y


def base_mul_mat_q4k(blocks, x, nth: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, row_bytes = blocks.shape
    K = row_bytes // Q4K_BYTES * QK_K
    N = x.shape[0]
    y = np.empty((N, M), dtype=np.float32)
    lib().base_mul_mat_q4k(_p(blocks), row_bytes, M, K, _p(x), K * 4, N, _p(y), nth)
    return y


def base_mul_mat_q6k(blocks, x, nth: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, row_bytes = blocks.shape
    K = row_bytes // Q6K_BYTES * QK_K
    N = x.shape[0]
    y = np.empty((N, M), dtype=np.float32)
    lib().base_mul_mat_q6k(_p(blocks), row_bytes, M, K, _p(x), K * 4, N, _p(y), nth)
    return y


def base_flash_attn(q, k_bits, v_bits, scale, kv_len=None, nth: int = 1) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    k_bits = np.ascontiguousarray(k_bits.view(np.uint16))
    v_bits = np.ascontiguousarray(v_bits.view(np.uint16))
    if kv_len is not None:
        kv_len = np.ascontiguousarray(kv_len, dtype=np.int32)
    B, Hq, NQ, _ = q.shape
    out = np.zeros((B, Hq, NQ, v_bits.shape[-1]), dtype=np.float32)
    c = _fa_struct(q, k_bits, v_bits, out, scale, None, kv_len)
    lib().base_flash_attn(C.byref(c), nth)
    return out


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def host_cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def rel_err(got: np.ndarray, want: np.ndarray) -> float:
    """max |got - want| / max |want| -- the parity gate used by every test."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    den = float(np.max(np.abs(want))) if want.size else 0.0
    if want.size == 0:
        return 0.0
    return float(np.max(np.abs(got - want))) / (den if den > 0 else 1.0)
