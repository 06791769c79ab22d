"""Host-side mirror of MLz's src/simd interface over the mlzc C ABI.

Names follow the reference where a reference function exists:

* :func:`ggml_simd_try_mul_mat` / :func:`ggml_simd_try_flash_attn` -- the ggml hooks
  (src/simd/ggml_simd_hook.cpp:153, :317): host tensors in, 1 = handled / 0 = fall back.
* :func:`flash_attn_dispatch` -- flash_attn_dispatch (src/simd/flash_attention.cpp:53)
  on device tensors.
* :func:`mul_mat` -- the compute of ggml_compute_forward_mul_mat for F32 / F16 / Q4_K
  weights (src/simd/ggml-cpu-simd.c:1246) on device tensors.

Device tensors are torch CUDA tensors (torch is only the allocator / stream provider);
every computation runs in libmlzc.so.  Layout: numpy / torch dims are ggml's ne[]
reversed, so W is (M, K), X is (N, K), Y is (N, M), attention tensors are (B, H, n, D).
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from ._lib import (FA_MODE_ALIBI, FA_MODE_SOFTCAP, TYPE_F16, TYPE_F32, TYPE_IQ4_NL, TYPE_Q4_0, TYPE_Q4_1, TYPE_Q4_K,
                   TYPE_Q5_0, TYPE_Q5_1, TYPE_Q6_K, TYPE_Q8_0,
                   FaDesc,
                   MlzcError, TensorView, check, lib)

QK_K = 256
Q4K_BYTES = 144


def _torch():
    import torch
    return torch


def _stream_handle(stream) -> int:
    torch = _torch()
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def weight_type_of(w) -> int:
    """ggml type id of a weight tensor: f16 -> F16, f32 -> F32, uint8 -> Q4_K blocks (pass
    w_type=TYPE_Q6_K to the calls for Q6_K blocks)."""
    torch = _torch()
    if w.dtype == torch.float16:
        return TYPE_F16
    if w.dtype == torch.float32:
        return TYPE_F32
    if w.dtype == torch.uint8:
        return TYPE_Q4_K
    raise TypeError(f"unsupported weight dtype {w.dtype}")


def mul_mat_workspace_bytes(w_type: int, M: int, K: int, N: int) -> int:
    out = C.c_size_t(0)
    check(lib().mlzc_mul_mat_workspace_bytes(w_type, M, K, N, C.byref(out)))
    return out.value


def mul_mat(w, x, *, out=None, workspace=None, stream=None, w_type=None):
    """y[n, m] = sum_k W[m, k] x[n, k] on the GPU (ggml mul_mat, dst = [M, N]).

    w: (M, K) float16 / float32, or uint8 super-blocks: (M, K/256*144) Q4_K (the default
    for uint8) or (M, K/256*210) Q6_K with w_type=TYPE_Q6_K.
    x: (N, K) float32 (row stride may exceed K).  Returns y: (N, M) float32.
    """
    torch = _torch()
    if w_type is None:
        w_type = weight_type_of(w)
    M = w.shape[0]
    N, K = x.shape
    if x.dtype != torch.float32:
        raise TypeError("activations must be float32")
    if w.stride(-1) != 1 or x.stride(-1) != 1:
        raise ValueError("rows must be contiguous")
    if out is None:
        out = torch.empty((N, M), dtype=torch.float32, device=x.device)
    if out.stride(-1) != 1:
        raise ValueError("output rows must be contiguous")
    wsb = mul_mat_workspace_bytes(w_type, M, K, N)
    if wsb and workspace is None:
        workspace = torch.empty(wsb, dtype=torch.uint8, device=x.device)
    check(lib().mlzc_mul_mat_dev(
        w_type, w.data_ptr(), w.stride(0) * w.element_size(), M, K,
        x.data_ptr(), x.stride(0) * 4, N, out.data_ptr(), out.stride(0) * 4,
        workspace.data_ptr() if workspace is not None else None,
        workspace.numel() if workspace is not None else 0, _stream_handle(stream)))
    return out


Q8K_BYTES = 292


def quantize_q8k(x, *, out=None, stream=None):
    """F32 activations (N, K) on the device -> Q8_K blocks (N, K/256*292) uint8
    (mlzc_quantize_q8k_dev; the reference's quantize_row_q8_k_reference per column)."""
    torch = _torch()
    N, K = x.shape
    if out is None:
        out = torch.empty((N, K // QK_K * Q8K_BYTES), dtype=torch.uint8, device=x.device)
    check(lib().mlzc_quantize_q8k_dev(x.data_ptr(), x.stride(0) * 4, K, N, out.data_ptr(),
                                      out.stride(0) * out.element_size(), _stream_handle(stream)))
    return out


def _nb(t, esz: int):
    """ggml byte strides nb[0..3] of a (d3, d2, d1, d0) tensor / array."""
    if hasattr(t, "stride") and callable(t.stride):
        st = [s * esz for s in t.stride()]
    else:
        st = list(t.strides)
    st = st[::-1]
    return tuple(st + [0] * (4 - len(st)))


def make_fa_desc(q_ptr, q_nb, k_ptr, k_nb, v_ptr, v_nb, dst_ptr, dst_nb, dims, scale,
                 mask_ptr=None, mask_nb=(0, 0, 0, 0), kv_len_ptr=None, softcap=0.0,
                 alibi=False, max_bias=0.0, kv_type=TYPE_F16) -> FaDesc:
    """dims = (B, Hq, NQ, Hkv, NKV, D); kv_type: TYPE_F16, or a quantised cache type
    (TYPE_Q8_0, TYPE_Q4_0, TYPE_Q4_1, TYPE_Q5_0, TYPE_Q5_1, TYPE_IQ4_NL; k_nb / v_nb then
    in bytes with nb[0] = the block size)."""
    B, Hq, NQ, Hkv, NKV, D = dims
    d = FaDesc()
    d.head_dim_k = d.head_dim_v = D
    d.n_queries, d.n_kv, d.n_head_q, d.n_head_kv, d.batch_size = NQ, NKV, Hq, Hkv, B
    d.scale = scale
    d.logit_softcap = softcap
    d.max_bias = max_bias
    mode = 0x04 if Hkv < Hq else 0
    if softcap:
        mode |= FA_MODE_SOFTCAP
    if alibi:
        mode |= FA_MODE_ALIBI
    d.mode = mode
    d.q, d.k, d.v, d.dst = q_ptr, k_ptr, v_ptr, dst_ptr
    d.mask = mask_ptr
    d.q_nb[:] = q_nb
    d.k_nb[:] = k_nb
    d.v_nb[:] = v_nb
    d.dst_nb[:] = dst_nb
    d.mask_nb[:] = mask_nb
    d.k_type = d.v_type = kv_type
    d.kv_len = kv_len_ptr
    return d


def flash_attn_workspace_bytes(desc: FaDesc) -> int:
    out = C.c_size_t(0)
    check(lib().mlzc_flash_attn_workspace_bytes(C.byref(desc), C.byref(out)))
    return out.value


def flash_attn_dispatch(q, k, v, scale: float, *, kv_len=None, mask=None, softcap: float = 0.0,
                        alibi: bool = False, out=None, workspace=None, stream=None):
    """Flash-attention on device tensors: q (B, Hq, NQ, D) f32; k, v (B, Hkv, L, D) f16
    (any strides with contiguous rows); kv_len (B,) int32 or None; mask (NQ, L) f32.
    Returns out (B, Hq, NQ, D) f32."""
    torch = _torch()
    B, Hq, NQ, D = q.shape
    _, Hkv, L, _ = k.shape
    if out is None:
        out = torch.empty((B, Hq, NQ, D), dtype=torch.float32, device=q.device)
    desc = make_fa_desc(q.data_ptr(), _nb(q, 4), k.data_ptr(), _nb(k, 2), v.data_ptr(), _nb(v, 2),
                        out.data_ptr(), _nb(out, 4), (B, Hq, NQ, Hkv, L, D), scale,
                        mask.data_ptr() if mask is not None else None,
                        _nb(mask, 4) if mask is not None else (0, 0, 0, 0),
                        kv_len.data_ptr() if kv_len is not None else None, softcap, alibi)
    wsb = flash_attn_workspace_bytes(desc)
    if wsb and workspace is None:
        workspace = torch.empty(wsb, dtype=torch.uint8, device=q.device)
    check(lib().mlzc_flash_attn_dev(C.byref(desc), workspace.data_ptr() if workspace is not None else None,
                                    workspace.numel() if workspace is not None else 0,
                                    _stream_handle(stream)))
    return out


# bytes per 32-value block of each quantised KV-cache type (GGUF layouts)
# (F32 rows: nb[0] is the 4-byte element)
KV_BLOCK_BYTES = {TYPE_Q8_0: 34, TYPE_Q4_0: 18, TYPE_Q4_1: 20, TYPE_Q5_0: 22, TYPE_Q5_1: 24, TYPE_IQ4_NL: 18,
                  TYPE_F32: 4}


def flash_attn_dispatch_quant(q, k, v, scale: float, kv_type: int, *, kv_len=None, mask=None,
                              softcap: float = 0.0, alibi: bool = False, out=None, workspace=None,
                              stream=None):
    """Flash-attention over a quantised KV cache on device tensors: q (B, Hq, NQ, D) f32;
    k, v (B, Hkv, L, D/32*block_bytes) uint8 rows of blocks of kv_type (Q8_0 34 bytes, Q4_0
    18, Q4_1 20, Q5_0 22, Q5_1 24, IQ4_NL 18), or (B, Hkv, L, 4 D) bytes of f32 rows for
    TYPE_F32 (D <= 128); any strides with contiguous rows.  Returns out (B, Hq, NQ, D) f32."""
    torch = _torch()
    B, Hq, NQ, D = q.shape
    _, Hkv, L, _ = k.shape
    bb = KV_BLOCK_BYTES[kv_type]
    if out is None:
        out = torch.empty((B, Hq, NQ, D), dtype=torch.float32, device=q.device)
    knb = (bb,) + tuple(_nb(k, 1)[1:])
    vnb = (bb,) + tuple(_nb(v, 1)[1:])
    desc = make_fa_desc(q.data_ptr(), _nb(q, 4), k.data_ptr(), knb, v.data_ptr(), vnb,
                        out.data_ptr(), _nb(out, 4), (B, Hq, NQ, Hkv, L, D), scale,
                        mask.data_ptr() if mask is not None else None,
                        _nb(mask, 4) if mask is not None else (0, 0, 0, 0),
                        kv_len.data_ptr() if kv_len is not None else None, softcap, alibi, kv_type=kv_type)
    wsb = flash_attn_workspace_bytes(desc)
    if wsb and workspace is None:
        workspace = torch.empty(wsb, dtype=torch.uint8, device=q.device)
    check(lib().mlzc_flash_attn_dev(C.byref(desc), workspace.data_ptr() if workspace is not None else None,
                                    workspace.numel() if workspace is not None else 0,
                                    _stream_handle(stream)))
    return out


# ----------------------------------------------------------------- host level

def tensor_view(arr: np.ndarray, ggml_type: int, ne0: Optional[int] = None) -> TensorView:
    """mlzc_tensor for a host numpy array whose dims are ggml's reversed.  For Q4_K / Q6_K
    pass the logical row length ne0 (arr is then (M, ne0/256*144) or (M, ne0/256*210) uint8)."""
    t = TensorView()
    t.type = ggml_type
    shape = list(arr.shape[::-1]) + [1] * (4 - arr.ndim)
    if ne0 is not None:
        shape[0] = ne0
    t.ne[:] = shape
    nb = list(arr.strides[::-1]) + [0] * (4 - arr.ndim)
    if ggml_type == TYPE_Q4_K:
        nb[0] = Q4K_BYTES
    elif ggml_type == TYPE_Q6_K:
        nb[0] = 210
    for i in range(arr.ndim, 4):
        nb[i] = nb[i - 1] * shape[i - 1] if i > 0 else 0
    t.nb[:] = nb
    t.data = arr.ctypes.data
    return t


def ggml_simd_try_mul_mat(src0: TensorView, src1: TensorView, dst: TensorView, ith: int = 0,
                          nth: int = 1) -> int:
    """The hook with host tensors; returns 1 (dst written) or 0 (caller falls back)."""
    return int(lib().mlzc_try_mul_mat(C.byref(src0), C.byref(src1), C.byref(dst), ith, nth))


def ggml_simd_try_flash_attn(desc: FaDesc, ith: int = 0, nth: int = 1) -> int:
    return int(lib().mlzc_try_flash_attn(C.byref(desc), ith, nth))


def init(device: int = 0) -> None:
    check(lib().mlzc_init(device))


def shutdown() -> None:
    check(lib().mlzc_shutdown())


def device_errors(device: int = 0) -> int:
    v = C.c_uint32(0)
    check(lib().mlzc_device_errors(device, C.byref(v)))
    return v.value


def selftest_wait_timeout(device: int = 0, limit_us: int = 20000) -> bool:
    """Runs the bounded-wait failure path once (mlzc_selftest_wait_timeout): a kernel waits
    on an mbarrier nothing arrives on and must give up after ``limit_us``.  Returns True
    when it gave up; the device error word then holds MLZC_DEVERR_WAIT_TIMEOUT."""
    v = C.c_int32(0)
    check(lib().mlzc_selftest_wait_timeout(device, limit_us, C.byref(v)))
    return bool(v.value)


class Weight:
    """Device-resident weight matrix for host-pointer calls (mlzc_weight)."""

    def __init__(self, w: np.ndarray, w_type: int, K: int, device: int = 0):
        self.M = w.shape[0]
        self.K = K
        self.w_type = w_type
        self._h = C.c_void_p()
        check(lib().mlzc_weight_upload(device, w_type, w.ctypes.data, w.strides[0], self.M, K,
                                       C.byref(self._h)))

    def mul_mat(self, x: np.ndarray, out: Optional[np.ndarray] = None) -> np.ndarray:
        N = x.shape[0]
        if out is None:
            out = np.empty((N, self.M), dtype=np.float32)
        check(lib().mlzc_mul_mat(self._h, x.ctypes.data, x.strides[0], N, out.ctypes.data, out.strides[0]))
        return out

    def mul_mat_ptr(self, x_ptr: int, x_col_bytes: int, N: int, y_ptr: int, y_col_bytes: int) -> None:
        check(lib().mlzc_mul_mat(self._h, x_ptr, x_col_bytes, N, y_ptr, y_col_bytes))

    def free(self) -> None:
        if self._h:
            lib().mlzc_weight_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Comm:
    """NCCL communicator of the row-sharded mul_mat (one process per GPU)."""

    def __init__(self, nranks: int, rank: int, device: int, unique_id: bytes, timeout_ms: int = 60000):
        self.nranks, self.rank, self.device = nranks, rank, device
        self._h = C.c_void_p()
        buf = C.create_string_buffer(unique_id, 128)
        check(lib().mlzc_comm_init(nranks, rank, device, buf, timeout_ms, C.byref(self._h)))

    @staticmethod
    def unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        check(lib().mlzc_comm_unique_id(buf))
        return buf.raw

    def workspace_bytes(self, w_type: int, M_total: int, K: int, N: int) -> int:
        out = C.c_size_t(0)
        check(lib().mlzc_mul_mat_sharded_workspace_bytes(self._h, w_type, M_total, K, N, C.byref(out)))
        return out.value

    def mul_mat_sharded(self, w_shard, x, M_total: int, *, out=None, workspace=None, stream=None):
        torch = _torch()
        w_type = weight_type_of(w_shard)
        N, K = x.shape
        if out is None:
            out = torch.empty((N, M_total), dtype=torch.float32, device=x.device)
        wsb = self.workspace_bytes(w_type, M_total, K, N)
        if workspace is None:
            workspace = torch.empty(max(wsb, 1), dtype=torch.uint8, device=x.device)
        check(lib().mlzc_mul_mat_sharded_dev(
            self._h, w_type, w_shard.data_ptr(), w_shard.stride(0) * w_shard.element_size(), M_total, K,
            x.data_ptr(), x.stride(0) * 4, N, out.data_ptr(), out.stride(0) * 4,
            workspace.data_ptr(), workspace.numel(), _stream_handle(stream)))
        return out

    def destroy(self) -> None:
        if self._h:
            lib().mlzc_comm_destroy(self._h)
            self._h = C.c_void_p()


__all__ = [
    "mul_mat", "mul_mat_workspace_bytes", "flash_attn_dispatch", "flash_attn_workspace_bytes",
    "make_fa_desc", "tensor_view", "ggml_simd_try_mul_mat", "ggml_simd_try_flash_attn", "init",
    "shutdown", "device_errors", "Weight", "Comm", "MlzcError", "weight_type_of",
    "TYPE_F16", "TYPE_F32", "TYPE_Q4_K", "TYPE_Q6_K",
]
