"""ctypes binding of libmlzc.so (the C ABI declared in include/mlzc.h).

Loading fails loudly: there is no CPU fallback anywhere in this package.  If the shared
library is missing it must be built first (``python mlz_b200/build.py``).
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmlzc.so")

MLZC_OK = 0
STATUS_NAMES = {
    0: "MLZC_OK", -1: "MLZC_ERR_INVALID", -2: "MLZC_ERR_UNSUPPORTED", -3: "MLZC_ERR_CUDA",
    -4: "MLZC_ERR_NOMEM", -5: "MLZC_ERR_DEVICE", -6: "MLZC_ERR_COMM",
}
TYPE_F32, TYPE_F16, TYPE_Q4_K, TYPE_Q6_K = 0, 1, 12, 14
TYPE_Q4_0, TYPE_Q8_0 = 2, 8
TYPE_Q4_1, TYPE_Q5_0, TYPE_Q5_1, TYPE_IQ4_NL = 3, 6, 7, 20   # quantised KV-cache types
FA_MODE_GQA_BATCH, FA_MODE_ALIBI, FA_MODE_SOFTCAP = 0x04, 0x08, 0x10
OVERLAP_OFF, OVERLAP_SAFE, OVERLAP_WEIGHTS = 0, 1, 2
UNIQUE_ID_BYTES = 128

# every symbol include/mlzc.h declares (checked by the CPU test suite)
EXPORTS = (
    "mlzc_launch_count", "mlzc_last_error", "mlzc_version", "mlzc_init", "mlzc_shutdown", "mlzc_device_errors",
    "mlzc_selftest_wait_timeout",
    "mlzc_set_launch_overlap", "mlzc_get_launch_overlap",
    "mlzc_mul_mat_workspace_bytes", "mlzc_mul_mat_dev", "mlzc_quantize_q8k_dev",
    "mlzc_flash_attn_workspace_bytes", "mlzc_flash_attn_dev", "mlzc_flash_attn_dev_noalloc",
    "mlzc_try_mul_mat", "mlzc_try_flash_attn",
    "mlzc_weight_upload", "mlzc_weight_free", "mlzc_mul_mat", "mlzc_weight_cache_clear",
    "mlzc_host_register", "mlzc_host_unregister",
    "mlzc_comm_unique_id", "mlzc_comm_init", "mlzc_comm_destroy",
    "mlzc_mul_mat_sharded_workspace_bytes", "mlzc_mul_mat_sharded_dev",
)


class MlzcError(RuntimeError):
    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


class FaDesc(C.Structure):
    """Mirror of mlzc_fa_desc."""
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
        ("k_type", C.c_int32), ("v_type", C.c_int32),
        ("kv_len", C.c_void_p),
    ]


class TensorView(C.Structure):
    """Mirror of mlzc_tensor (the part of struct ggml_tensor the hook reads)."""
    _fields_ = [("type", C.c_int32), ("ne", C.c_int64 * 4), ("nb", C.c_size_t * 4), ("data", C.c_void_p)]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python mlz_b200/build.py`")
        L = C.CDLL(LIB_PATH)
        _declare(L)
        _lib = L
    return _lib


def _declare(L: C.CDLL) -> None:
    vp, i64, sz, i32, u32 = C.c_void_p, C.c_int64, C.c_size_t, C.c_int, C.c_uint32
    psz = C.POINTER(C.c_size_t)
    for name in EXPORTS:
        getattr(L, name).restype = C.c_int
    L.mlzc_launch_count.argtypes = [C.POINTER(C.c_uint64)]
    L.mlzc_set_launch_overlap.argtypes = [i32]
    L.mlzc_get_launch_overlap.argtypes = [C.POINTER(i32)]
    L.mlzc_last_error.restype = C.c_char_p
    L.mlzc_last_error.argtypes = []
    L.mlzc_version.argtypes = []
    L.mlzc_init.argtypes = [i32]
    L.mlzc_shutdown.argtypes = []
    L.mlzc_device_errors.argtypes = [i32, C.POINTER(u32)]
    L.mlzc_selftest_wait_timeout.argtypes = [i32, u32, C.POINTER(i32)]
    L.mlzc_mul_mat_workspace_bytes.argtypes = [i32, i64, i64, i64, psz]
    L.mlzc_mul_mat_dev.argtypes = [i32, vp, sz, i64, i64, vp, sz, i64, vp, sz, vp, sz, vp]
    L.mlzc_quantize_q8k_dev.argtypes = [vp, sz, i64, i64, vp, sz, vp]
    L.mlzc_flash_attn_workspace_bytes.argtypes = [C.POINTER(FaDesc), psz]
    L.mlzc_flash_attn_dev.argtypes = [C.POINTER(FaDesc), vp, sz, vp]
    L.mlzc_flash_attn_dev_noalloc.argtypes = [C.POINTER(FaDesc), vp]
    L.mlzc_try_mul_mat.argtypes = [C.POINTER(TensorView)] * 3 + [i32, i32]
    L.mlzc_try_flash_attn.argtypes = [C.POINTER(FaDesc), i32, i32]
    L.mlzc_weight_upload.argtypes = [i32, i32, vp, sz, i64, i64, C.POINTER(vp)]
    L.mlzc_weight_free.argtypes = [vp]
    L.mlzc_mul_mat.argtypes = [vp, vp, sz, i64, vp, sz]
    L.mlzc_weight_cache_clear.argtypes = []
    L.mlzc_host_register.argtypes = [vp, sz]
    L.mlzc_host_unregister.argtypes = [vp]
    L.mlzc_comm_unique_id.argtypes = [vp]
    L.mlzc_comm_init.argtypes = [i32, i32, i32, vp, i32, C.POINTER(vp)]
    L.mlzc_comm_destroy.argtypes = [vp]
    L.mlzc_mul_mat_sharded_workspace_bytes.argtypes = [vp, i32, i64, i64, i64, psz]
    L.mlzc_mul_mat_sharded_dev.argtypes = [vp, i32, vp, sz, i64, i64, vp, sz, i64, vp, sz, vp, sz, vp]


def launch_count() -> int:
    v = C.c_uint64(0)
    check(lib().mlzc_launch_count(C.byref(v)))
    return v.value


def set_launch_overlap(mode: int) -> None:
    """OVERLAP_OFF / OVERLAP_SAFE (default) / OVERLAP_WEIGHTS, process-wide (see mlzc.h)."""
    check(lib().mlzc_set_launch_overlap(mode))


def get_launch_overlap() -> int:
    v = C.c_int32(0)
    check(lib().mlzc_get_launch_overlap(C.byref(v)))
    return v.value


def last_error() -> str:
    return lib().mlzc_last_error().decode(errors="replace")


def check(status: int) -> int:
    if status < 0:
        raise MlzcError(status, last_error())
    return status
