"""B200-native (sm_100a) implementation of MLz's src/simd hot path.

The compute lives in ``libmlzc.so`` (CUDA kernels + C ABI, see include/mlzc.h); this
package is the host-side mirror of the reference's dispatch interface over that ABI.
The library is loaded by the first call that needs it (or by :func:`lib`), and that call
raises ImportError if it has not been built -- there is no CPU fallback.  Importing the
package alone maps no native code, so ``mlz_b200.synth`` (the seeded input generators)
can be used by code that must not load the library.
"""
from ._lib import (EXPORTS, FA_MODE_ALIBI, FA_MODE_GQA_BATCH, FA_MODE_SOFTCAP, LIB_PATH,
                   OVERLAP_OFF, OVERLAP_SAFE, OVERLAP_WEIGHTS, TYPE_F16, TYPE_F32, TYPE_IQ4_NL, TYPE_Q4_0, TYPE_Q4_1,
                   TYPE_Q4_K, TYPE_Q5_0, TYPE_Q5_1, TYPE_Q6_K, TYPE_Q8_0,
                   UNIQUE_ID_BYTES, FaDesc, MlzcError, TensorView, check, get_launch_overlap,
                   last_error, launch_count, lib, set_launch_overlap)
from .ops import (Comm, Weight, device_errors, flash_attn_dispatch, flash_attn_dispatch_quant,
                  flash_attn_workspace_bytes,
                  ggml_simd_try_flash_attn, ggml_simd_try_mul_mat, init, make_fa_desc, mul_mat,
                  mul_mat_workspace_bytes, quantize_q8k, selftest_wait_timeout, shutdown, tensor_view,
                  weight_type_of)

__all__ = [
    "EXPORTS", "FA_MODE_ALIBI", "FA_MODE_GQA_BATCH", "FA_MODE_SOFTCAP", "LIB_PATH", "OVERLAP_OFF",
    "OVERLAP_SAFE", "OVERLAP_WEIGHTS", "get_launch_overlap", "set_launch_overlap", "TYPE_F16",
    "TYPE_F32", "TYPE_IQ4_NL", "TYPE_Q4_0", "TYPE_Q4_1", "TYPE_Q4_K", "TYPE_Q5_0", "TYPE_Q5_1",
    "TYPE_Q6_K", "TYPE_Q8_0", "UNIQUE_ID_BYTES", "FaDesc", "MlzcError", "TensorView", "check",
    "last_error", "launch_count", "lib", "Comm", "Weight", "device_errors", "flash_attn_dispatch", "flash_attn_dispatch_quant",
    "flash_attn_workspace_bytes", "ggml_simd_try_flash_attn", "ggml_simd_try_mul_mat", "init",
    "make_fa_desc", "mul_mat", "mul_mat_workspace_bytes", "quantize_q8k", "selftest_wait_timeout", "shutdown", "tensor_view",
    "weight_type_of",
]
