"""CPU: the C-ABI library loads, exports every symbol include/mlzc.h declares, and its
argument gates answer without touching a GPU."""
import ctypes as C
import os
import re
import subprocess
import threading

import numpy as np

import mlz_b200
from mlz_b200 import synth
from tests.conftest import ROOT


def _header_functions():
    text = open(os.path.join(ROOT, "include", "mlzc.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(mlzc_[a-z0-9_]+)\s*\(", text))


def test_header_and_exports_agree():
    declared = _header_functions()
    assert declared == set(mlz_b200.EXPORTS)
    out = subprocess.run(["nm", "-D", "--defined-only", mlz_b200.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = declared - exported
    assert not missing, missing


def test_version_and_error_string():
    L = mlz_b200.lib()
    assert L.mlzc_version() == 1
    st = L.mlzc_mul_mat_dev(7, None, 0, 4, 4, None, 16, 1, None, 16, None, 0, None)
    assert st == -2  # MLZC_ERR_UNSUPPORTED
    assert "weight type 7" in mlz_b200.last_error()


def test_launch_overlap_mode():
    assert mlz_b200.get_launch_overlap() == mlz_b200.OVERLAP_SAFE   # the default
    try:
        for m in (mlz_b200.OVERLAP_OFF, mlz_b200.OVERLAP_WEIGHTS, mlz_b200.OVERLAP_SAFE):
            mlz_b200.set_launch_overlap(m)
            assert mlz_b200.get_launch_overlap() == m
        for bad in (-1, 3):
            try:
                mlz_b200.set_launch_overlap(bad)
                raise AssertionError("mode %d accepted" % bad)
            except mlz_b200.MlzcError as e:
                assert e.status == -1
        assert mlz_b200.get_launch_overlap() == mlz_b200.OVERLAP_SAFE
    finally:
        mlz_b200.set_launch_overlap(mlz_b200.OVERLAP_SAFE)


def test_q4k_workspace_follows_the_dispatch():
    """Host arithmetic only: every Q4_K path reads prepared activations from the workspace.
    N <= 4 (int8 path): per 8 blocks a record of 2 int8 vectors (2080 B each), 8 scales and
    8 x 2 f16 sub-block sums per column (columns padded to 1, 2 or 4); independent of M."""
    ws = lambda M, K, N: mlz_b200.mul_mat_workspace_bytes(mlz_b200.TYPE_Q4_K, M, K, N)
    for N, nct in ((1, 1), (2, 2), (3, 4), (4, 4)):
        for K in (256, 4096, 14336):
            rec = (K // 256 + 7) // 8 * (2 * nct * 2080 + nct * 32 + 8 * 2 * nct * 16)
            assert ws(4096, K, N) >= rec
            assert ws(1, K, N) == ws(14336, K, N)
    for N in (5, 8, 9, 16, 63):
        for K in (256, 4096, 14336):
            # f16 fragments (512 B per column and block) + sums (32 B); columns padded to a
            # whole 8-column tile, or pairs of them above 8
            pad = 8 if N <= 8 else (N + 15) // 16 * 16
            assert ws(4096, K, N) >= pad * (K // 256) * (512 + 32)
    for N in (64, 256):
        for K in (1024, 4096, 14336):
            # prefill sizes of matrices of >= 4 M weights: the rows dequantised to f16 (2 B per
            # weight) + the GEMM's share
            assert ws(4096, K, N) >= 4096 * K * 2
            assert mlz_b200.mul_mat_workspace_bytes(mlz_b200.TYPE_Q6_K, 4096, K, N) >= 4096 * K * 2


def test_argument_gates():
    L = mlz_b200.lib()
    # Q4_K with K not a multiple of 256
    st = L.mlzc_mul_mat_dev(mlz_b200.TYPE_Q4_K, C.c_void_p(16), 144, 4, 300, C.c_void_p(16), 1200, 1,
                            C.c_void_p(16), 16, None, 0, None)
    assert st == -1 and "256" in mlz_b200.last_error()
    # row stride shorter than a row
    st = L.mlzc_mul_mat_dev(mlz_b200.TYPE_F16, C.c_void_p(16), 8, 4, 8, C.c_void_p(16), 32, 1,
                            C.c_void_p(16), 16, None, 0, None)
    assert st == -1 and "w_row_bytes" in mlz_b200.last_error()
    # workspace query is pure host arithmetic
    assert mlz_b200.mul_mat_workspace_bytes(mlz_b200.TYPE_F32, 64, 64, 1) == 0


def test_fa_gate_rejects_unsupported_layouts():
    d = mlz_b200.make_fa_desc(16, (4, 512, 512, 4096), 16, (2, 256, 2560, 20480), 16, (2, 256, 2560, 20480),
                              16, (4, 512, 512, 4096), (1, 4, 1, 2, 10, 96), 0.1)
    out = C.c_size_t(0)
    assert mlz_b200.lib().mlzc_flash_attn_workspace_bytes(C.byref(d), C.byref(out)) == -2  # head_dim 96
    d.head_dim_k = d.head_dim_v = 128
    d.k_type = 0
    assert mlz_b200.lib().mlzc_flash_attn_workspace_bytes(C.byref(d), C.byref(out)) == -2  # F32 K


def test_hook_gate_declines_untaken_types_on_every_thread():
    # Q8_0 weights (type 8) are not handled: every thread gets 0 without any device work
    w = np.zeros((4, 34), dtype=np.uint8)
    x = np.zeros((1, 32), dtype=np.float32)
    y = np.zeros((1, 4), dtype=np.float32)
    s0 = mlz_b200.tensor_view(w, 8, ne0=32)
    s1 = mlz_b200.tensor_view(x, mlz_b200.TYPE_F32)
    d = mlz_b200.tensor_view(y, mlz_b200.TYPE_F32)
    assert mlz_b200.ggml_simd_try_mul_mat(s0, s1, d, 0, 1) == 0


def test_hook_threads_agree_on_fallback_without_gpu():
    """nth ggml threads enter the hook for the same node; on a host without a usable GPU
    thread 0's device work fails and all nth threads must return the same 0 (no thread
    may return 1 and skip the shared CPU fallback), without deadlock."""
    import torch
    if torch.cuda.is_available():
        return  # covered by the GPU hook tests on a real device
    g = synth.rng(4)
    w = synth.f16_weights(g, 32, 64)
    x = synth.f32_acts(g, 2, 64)
    y = np.zeros((2, 32), dtype=np.float32)
    s0 = mlz_b200.tensor_view(w, mlz_b200.TYPE_F16)
    s1 = mlz_b200.tensor_view(x, mlz_b200.TYPE_F32)
    d = mlz_b200.tensor_view(y, mlz_b200.TYPE_F32)
    for nth in (1, 4, 8):
        results = [None] * nth
        def run(i):
            results[i] = mlz_b200.ggml_simd_try_mul_mat(s0, s1, d, i, nth)
        ts = [threading.Thread(target=run, args=(i,)) for i in range(nth)]
        for t in ts[::-1]:
            t.start()
        for t in ts:
            t.join(timeout=30)
        assert all(not t.is_alive() for t in ts)
        assert results == [0] * nth


def test_init_and_error_word_without_a_gpu_fail_with_a_status():
    """On a host without a usable GPU the runtime entry points return a status (no abort),
    with a message naming the failing CUDA call."""
    import torch
    if torch.cuda.is_available():
        return  # the GPU failure tests cover a real device
    L = mlz_b200.lib()
    assert L.mlzc_init(0) == -3                               # MLZC_ERR_CUDA
    assert "cudaGetDeviceCount" in mlz_b200.last_error()
    v = C.c_uint32(0)
    assert L.mlzc_device_errors(0, C.byref(v)) == -3
    g = C.c_int32(0)
    assert L.mlzc_selftest_wait_timeout(0, 1000, C.byref(g)) == -3
