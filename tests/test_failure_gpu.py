"""GPU: the failure-detection paths, exercised without any GPU fault.

(a) a device wait that nothing completes gives up after its bound, sets
    MLZC_DEVERR_WAIT_TIMEOUT and returns (the same bounded wait every kernel uses);
(b) a communicator whose peer never joins fails with MLZC_ERR_COMM within its timeout
    (host-side: rank 0 of 2 alone, in a child process);
(c) an out-of-range device id is refused;
(d) a call whose workspace is too small is refused with MLZC_ERR_NOMEM before any launch.
"""
import ctypes as C
import os
import subprocess
import sys
import time

import numpy as np
import pytest

import mlz_b200
import oracle
from mlz_b200 import synth
from mlz_b200.ops import _nb

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_bounded_wait_gives_up_and_reports(dev):
    import torch
    assert mlz_b200.device_errors(0) == 0
    t0 = time.perf_counter()
    assert mlz_b200.selftest_wait_timeout(0, 20000)        # 20 ms bound
    dt = time.perf_counter() - t0
    assert dt < 5.0
    assert mlz_b200.device_errors(0) == 0x1               # MLZC_DEVERR_WAIT_TIMEOUT, now cleared
    assert mlz_b200.device_errors(0) == 0
    # the context is still usable: a mul_mat after the expired wait is correct
    g = synth.rng(31)
    w = synth.f16_weights(g, 256, 512)
    x = synth.f32_acts(g, 3, 512)
    y = mlz_b200.mul_mat(torch.from_numpy(w).to(dev), torch.from_numpy(x).to(dev))
    torch.cuda.synchronize()
    assert oracle.rel_err(y.cpu().numpy(), oracle.mul_mat_f16(w.view(np.uint16), x)) <= 1e-3
    with pytest.raises(mlz_b200.MlzcError):
        mlz_b200.selftest_wait_timeout(0, 0)               # limit out of range


_LONELY_RANK = r"""
import ctypes as C, sys, time
sys.path.insert(0, %r)
import mlz_b200
L = mlz_b200.lib()
idb = C.create_string_buffer(128)
assert L.mlzc_comm_unique_id(idb) == 0
h = C.c_void_p()
t0 = time.perf_counter()
st = L.mlzc_comm_init(2, 0, 0, idb, 2000, C.byref(h))
dt = time.perf_counter() - t0
print("STATUS", st, "%%.2f" %% dt, mlz_b200.last_error())
"""


def test_comm_init_without_peer_times_out():
    """Rank 0 of a 2-rank communicator whose rank 1 never starts: mlzc_comm_init must
    return MLZC_ERR_COMM once its 2 s timeout passes (the communicator is aborted), not
    wait forever.  Runs in a child process so that a stuck NCCL could only cost this test."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", _LONELY_RANK % ROOT], capture_output=True, text=True,
                       env=env, timeout=120)
    line = [l for l in r.stdout.splitlines() if l.startswith("STATUS")]
    assert line, r.stdout[-2000:] + r.stderr[-2000:]
    _, st, dt, *msg = line[0].split()
    assert int(st) == -6, line[0]                           # MLZC_ERR_COMM
    assert 1.9 <= float(dt) < 60.0, line[0]
    assert "aborted" in " ".join(msg) or "timeout" in " ".join(msg).lower(), line[0]


def test_bad_device_ids_are_refused(dev):
    import torch
    L = mlz_b200.lib()
    for bad in (-1, torch.cuda.device_count(), 1000):
        assert L.mlzc_init(bad) == -1                       # MLZC_ERR_INVALID
        assert "out of range" in mlz_b200.last_error()
        v = C.c_uint32(0)
        assert L.mlzc_device_errors(bad, C.byref(v)) == -1


def test_too_small_workspaces_are_refused_before_launch(dev):
    import torch
    L = mlz_b200.lib()
    n0 = mlz_b200.launch_count()
    # flash attention
    g = synth.rng(32)
    q, k, v = synth.fa_inputs(g, 2, 8, 2, 300, 128)
    q, k, v = (torch.from_numpy(a).to(dev) for a in (q, k, v))
    out = torch.zeros((2, 8, 1, 128), device=dev)
    d = mlz_b200.make_fa_desc(q.data_ptr(), _nb(q, 4), k.data_ptr(), _nb(k, 2), v.data_ptr(), _nb(v, 2),
                              out.data_ptr(), _nb(out, 4), (2, 8, 1, 2, 300, 128), 1 / np.sqrt(128))
    need = mlz_b200.flash_attn_workspace_bytes(d)
    assert need > 0
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    assert L.mlzc_flash_attn_dev(C.byref(d), ws.data_ptr(), need - 16, None) == -4   # MLZC_ERR_NOMEM
    assert "workspace" in mlz_b200.last_error()
    assert L.mlzc_flash_attn_dev(C.byref(d), None, 0, None) == -4
    # tensor-core GEMM (N = 64 needs the narrowed-activation workspace)
    w = torch.zeros((256, 512), dtype=torch.float16, device=dev)
    x = torch.zeros((64, 512), device=dev)
    y = torch.zeros((64, 256), device=dev)
    need = mlz_b200.mul_mat_workspace_bytes(mlz_b200.TYPE_F16, 256, 512, 64)
    assert need > 0
    st = L.mlzc_mul_mat_dev(mlz_b200.TYPE_F16, w.data_ptr(), 1024, 256, 512, x.data_ptr(), 2048, 64,
                            y.data_ptr(), 1024, ws.data_ptr(), need - 1, None)
    assert st == -4
    torch.cuda.synchronize()
    assert mlz_b200.launch_count() == n0                    # nothing was launched
