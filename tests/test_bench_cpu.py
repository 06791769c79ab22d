"""CPU: the bench's reference arm runs the oracle's restatement of the reference kernels
alone -- it maps none of this repository's CUDA library -- and names the same workload
and metric as the GPU arm."""
import json
import os
import subprocess
import sys

from tests.conftest import ROOT

_PROBE = r"""
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--config", "%s", "--n", "%d", "--steps", "1",
            "--warmup", "0", "--cpu-seconds", "0.1"]
runpy.run_path("bench.py", run_name="__main__")
maps = open("/proc/self/maps").read()
print("MAPPED", "libmlzc" in maps, "liboracle" in maps)
"""


def test_reference_arm_maps_only_the_oracle():
    out = subprocess.run([sys.executable, "-c", _PROBE % ("c1", 1)], cwd=ROOT, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = out.stdout.splitlines()
    d = json.loads([l for l in lines if l.startswith("{")][0])
    assert [l for l in lines if l.startswith("MAPPED")][0] == "MAPPED False True"
    sys.path.insert(0, ROOT)
    import bench
    assert d["config"]["workload"] == bench.workload_name("c1", 1, 1)
    assert d["metric"] == bench.metric_name("c1", 1, 1)
    assert d["unit"] == "GB/s" and d["value"] > 0


def test_workload_names_agree_between_arms():
    sys.path.insert(0, ROOT)
    import bench
    for cfg, n in (("c1", 8), ("c2", 2048), ("c3", 4), ("c4", 16), ("c5", 256)):
        assert bench.workload_name(cfg, n, 1).startswith(cfg)
        assert bench.metric_name(cfg, n, 1)
    assert "sum L = " in bench.workload_name("c4", 16, 1)


def test_c7_reference_arm_per_kv_type():
    """The reference arm of c7 times the same KV-cache type as the GPU arm (--kv-type) and
    names it in the metric, the workload and the dtype."""
    probe = r"""
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--config", "c7", "--kv-type", "q5_1", "--steps", "1",
            "--warmup", "0", "--cpu-seconds", "0.1"]
runpy.run_path("bench.py", run_name="__main__")
"""
    out = subprocess.run([sys.executable, "-c", probe], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads([l for l in out.stdout.splitlines() if l.startswith("{")][0])
    assert "Q5_1 KV" in d["metric"] and "Q5_1 KV cache" in d["config"]["workload"]
    assert d["dtype"] == "q5_1 kv / f32" and d["value"] > 0
