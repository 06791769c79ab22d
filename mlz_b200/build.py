"""Builds mlz_b200/libmlzc.so from mlz_b200/csrc with nvcc for sm_100a (in-tree).

Usage: ``python mlz_b200/build.py [--force]`` (runs without importing the package,
whose import needs the built library).  Object files go to mlz_b200/_build/.
Compiles on a machine without a GPU (nvcc cross-compiles); the .so is what ships.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libmlzc.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cuda_home() -> str:
    env = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if env and os.path.exists(os.path.join(env, "bin", "nvcc")):
        return env
    nvcc = shutil.which("nvcc")
    if nvcc:
        return os.path.dirname(os.path.dirname(os.path.realpath(nvcc)))
    return "/usr/local/cuda"


def _nccl_include() -> list[str]:
    for d in ("/usr/include", os.path.join(_cuda_home(), "include")):
        if os.path.exists(os.path.join(d, "nccl.h")):
            return ["-I" + d]
    try:  # torch wheels ship the header next to their NCCL
        import nvidia.nccl  # type: ignore
        for p in nvidia.nccl.__path__:
            inc = os.path.join(p, "include")
            if os.path.exists(os.path.join(inc, "nccl.h")):
                return ["-I" + inc]
    except Exception:
        pass
    raise RuntimeError("nccl.h not found")


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _compile_cmd(src: str, obj: str) -> list[str]:
    cuda = _cuda_home()
    if src.endswith(".cu"):
        return [os.path.join(cuda, "bin", "nvcc"), *ARCH, "-O3", "-lineinfo", "-std=c++17",
                "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-Wall", "-I" + INCLUDE,
                *_nccl_include(), "-c", src, "-o", obj]
    return ["g++", "-O2", "-fPIC", "-std=c++17", "-Wall", "-I" + INCLUDE,
            "-I" + os.path.join(cuda, "include"), *_nccl_include(), "-c", src, "-o", obj]


def _stale(obj: str, src: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src, *_headers()])


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    srcs = _sources()
    objs = [os.path.join(OUT_DIR, os.path.basename(s) + ".o") for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or _stale(o, s)]

    def run(pair):
        s, o = pair
        cmd = _compile_cmd(s, o)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return s, cmd, r

    failed = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for s, cmd, r in ex.map(run, todo):
            if verbose or r.returncode != 0:
                sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
            if r.returncode != 0:
                failed.append(s)
    if failed:
        raise RuntimeError("compilation failed: " + ", ".join(os.path.basename(f) for f in failed))
    if force or todo or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cuda = _cuda_home()
        cmd = [os.path.join(cuda, "bin", "nvcc"), *ARCH, "-shared", "-o", LIB, *objs,
               "-cudart", "static", "-ldl", "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
