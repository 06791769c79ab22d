#!/usr/bin/env python3
"""Benchmark of the MLz src/simd hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1..c5] [--n N]
                    [--impl mlz|reference]

Workloads (synthetic seeded inputs of the named shapes; random-init weights):
  c1  F16 mul_mat, Llama-3.2-3B FFN up-proj: W 8192x3072 f16, X 3072xN f32, N in {1,8,32}
  c2  prefill GEMM of one Llama-3.2-3B layer: 7 F16 projections (Q 3072^2, K/V 1024x3072,
      O 3072^2, gate/up 8192x3072, down 3072x8192) over M tokens, M in {512, 2048}
  c3  Q4_K decode mul_mat on Llama-3.1-8B shapes 4096x4096, 14336x4096, 4096x14336, batch N
  c4  flash-attention decode, 16 sequences, L ~ U{512..8192}, 32 q / 8 kv heads, D = 128
  c5  Llama-3-70B FFN (gate/up 28672x8192, down 8192x28672) row-sharded over the ranks, the
      output slices all-gathered through NVLink peer memory, N in {1, 256}
      (default workload: c5, N = 1, the decode GB/s of the configuration quoted at 1/2/4/8
      GPUs; the line carries measured rows of the other configurations -- every one on one
      GPU, the other c5 size on several)
  c6  Q6_K decode mul_mat on the Llama-3.1-8B shapes of c3, batch N (Q4_K_M files carry
      Q6_K tensors; the reference hook routes them with Q4_K)
  c7  flash-attention decode of c4 over a quantised KV cache (Q8_0; --kv-type q4_0, q4_1,
      q5_0, q5_1 or iq4_nl for the other block types, f32 for an F32 cache)

A step is one pass of the hot path over one batch.  `value` is whole-job throughput with
inputs resident in HBM; `e2e` is the same metric through the reference-facing plugin
(mlzc_try_mul_mat / mlzc_try_flash_attn) with pinned host buffers, copies included.
The reference arm (--impl reference) times the CPU restatement of the reference kernels
(oracle/) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

L2_BYTES = 126 * 1024 * 1024

# DRAM bytes per call of the roofline's call (dram__bytes_read.sum + dram__bytes_write.sum),
# from one ncu capture of the same kernels on the same workload (the capture commands and
# summaries are kept with the profiles).
NCU_TRAFFIC = {
    ("c1", 1): (50.35e6 + 0.02e6, "ncu capture: gemv_vec_kernel, 8192x3072, N=1"),
    ("c1", 4): (50.39e6 + 0.07e6, "ncu capture: gemv_f16_mma_kernel, 8192x3072, N=4"),
    ("c1", 8): (50.44e6 + 0.01e6, "ncu capture: gemv_f16_mma_kernel<1, 1, 4>, 8192x3072, N=8"),
    ("c4", 16): (250.80e6 + 5.98e6, "ncu capture: fa_decode_kernel of the c4 call (16 sequences)"),
    ("c3", 1): (33.14e6, "ncu capture: q4k_i8_kernel, 14336x4096 launch, batch 1 (the 4096x14336 launch reads the "
                         "same block bytes)"),
    ("c6", 1): (48.29e6 + 0.01e6, "ncu capture: q6k_i8_kernel, 14336x4096 launch, batch 1 (the 4096x14336 launch "
                                  "reads the same block bytes)"),
    ("c7", 16): (132.51e6 + 4.60e6, "ncu capture: fa_quant_kernel of the c7 call (16 sequences)"),
    ("c3", 8): (33.29e6, "ncu capture: q4k_ring_xs_kernel, 4096x14336 launch, batch 8 (the 14336x4096 launch "
                         "reads the same block bytes)"),
    ("c3", 16): (33.31e6, "ncu capture: q4k_mma_kernel, 14336x4096 launch, batch 16"),
    ("c5", 1): (469.85e6 + 3.33e6, "ncu capture: gemv_vec_kernel, 28672x8192 gate launch, N=1, one GPU (the "
                                   "8192x28672 down launch reads the same weight bytes)"),
}


def traffic_of(cfg: str, n: int, w, world: int):
    """The committed capture's DRAM bytes for this workload's dominant call, or None: none for
    the pooled c2 calls, and the c5 captures hold one GPU's whole matrix, not a shard."""
    if isinstance(w, C2) or (isinstance(w, C5) and world > 1) or (cfg == "c7" and C7_TYPE["kv"] != "q8_0"):
        return None
    return NCU_TRAFFIC.get((cfg, n))


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c5", choices=["c1", "c2", "c3", "c4", "c5", "c6", "c7"])
    ap.add_argument("--n", "--size", dest="n", type=int, default=None,
                    help="activation columns / tokens / batch (--size under torchrun, whose parser takes --n)")
    ap.add_argument("--impl", default="mlz", choices=["mlz", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-rows", action="store_true",
                    help="measure the headline workload only (no rows of the other configurations)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="target CPU sample length")
    ap.add_argument("--no-graph", action="store_true",
                    help="time the eager launches instead of a CUDA-graph replay of the K steps")
    ap.add_argument("--overlap", default="weights", choices=["off", "safe", "weights"],
                    help="launch overlap of consecutive kernels (mlzc_set_launch_overlap); 'weights' "
                         "is valid here because no kernel of any workload writes the weights")
    ap.add_argument("--kv-type", default="q8_0", choices=sorted(C7_KV),
                    help="c7: the KV-cache block type")
    ap.add_argument("--profile-run", action="store_true",
                    help="for ncu launch lists: no clock-sampling load loop, no e2e, no CPU leg "
                         "(launch order = warm-up steps, then the timed steps)")
    return ap.parse_args()


DEFAULT_N = {"c1": 8, "c2": 2048, "c3": 4, "c4": 16, "c5": 1, "c6": 4, "c7": 16}
# c7's KV-cache block types: name -> ggml type id (block layouts in mlz_b200.synth.KV_QUANT)
C7_KV = {"q8_0": 8, "q4_0": 2, "q4_1": 3, "q5_0": 6, "q5_1": 7, "iq4_nl": 20, "f32": 0}
C7_TYPE = {"kv": "q8_0"}   # set from --kv-type
DTYPE = {"c1": "f16", "c2": "f16", "c3": "q4_k/f32", "c4": "f16 kv / f32", "c5": "f16", "c6": "q6_k/f32",
         "c7": "q8_0 kv / f32"}


def metric_name(cfg: str, n: int, world: int) -> str:
    """`metric` of a line (the same for both arms)."""
    if cfg == "c1":
        return f"decode mul_mat GB/s (F16 W 8192x3072 . X 3072x{n}, fp32 acc)"
    if cfg == "c2":
        return f"prefill mul_mat TFLOP/s (Llama-3.2-3B layer, 7 F16 projections, M={n} tokens, fp32 acc)"
    if cfg == "c3":
        return f"decode Q4_K mul_mat GB/s (Llama-3.1-8B 4096x4096, 14336x4096, 4096x14336; batch {n})"
    if cfg == "c4":
        return f"flash-attention decode GB/s (F16 KV, {n} seqs, L~U[512,8192], 32q/8kv heads, D=128)"
    if cfg == "c6":
        return f"decode Q6_K mul_mat GB/s (Llama-3.1-8B 4096x4096, 14336x4096, 4096x14336; batch {n})"
    if cfg == "c7":
        kv = C7_TYPE["kv"].upper()
        return f"flash-attention decode GB/s ({kv} KV, {n} seqs, L~U[512,8192], 32q/8kv heads, D=128)"
    return (f"sharded FFN mul_mat {'GB/s' if n == 1 else 'TFLOP/s'} (Llama-3-70B gate/up 28672x8192, "
            f"down 8192x28672, F16, N={n}, row-sharded over {world} GPU, all-gather of the slices)")


C2_PROJ = [("q", 3072, 3072, 0), ("k", 1024, 3072, 0), ("v", 1024, 3072, 0), ("o", 3072, 3072, 1),
           ("gate", 8192, 3072, 2), ("up", 8192, 3072, 2), ("down", 3072, 8192, 3)]
C3_SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336)]
C5_MATS = [("gate", 28672, 8192), ("up", 28672, 8192), ("down", 8192, 28672)]


def c4_lengths(n: int):
    from mlz_b200 import synth
    return synth.kv_lengths(synth.rng(synth.seed_for(4, n)), n, 512, 8192)


def workload_name(cfg: str, n: int, world: int) -> str:
    """config.workload of a line; both arms print the same string for the same workload."""
    if cfg == "c1":
        return f"c1 F16 mul_mat Llama-3.2-3B up-proj 8192x3072, N={n}"
    if cfg == "c2":
        return f"c2 Llama-3.2-3B layer prefill, 7 F16 projections, M={n} tokens"
    if cfg == "c3":
        return f"c3 Q4_K mul_mat Llama-3.1-8B shapes, batch {n}"
    if cfg == "c4":
        return f"c4 FA decode GQA, {n} sequences, sum L = {int(c4_lengths(n).sum())}"
    if cfg == "c6":
        return f"c6 Q6_K mul_mat Llama-3.1-8B shapes, batch {n}"
    if cfg == "c7":
        kv = C7_TYPE["kv"].upper()
        return f"c7 FA decode GQA over a {kv} KV cache, {n} sequences, sum L = {int(c4_lengths(n).sum())}"
    return f"c5 Llama-3-70B FFN, N={n}, row-sharded x{world}"


def load_peaks():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# --------------------------------------------------------------------------- workloads

class Workload:
    """A configuration: device operands, one step, and its algorithmic work."""
    metric = ""
    unit = ""
    bound = "hbm"
    scaling = "weak"
    dtype = "f16"

    def work_units(self) -> float:        # bytes (GB/s metrics) or flops (TFLOP/s) per step per rank
        raise NotImplementedError

    def unit_scale(self) -> float:        # units/s -> metric unit
        return 1e-9 if self.unit == "GB/s" else 1e-12

    def roofline_kernel(self, j: int) -> str:  # what the roofline's call runs
        return f"call {j} of the step"


def _rot_copies(nbytes: int) -> int:
    return max(1, math.ceil(4 * L2_BYTES / max(nbytes, 1)))


class C1(Workload):
    unit = "GB/s"
    bound = "hbm"

    def roofline_kernel(self, j):
        # the library's dispatch (gemv_f16_mma_applicable, use_gemm)
        if self.N == 1:
            return "gemv_vec_kernel (one call, one launch)"
        if self.N <= 16:
            return "gemv_f16_mma_kernel (one call, one launch)"
        return "one mul_mat call: narrow_f16_kernel + gemm_f16_tc_kernel"

    def __init__(self, n, dev, gen):
        import torch
        from mlz_b200 import synth
        self.M, self.K, self.N = 8192, 3072, n
        self.metric = metric_name("c1", n, 1)
        self.R = _rot_copies(2 * self.M * self.K)
        self.W = [synth.f16_weights_dev(gen, self.M, self.K, dev) for _ in range(self.R)]
        self.X = synth.f32_acts_dev(gen, n, self.K, dev)
        self.Y = torch.empty((n, self.M), dtype=torch.float32, device=dev)
        import mlz_b200
        wsb = mlz_b200.mul_mat_workspace_bytes(mlz_b200.TYPE_F16, self.M, self.K, n)
        self.ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
        self.config = {"workload": workload_name("c1", n, 1),
                       "M": self.M, "K": self.K, "N": n,
                       "l2": f"rotates {self.R} weight copies ({self.R * 2 * self.M * self.K / 1e6:.0f} MB >= 4x L2)"}

    def work_units(self):
        return 2 * self.M * self.K + 4 * self.K * self.N + 4 * self.M * self.N

    def launches(self, i):
        import mlz_b200
        W = self.W[i % self.R]
        return [(lambda W=W: mlz_b200.mul_mat(W, self.X, out=self.Y, workspace=self.ws), self.work_units())]

    def host_weights(self):
        import numpy as np
        self.hW = self.W[0].cpu().numpy()
        return [(self.hW, 1, self.K)]

    def e2e_calls(self, pinned):
        import torch
        x = self.X.cpu().pin_memory()
        y = torch.empty((self.N, self.M), dtype=torch.float32).pin_memory()
        pinned.extend([x, y])
        return [(0, x, y)], x.numel() * 4, y.numel() * 4


class C2(Workload):
    unit = "TFLOP/s"
    bound = "tensor"
    PROJ = C2_PROJ

    def roofline_kernel(self, j):
        return "the 7 mul_mat calls pooled (narrow_f16_kernel + gemm_f16_tc_kernel each)"

    def __init__(self, n, dev, gen):
        import torch
        import mlz_b200
        from mlz_b200 import synth
        self.Mtok = n
        self.metric = metric_name("c2", n, 1)
        self.W = [synth.f16_weights_dev(gen, o, i, dev) for (_, o, i, _) in self.PROJ]
        ins = [3072, 3072, 3072, 8192]
        self.X = [synth.f32_acts_dev(gen, n, k, dev) for k in ins]
        self.Y = [torch.empty((n, o), dtype=torch.float32, device=dev) for (_, o, _, _) in self.PROJ]
        wsb = max(mlz_b200.mul_mat_workspace_bytes(mlz_b200.TYPE_F16, o, i, n) for (_, o, i, _) in self.PROJ)
        self.ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
        self.config = {"workload": workload_name("c2", n, 1),
                       "tokens": n, "projections": "q,k,v,o 3072/1024x3072; gate,up 8192x3072; down 3072x8192",
                       "l2": "inputs larger than L2 (201 MB of weights per step)"}

    def work_units(self):
        return sum(2.0 * self.Mtok * o * i for (_, o, i, _) in self.PROJ)

    def launches(self, i):
        import mlz_b200
        out = []
        for j, (_, o, k, xi) in enumerate(self.PROJ):
            out.append((lambda j=j, xi=xi: mlz_b200.mul_mat(self.W[j], self.X[xi], out=self.Y[j], workspace=self.ws),
                        2.0 * self.Mtok * o * k))
        return out

    def host_weights(self):
        self.hW = [w.cpu().numpy() for w in self.W]
        return [(w, 1, w.shape[1]) for w in self.hW]

    def e2e_calls(self, pinned):
        import torch
        xs = [x.cpu().pin_memory() for x in self.X]
        ys = [torch.empty(y.shape, dtype=torch.float32).pin_memory() for y in self.Y]
        pinned.extend(xs + ys)
        calls = [(j, xs[xi], ys[j]) for j, (_, _, _, xi) in enumerate(self.PROJ)]
        h2d = sum(xs[xi].numel() * 4 for (_, _, _, xi) in self.PROJ)
        d2h = sum(y.numel() * 4 for y in ys)
        return calls, h2d, d2h


class C3(Workload):
    unit = "GB/s"
    bound = "hbm"
    dtype = "q4_k/f32"
    SHAPES = C3_SHAPES

    def roofline_kernel(self, j):
        m, k = self.SHAPES[j]
        n = self.N
        # the library's dispatch (q4k_i8_applicable, q4k_ring_xs_applicable, launch_q4k_mma)
        if n <= 4:
            kern = "act_i8::prep_kernel<8> + q4k_i8_kernel"
        elif n <= 8:
            kern = "q4k_prep_kernel + q4k_ring_xs_kernel"
        else:
            kern = "q4k_prep_kernel + q4k_mma_kernel"
        return f"{kern}, {m}x{k} (one call)"

    def __init__(self, n, dev, gen):
        import torch
        from mlz_b200 import synth
        self.N = n
        self.metric = metric_name("c3", n, 1)
        per_step = sum(m * k // 256 * 144 for m, k in self.SHAPES)
        self.R = _rot_copies(per_step)
        self.W = [[synth.q4k_blocks_dev(gen, m, k, dev) for (m, k) in self.SHAPES] for _ in range(self.R)]
        self.X = [synth.f32_acts_dev(gen, n, k, dev) for (_, k) in self.SHAPES]
        self.Y = [torch.empty((n, m), dtype=torch.float32, device=dev) for (m, _) in self.SHAPES]
        import mlz_b200
        wsb = max(mlz_b200.mul_mat_workspace_bytes(mlz_b200.TYPE_Q4_K, m, k, n) for (m, k) in self.SHAPES)
        self.ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
        self.config = {"workload": workload_name("c3", n, 1), "batch": n,
                       "shapes": "4096x4096, 14336x4096, 4096x14336",
                       "l2": f"rotates {self.R} weight sets ({self.R * per_step / 1e6:.0f} MB >= 4x L2)"}

    def _bytes(self, m, k):
        return m * k // 256 * 144 + 4 * k * self.N + 4 * m * self.N

    def work_units(self):
        return sum(self._bytes(m, k) for m, k in self.SHAPES)

    def launches(self, i):
        import mlz_b200
        Ws = self.W[i % self.R]
        return [(lambda j=j: mlz_b200.mul_mat(Ws[j], self.X[j], out=self.Y[j], workspace=self.ws), self._bytes(m, k))
                for j, (m, k) in enumerate(self.SHAPES)]

    def host_weights(self):
        self.hW = [w.cpu().numpy() for w in self.W[0]]
        return [(w, 12, k) for w, (_, k) in zip(self.hW, self.SHAPES)]

    def e2e_calls(self, pinned):
        import torch
        xs = [x.cpu().pin_memory() for x in self.X]
        ys = [torch.empty(y.shape, dtype=torch.float32).pin_memory() for y in self.Y]
        pinned.extend(xs + ys)
        return ([(j, xs[j], ys[j]) for j in range(3)], sum(x.numel() * 4 for x in xs),
                sum(y.numel() * 4 for y in ys))


class C6(C3):
    """Q6_K decode mul_mat on the shapes of c3 (210-byte blocks)."""
    dtype = "q6_k/f32"

    def roofline_kernel(self, j):
        m, k = self.SHAPES[j]
        if self.N <= 4 and k % 1024 == 0:
            return f"act_i8::prep_kernel<16> + q6k_i8_kernel, {m}x{k} (one call)"
        return f"q6k_mma_kernel<{2 if self.N > 8 else 1}>, {m}x{k} (one call)"

    def __init__(self, n, dev, gen):
        import torch
        from mlz_b200 import synth
        self.N = n
        self.metric = metric_name("c6", n, 1)
        per_step = sum(m * k // 256 * 210 for m, k in self.SHAPES)
        self.R = _rot_copies(per_step)
        self.W = [[synth.q6k_blocks_dev(gen, m, k, dev) for (m, k) in self.SHAPES] for _ in range(self.R)]
        self.X = [synth.f32_acts_dev(gen, n, k, dev) for (_, k) in self.SHAPES]
        self.Y = [torch.empty((n, m), dtype=torch.float32, device=dev) for (m, _) in self.SHAPES]
        self.ws = None
        self.config = {"workload": workload_name("c6", n, 1), "batch": n,
                       "shapes": "4096x4096, 14336x4096, 4096x14336",
                       "l2": f"rotates {self.R} weight sets ({self.R * per_step / 1e6:.0f} MB >= 4x L2)"}

    def _bytes(self, m, k):
        return m * k // 256 * 210 + 4 * k * self.N + 4 * m * self.N

    def launches(self, i):
        import mlz_b200
        Ws = self.W[i % self.R]
        return [(lambda j=j: mlz_b200.mul_mat(Ws[j], self.X[j], out=self.Y[j], w_type=mlz_b200.TYPE_Q6_K),
                 self._bytes(m, k)) for j, (m, k) in enumerate(self.SHAPES)]

    def host_weights(self):
        self.hW = [w.cpu().numpy() for w in self.W[0]]
        return [(w, 14, k) for w, (_, k) in zip(self.hW, self.SHAPES)]


class C4(Workload):
    unit = "GB/s"
    bound = "hbm"
    dtype = "f16 kv / f32"

    def roofline_kernel(self, j):
        return "one flash-attention call: fa_decode_kernel + fa_combine_kernel"

    def __init__(self, n, dev, gen):
        import numpy as np
        import torch
        import mlz_b200
        from mlz_b200 import synth
        self.B, self.Hq, self.Hkv, self.D = n, 32, 8, 128
        self.kv_len_np = c4_lengths(n)
        self.L = 8192
        s = 1.0 / math.sqrt(self.D)
        self.q = torch.randn((n, self.Hq, 1, self.D), generator=gen, device=dev) * s
        self.k = (torch.randn((n, self.Hkv, self.L, self.D), generator=gen, device=dev) * s).half()
        self.v = (torch.randn((n, self.Hkv, self.L, self.D), generator=gen, device=dev) * s).half()
        self.kv_len = torch.from_numpy(self.kv_len_np).to(dev)
        self.out = torch.empty((n, self.Hq, 1, self.D), dtype=torch.float32, device=dev)
        from mlz_b200.ops import _nb
        desc = mlz_b200.make_fa_desc(self.q.data_ptr(), _nb(self.q, 4), self.k.data_ptr(), _nb(self.k, 2),
                                     self.v.data_ptr(), _nb(self.v, 2), self.out.data_ptr(), _nb(self.out, 4),
                                     (n, self.Hq, 1, self.Hkv, self.L, self.D), s,
                                     kv_len_ptr=self.kv_len.data_ptr())
        self.ws = torch.empty(max(mlz_b200.flash_attn_workspace_bytes(desc), 1), dtype=torch.uint8, device=dev)
        self.metric = metric_name("c4", n, 1)
        tot = int(self.kv_len_np.sum())
        self.config = {"workload": workload_name("c4", n, 1), "batch": n,
                       "sum_kv_len": tot, "l2": "inputs larger than L2 (KV cache 537 MB)"}

    def work_units(self):
        return 4096 * float(self.kv_len_np.sum()) + 2 * self.B * self.Hq * self.D * 4

    def launches(self, i):
        import mlz_b200
        return [(lambda: mlz_b200.flash_attn_dispatch(self.q, self.k, self.v, 1.0 / math.sqrt(self.D),
                                                      kv_len=self.kv_len, out=self.out, workspace=self.ws),
                 self.work_units())]


class C7(Workload):
    """c4's batch and lengths over a quantised KV cache (32-value blocks; Q8_0 by default,
    --kv-type for the others)."""
    unit = "GB/s"
    bound = "hbm"

    def roofline_kernel(self, j):
        return f"one flash-attention call: fa_quant_kernel<128, {C7_TYPE['kv'].upper()}> + fa_quant_combine_kernel"

    def __init__(self, n, dev, gen):
        import torch
        import mlz_b200
        from mlz_b200.ops import _nb
        from mlz_b200 import synth
        self.B, self.Hq, self.Hkv, self.D = n, 32, 8, 128
        self.kv_len_np = c4_lengths(n)
        self.L = 8192
        self.kv_type = C7_KV[C7_TYPE["kv"]]
        self.dtype = f"{C7_TYPE['kv']} kv / f32"
        # F32 rows: nb[0] = the 4-byte element, 4 D bytes per row
        self.bb, self.qmag, self.moff = synth.KV_QUANT[self.kv_type] if self.kv_type else (4, None, None)
        self.rb = self.D // 32 * self.bb if self.kv_type else 4 * self.D
        s = 1.0 / math.sqrt(self.D)
        self.q = torch.randn((n, self.Hq, 1, self.D), generator=gen, device=dev) * s
        self.k = self._rows(gen, dev)
        self.v = self._rows(gen, dev)
        self.kv_len = torch.from_numpy(self.kv_len_np).to(dev)
        self.out = torch.empty((n, self.Hq, 1, self.D), dtype=torch.float32, device=dev)
        desc = mlz_b200.make_fa_desc(self.q.data_ptr(), _nb(self.q, 4), self.k.data_ptr(),
                                     (self.bb,) + _nb(self.k, 1)[1:], self.v.data_ptr(), (self.bb,) + _nb(self.v, 1)[1:],
                                     self.out.data_ptr(), _nb(self.out, 4), (n, self.Hq, 1, self.Hkv, self.L, self.D), s,
                                     kv_len_ptr=self.kv_len.data_ptr(), kv_type=self.kv_type)
        self.ws = torch.empty(max(mlz_b200.flash_attn_workspace_bytes(desc), 1), dtype=torch.uint8, device=dev)
        self.metric = metric_name("c7", n, 1)
        self.config = {"workload": workload_name("c7", n, 1), "batch": n, "sum_kv_len": int(self.kv_len_np.sum()),
                       "kv_type": C7_TYPE["kv"],
                       "l2": f"inputs larger than L2 (KV cache {2 * n * self.Hkv * self.L * self.rb / 1e6:.0f} MB)"}

    def _rows(self, gen, dev):
        """Random quants; block scales d with the spread of N(0, 1)/sqrt(D) values; block
        minima m = offset * d * (1 + N(0, 0.1)) for the types that carry one."""
        import torch
        if self.kv_type == 0:
            v = torch.randn((self.B, self.Hkv, self.L, self.D), generator=gen, device=dev) / math.sqrt(self.D)
            return v.view(torch.uint8)
        nb, bb = self.D // 32, self.bb
        shape = (self.B, self.Hkv, self.L, nb)
        if self.kv_type == 8:
            r = torch.randint(-127, 128, shape + (bb,), generator=gen, device=dev,
                              dtype=torch.int16).to(torch.int8).view(torch.uint8)
        else:
            r = torch.randint(0, 256, shape + (bb,), generator=gen, device=dev, dtype=torch.int16).to(torch.uint8)
        d = torch.randn(shape + (1,), generator=gen, device=dev).abs() / (self.qmag * math.sqrt(self.D))
        r[..., 0:2] = d.to(torch.float16).view(torch.uint8)
        if self.moff is not None:
            jit = 1.0 + 0.1 * torch.randn(shape + (1,), generator=gen, device=dev)
            r[..., 2:4] = (self.moff * d * jit).to(torch.float16).view(torch.uint8)
        return r.reshape(self.B, self.Hkv, self.L, nb * bb)

    def work_units(self):
        return 2 * self.Hkv * self.rb * float(self.kv_len_np.sum()) + 2 * self.B * self.Hq * self.D * 4

    def launches(self, i):
        import mlz_b200
        return [(lambda: mlz_b200.flash_attn_dispatch_quant(self.q, self.k, self.v, 1.0 / math.sqrt(self.D),
                                                            self.kv_type, kv_len=self.kv_len, out=self.out,
                                                            workspace=self.ws),
                 self.work_units())]


class C5(Workload):
    scaling = "strong"

    def __init__(self, n, dev, gen, rank, world, comm):
        import torch
        from mlz_b200 import synth
        self.N, self.rank, self.world, self.comm = n, rank, world, comm
        self.unit = "GB/s" if n == 1 else "TFLOP/s"
        self.bound = "hbm" if n == 1 else "tensor"
        self.mats = C5_MATS
        self.metric = metric_name("c5", n, world)
        self.W = [synth.f16_weights_dev(gen, m // world, k, dev) for (_, m, k) in self.mats]
        self.X = [synth.f32_acts_dev(gen, n, k, dev) for (_, _, k) in self.mats]
        self.Y = [torch.empty((n, m), dtype=torch.float32, device=dev) for (_, m, _) in self.mats]
        import mlz_b200
        wsb = (max(comm.workspace_bytes(1, m, k, n) for (_, m, k) in self.mats) if comm else
               max(mlz_b200.mul_mat_workspace_bytes(mlz_b200.TYPE_F16, m, k, n) for (_, m, k) in self.mats))
        self.ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
        self.config = {"workload": workload_name("c5", n, world), "N": n,
                       "parallelism": (f"row-shard x{world}, slices all-gathered through NVLink peer memory"
                                       if world > 1 else "single GPU (unsharded)"),
                       "l2": "inputs larger than L2"}

    def work_units(self):  # whole-job units (all ranks together), reported once
        if self.N == 1:
            return sum(2.0 * m * k + 4 * k + 4 * m for (_, m, k) in self.mats)
        return sum(2.0 * self.N * m * k for (_, m, k) in self.mats)

    def launches(self, i):
        import mlz_b200
        out = []
        for j, (_, m, k) in enumerate(self.mats):
            u = (2.0 * m * k + 4 * k + 4 * m) if self.N == 1 else 2.0 * self.N * m * k
            if self.comm is not None:
                f = (lambda j=j, m=m: self.comm.mul_mat_sharded(self.W[j], self.X[j], m, out=self.Y[j], workspace=self.ws))
            else:
                f = (lambda j=j: mlz_b200.mul_mat(self.W[j], self.X[j], out=self.Y[j], workspace=self.ws))
            out.append((f, u))
        return out


# --------------------------------------------------------------------------- helpers

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], None, set()
        for line in out.splitlines():
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                smax = float(p[2])
            except ValueError:
                continue
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), p[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def max_over_ranks(x: float, world: int) -> float:
    if world <= 1:
        return x
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class CpuStep:
    """One step of a workload on the host cores through the oracle's restatement of the
    reference kernels (all host threads): every matrix of the step with all its rows
    (c1/c2/c3/c5), or every sequence of the batch with its own length (c4).  Inputs are
    generated once; rows past a generated block of weights reuse the block."""

    def __init__(self, cfg: str, n: int):
        import numpy as np
        import oracle
        from mlz_b200 import synth
        self.cfg, self.n = cfg, n
        self.nth = oracle.host_threads()
        g = synth.rng(77)
        self.parts = []          # (M, K, weight block, x)
        if cfg in ("c1", "c2", "c5"):
            shapes = {"c1": [(8192, 3072)], "c2": [(o, i) for (_, o, i, _) in C2_PROJ],
                      "c5": [(m, k) for (_, m, k) in C5_MATS]}[cfg]
            blocks = {}
            for (M, K) in shapes:
                if K not in blocks:
                    blocks[K] = synth.f16_weights(g, min(M, 4096), K)
                self.parts.append((M, K, blocks[K], synth.f32_acts(g, n, K)))
            self.kernel = lambda w, x: oracle.base_mul_mat_f16(w, x, self.nth)
            self.flops = cfg == "c2" or (cfg == "c5" and n > 1)
            self.what = "convert-then-GEMM restatement"
        elif cfg in ("c3", "c6"):
            q6 = cfg == "c6"
            for (M, K) in C3_SHAPES:
                blk = (synth.q6k_blocks if q6 else synth.q4k_blocks)(g, min(M, 4096), K)
                self.parts.append((M, K, blk, synth.f32_acts(g, n, K)))
            self.kernel = ((lambda w, x: oracle.base_mul_mat_q6k(w, x, self.nth)) if q6 else
                           (lambda w, x: oracle.base_mul_mat_q4k(w, x, self.nth)))
            self.flops = False
            self.block_bytes = 210 if q6 else 144
            self.what = f"Q8_K quantise + {'Q6_K' if q6 else 'Q4_K'} x Q8_K dot restatement"
        elif cfg in ("c4", "c7"):
            self.kl = c4_lengths(n)
            self.slots = 4
            self.q, self.k, self.v = synth.fa_inputs(g, self.slots, 32, 8, int(self.kl.max()), 128)
            self.flops = False
            self.kv_type = 1
            self.row_bytes = 256
            if cfg == "c7":
                self.kv_type = C7_KV[C7_TYPE["kv"]]
                self.row_bytes = 4 * synth.KV_QUANT[self.kv_type][0] if self.kv_type else 512
                self.k = synth.kv_quant_rows(g, (self.slots, 8, int(self.kl.max())), 128, self.kv_type)
                self.v = synth.kv_quant_rows(g, (self.slots, 8, int(self.kl.max())), 128, self.kv_type)
            kv = C7_TYPE["kv"].upper()
            self.what = "FA2 skeleton restatement" + (f" ({kv} K/V dequantised per row)" if cfg == "c7" else "")
        else:
            raise ValueError(cfg)

    def run(self) -> float:
        """One step; returns its units (bytes or flops)."""
        import oracle
        n = self.n
        units = 0.0
        if self.cfg in ("c4", "c7"):
            for b in range(len(self.kl)):
                j = b % self.slots
                if self.kv_type == 1:
                    oracle.base_flash_attn(self.q[j:j + 1], self.k[j:j + 1], self.v[j:j + 1], 1 / math.sqrt(128),
                                           kv_len=self.kl[b:b + 1], nth=self.nth)
                else:
                    oracle.base_flash_attn_q(self.q[j:j + 1], self.k[j:j + 1], self.v[j:j + 1], 1 / math.sqrt(128),
                                             self.kv_type, kv_len=self.kl[b:b + 1], nth=self.nth)
                units += 2 * 8 * self.row_bytes * float(int(self.kl[b])) + 2 * 32 * 128 * 4
            return units
        for (M, K, w, x) in self.parts:
            reps, r = divmod(M, w.shape[0])
            for _ in range(reps):
                self.kernel(w, x)
            if r:
                self.kernel(w[:r], x)
            if self.flops:
                units += 2.0 * M * K * n
            elif self.cfg in ("c3", "c6"):
                units += M * (K // 256) * self.block_bytes + 4 * K * n + 4 * M * n
            else:
                units += 2.0 * M * K + 4 * K * n + 4 * M * n
        return units


_CPU_STEPS = {}


def cpu_sample(cfg: str, n: int, target_s: float):
    """Times whole steps of the workload on the host cores (CpuStep), as many as fit in
    about `target_s` (at least one).  Returns (value in the metric's unit, description,
    threads)."""
    import oracle
    key = (cfg, n)
    if key not in _CPU_STEPS:
        _CPU_STEPS[key] = CpuStep(cfg, n)
    st = _CPU_STEPS[key]
    t0 = time.perf_counter()
    units = st.run()
    dt = time.perf_counter() - t0
    steps = 1
    more = int(target_s / max(dt, 1e-6)) - 1
    if more > 0:
        t1 = time.perf_counter()
        for _ in range(more):
            units += st.run()
        dt += time.perf_counter() - t1
        steps += more
    scale = 1e-12 if st.flops else 1e-9
    return (units / dt * scale, f"{steps} whole step(s) of the workload in {dt:.2f}s ({st.what}, "
            f"{st.nth} threads); host {oracle.host_cpu_model()}", st.nth)


# --------------------------------------------------------------------------- arms

def reference_arm(a):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    n = a.n or DEFAULT_N[a.config]
    unit = {"c1": "GB/s", "c2": "TFLOP/s", "c3": "GB/s", "c4": "GB/s", "c5": "GB/s" if n == 1 else "TFLOP/s",
            "c6": "GB/s", "c7": "GB/s"}[a.config]
    import oracle
    oracle.build()
    per_step = max(a.cpu_seconds / max(a.steps, 1), 0.5)
    for _ in range(a.warmup):
        cpu_sample(a.config, n, min(per_step, 0.5))
    vals, desc, nth = [], "", 1
    t0 = time.perf_counter()
    for _ in range(a.steps):
        v, desc, nth = cpu_sample(a.config, n, per_step)
        vals.append(v)
    wall = time.perf_counter() - t0
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": metric_name(a.config, n, world), "value": value, "unit": unit,
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * wall / max(a.steps, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": DTYPE[a.config] if a.config != "c7" else f"{C7_TYPE['kv']} kv / f32",
        "data": "synthetic (seeded), random-init weights",
        "config": {"workload": workload_name(a.config, n, world),
                   "implementation": "CPU restatement of the reference kernels (oracle/) on the host cores"},
        "cpu_baseline": {"value": value, "unit": unit, "cores": nth, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def make_workload(cfg: str, n: int, dev, rank: int, world: int, comm):
    import torch
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + 100 * int(cfg[1]) + n + rank)
    wl = {"c1": C1, "c2": C2, "c3": C3, "c4": C4, "c6": C6, "c7": C7}.get(cfg)
    return wl(n, dev, gen) if wl else C5(n, dev, gen, rank, world, comm)


def time_workload(w, a, world, K: int, warmup: int, use_graph: bool):
    """Warm-up, then K steps timed on the device: a CUDA-graph replay of the K steps (or the
    eager launches), and each call's K repetitions replayed as their own graph for the
    roofline.  Returns a dict of the timings (milliseconds, this rank)."""
    import torch
    import mlz_b200
    stream = torch.cuda.current_stream()
    for i in range(warmup):
        for f, _ in w.launches(i):
            f()
    torch.cuda.synchronize()
    units_l = [u for _, u in w.launches(0)]
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in units_l]
          for _ in range(K)]
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    # Hold the GPU with a short spin (torch.cuda._sleep) while the host queues the K steps
    # and their events, so the per-launch events time the kernels rather than the host's
    # launch cadence.  The spin is enqueued before t0 and is not part of the timed region.
    t_host = time.perf_counter()
    for f, _ in w.launches(0):
        f()
    torch.cuda.synchronize()
    host_per_step = time.perf_counter() - t_host
    torch.cuda._sleep(int(min(2e9, max(2e6, 3.0 * host_per_step * K * 2.0e9))))
    n0 = mlz_b200.launch_count()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for s_ in range(K):
        for j, (f, _) in enumerate(w.launches(s_)):
            ev[s_][j][0].record(stream)
            f()
            ev[s_][j][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    out = {"n_launch": mlz_b200.launch_count() - n0, "ms_eager": t0.elapsed_time(t1),
           "per_launch_ms": [sum(ev[s_][j][0].elapsed_time(ev[s_][j][1]) for s_ in range(K)) / K
                             for j in range(len(units_l))],
           "timing": "eager launches", "call_timing": "eager events around each call", "units_l": units_l}
    out["ms_local"] = out["ms_eager"]
    # The same K steps captured once as a CUDA graph and replayed: the decode kernels are
    # shorter than the host's per-call launch cost, so the eager loop would time Python.
    if use_graph:
        gs = torch.cuda.Stream()
        gs.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        n0 = mlz_b200.launch_count()
        try:
            with torch.cuda.graph(graph, stream=gs):
                for s_ in range(K):
                    for f, _ in w.launches(s_):
                        f()
        except Exception as exc:  # a call that cannot be captured: keep the eager timing
            use_graph = False
            out["timing"] = f"eager launches ({type(exc).__name__} in graph capture)"
            del graph
            torch.cuda.synchronize()
    if use_graph:
        out["n_launch"] = mlz_b200.launch_count() - n0       # kernels the replay runs
        with torch.cuda.stream(gs):
            graph.replay()                                     # untimed first replay
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()
        g0 = torch.cuda.Event(enable_timing=True)
        g1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(gs):
            g0.record(gs)
            graph.replay()
            g1.record(gs)
        torch.cuda.synchronize()
        out["ms_local"] = g0.elapsed_time(g1)
        out["timing"] = "CUDA graph replay of the K steps"
        del graph
        # Per-call device times for the roofline: each call's K repetitions (the same
        # inputs and weight rotation as in the steps) captured as their own graph and timed
        # by events around its replay -- event nodes inside a graph would add microseconds
        # to every call.  The sharded calls wait on their peers, so every rank replays
        # every call's graph in the same order.
        try:
            per = []
            for j in range(len(units_l)):
                gj = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gj, stream=gs):
                    for s_ in range(K):
                        w.launches(s_)[j][0]()
                with torch.cuda.stream(gs):
                    gj.replay()                                # untimed first replay
                torch.cuda.synchronize()
                c0 = torch.cuda.Event(enable_timing=True)
                c1 = torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(gs):
                    c0.record(gs)
                    gj.replay()
                    c1.record(gs)
                torch.cuda.synchronize()
                per.append(c0.elapsed_time(c1) / K)
                del gj
            out["per_launch_ms"] = per
            out["call_timing"] = "each call's K repetitions replayed as a CUDA graph, timed by events"
        except Exception as exc:  # keep the eager per-call events
            out["call_timing"] = f"eager events around each call ({type(exc).__name__} with per-call graphs)"
    return out


def roofline_of(w, t, peaks, clocks, ms):
    """Roofline of the dominant call (largest average device time); c2 pools its 7 calls."""
    units_l, per = t["units_l"], t["per_launch_ms"]
    jdom = max(range(len(units_l)), key=lambda j: per[j])
    if isinstance(w, C2):  # all 7 projections run the same GEMM kernel: pool them
        ach = sum(units_l) / (sum(per) * 1e-3) * 1e-12
    else:
        ach = units_l[jdom] / (per[jdom] * 1e-3) * w.unit_scale()
    # tensor peak: the sustained (power-capped) figure when the timed region ran under the
    # power cap or for over a second -- the regime that figure was measured in -- else burst
    power_capped = "sw_power_cap" in ((clocks or {}).get("reasons") or [])
    long_run = ms * 1e-3 > 1.0 or power_capped
    if w.bound == "hbm":
        peak, peak_name = peaks["hbm_gbs"], "hbm_gbs"
    else:
        peak = peaks["bf16_tflops_sustained"] if long_run else peaks["bf16_tflops"]
        peak_name = "bf16_tflops_sustained" if long_run else "bf16_tflops"
    # a row-sharded call's work is the whole matrix, spread over the ranks: its roof is the
    # per-GPU peak times the ranks
    shards = getattr(w, "world", 1) if isinstance(w, C5) else 1
    peak *= shards
    r = {"bound": w.bound, "achieved": ach, "peak": peak, "unit": "GB/s" if w.bound == "hbm" else "TFLOP/s",
         "frac": ach / peak, "traffic": None,
         "peak_source": f"{peaks['source']} {peak_name}" + (f" x {shards} GPUs" if shards > 1 else "")
                        + (" (sw_power_cap active in the timed region)" if power_capped and w.bound != "hbm" else ""),
         "kernel": w.roofline_kernel(jdom), "call_timing": t["call_timing"]}
    if w.bound != "hbm":
        r["frac_of_burst"] = ach / (peaks["bf16_tflops"] * shards)
    return r


# Measured rows that the default line carries besides its headline workload, so that one
# run records every configuration: (config, N).  On several GPUs only the other c5 size.
EXTRA_ROWS_1GPU = [("c2", 2048), ("c2", 512), ("c1", 1), ("c1", 8), ("c1", 32), ("c3", 1), ("c3", 4), ("c3", 16),
                   ("c4", 16), ("c5", 256), ("c6", 1), ("c6", 4), ("c6", 16), ("c7", 16)]


def extra_rows(a, n_head, dev, rank, world, comm, peaks):
    import torch
    rows_cfg = EXTRA_ROWS_1GPU if world == 1 else [("c5", 256 if n_head == 1 else 1)]
    rows = []
    for cfg, n in rows_cfg:
        if cfg == a.config and n == n_head:
            continue
        try:
            w = make_workload(cfg, n, dev, rank, world, comm if cfg == "c5" else None)
            t = time_workload(w, a, world, max(5, min(a.steps, 20)), 3, not a.no_graph)
            ms = max_over_ranks(t["ms_local"], world)
            K = max(5, min(a.steps, 20))
            units = w.work_units()
            job = units if isinstance(w, C5) else units * world
            rl = roofline_of(w, t, peaks, None, ms)
            tr = traffic_of(cfg, n, w, world)
            if tr is not None:
                rl["traffic"], rl["traffic_source"] = tr
            row = {"workload": w.config["workload"], "metric": w.metric, "unit": w.unit,
                   "value": job * K / (ms * 1e-3) * w.unit_scale(), "ms_per_step": ms / K,
                   "roofline": rl, "gpu_launches": t["n_launch"]}
            if rank == 0 and world == 1 and not a.no_cpu_baseline:
                v, desc, nth = cpu_sample(cfg, n, 1.0)
                row["cpu_baseline"] = {"value": v, "unit": w.unit, "cores": nth, "kind": "port", "sample": desc}
            rows.append(row)
            del w
        except Exception as exc:  # a row is reported, never required
            rows.append({"workload": f"{cfg} N={n}", "error": f"{type(exc).__name__}: {exc}"[:300]})
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return rows


def mlz_arm(a):
    import torch
    import mlz_b200

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    mlz_b200.init(local)
    mlz_b200.set_launch_overlap({"off": mlz_b200.OVERLAP_OFF, "safe": mlz_b200.OVERLAP_SAFE,
                                 "weights": mlz_b200.OVERLAP_WEIGHTS}[a.overlap])
    n = a.n or DEFAULT_N[a.config]
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    comm = None   # one GPU runs c5 unsharded (the plain mul_mat): nothing to gather
    if world > 1 and (a.config == "c5" or not a.no_rows):
        obj = [mlz_b200.Comm.unique_id() if rank == 0 else None]
        if world > 1:
            import torch.distributed as dist
            dist.broadcast_object_list(obj, src=0)
        comm = mlz_b200.Comm(world, rank, local, obj[0], timeout_ms=60000)

    w = make_workload(a.config, n, dev, rank, world, comm)
    peaks = load_peaks()

    # warm-up (first calls also create contexts / workspaces outside the timed region)
    for i in range(a.warmup if a.profile_run else max(a.warmup, 3)):
        for f, _ in w.launches(i):
            f()
    torch.cuda.synchronize()

    # about a second of load for the clock sampler; the same number of steps on every rank
    # (the sharded calls are collective)
    t_step = time.perf_counter()
    for f, _ in w.launches(0):
        f()
    torch.cuda.synchronize()
    n_load = 0 if a.profile_run else int(max_over_ranks(min(20000.0, max(8.0, 1.0 / max(time.perf_counter() - t_step,
                                                                                          1e-5))), world))
    sampler = ClockSampler(local)
    sampler.start()
    for i in range(n_load):
        for f, _ in w.launches(i):
            f()
        if i % 8 == 7:
            torch.cuda.synchronize()
    torch.cuda.synchronize()

    K = a.steps
    t = time_workload(w, a, world, K, 0, not a.no_graph and not a.profile_run)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    clocks = sampler.stop()
    ms = max_over_ranks(t["ms_local"], world)
    max_ms_eager = max_over_ranks(t["ms_eager"], world)

    units = w.work_units()
    job_units = units if isinstance(w, C5) else units * world
    value = job_units * K / (ms * 1e-3) * w.unit_scale()
    roofline = roofline_of(w, t, peaks, clocks, ms)
    tr = traffic_of(a.config, n, w, world)
    if tr is not None:
        roofline["traffic"] = tr[0]
        roofline["traffic_source"] = tr[1]

    # end to end through the public API with host buffers
    e2e = None
    if not a.no_e2e and not a.profile_run:
        e2e = run_e2e_sharded(w, a, world) if isinstance(w, C5) else run_e2e(w, a, world, value)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline and not a.profile_run:
        try:
            v, desc, nth = cpu_sample(a.config, n, a.cpu_seconds)
            cpu = {"value": v, "unit": w.unit, "cores": nth, "kind": "port", "sample": desc}
        except Exception as exc:  # the baseline is reported, never required
            cpu = {"value": None, "unit": w.unit, "cores": None, "kind": "port", "sample": f"failed: {exc}"}

    head = {"metric": w.metric, "unit": w.unit, "scaling": w.scaling, "dtype": w.dtype, "config": dict(w.config)}
    rows = None
    if not a.no_rows and not a.profile_run:
        del w
        torch.cuda.empty_cache()
        rows = extra_rows(a, n, dev, rank, world, comm, peaks)

    if rank == 0:
        cfg = head["config"]
        cfg["parallelism"] = cfg.get("parallelism", f"replicas x{world}" if world > 1 else "single GPU")
        cfg["timing"] = t["timing"]
        cfg["launch_overlap"] = a.overlap
        cfg["eager_ms_per_step"] = max_ms_eager / K
        line = {"metric": head["metric"], "value": value, "unit": head["unit"], "n_gpus": world, "steps": K,
                "warmup": a.warmup, "ms_per_step": ms / K, "higher_is_better": True, "scaling": head["scaling"],
                "vs_baseline": None, "dtype": head["dtype"], "data": "synthetic (seeded), random-init weights",
                "config": cfg, "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": t["n_launch"],
                "clocks": clocks}
        if rows is not None:
            line["rows"] = rows
        print(json.dumps(line), flush=True)
    if comm is not None:
        comm.destroy()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_e2e_sharded(w, a, world):
    """c5 end to end through the public device API with host buffers: every step copies the
    three activation matrices from page-locked host memory to the device, runs the three
    row-sharded calls (mlzc_mul_mat_sharded_dev) and reads the three gathered outputs back
    to page-locked host memory, then synchronises.  Host wall clock, max over ranks."""
    import torch
    hx = [x.cpu().pin_memory() for x in w.X]
    hy = [torch.empty(y.shape, dtype=torch.float32).pin_memory() for y in w.Y]
    calls = w.launches(0)

    def step():
        for x, h in zip(w.X, hx):
            x.copy_(h, non_blocking=True)
        for f, _ in calls:
            f()
        for y, h in zip(w.Y, hy):
            h.copy_(y, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    for _ in range(max(a.warmup, 2)):
        step()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    K = max(3, min(a.steps, 10))
    t0 = time.perf_counter()
    for _ in range(K):
        step()
    dt = max_over_ranks((time.perf_counter() - t0) / K, world)
    h2d = sum(x.numel() * 4 for x in hx)
    d2h = sum(y.numel() * 4 for y in hy)
    return {"value": w.work_units() / dt * w.unit_scale(), "unit": w.unit, "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "path": "mlzc_mul_mat_sharded_dev with host copies",
            "host_buffers": "page-locked", "ms_per_step": 1e3 * dt}


def run_e2e(w, a, world, value_dev):
    """Same metric through mlzc_try_mul_mat / mlzc_try_flash_attn with host buffers."""
    import numpy as np
    import torch
    import mlz_b200
    pinned = []
    fa = isinstance(w, (C4, C7))
    if fa:
        q = w.q.cpu().pin_memory()
        k = w.k.cpu().pin_memory()
        v = w.v.cpu().pin_memory()
        kl = torch.from_numpy(w.kv_len_np).pin_memory()
        o = torch.empty(w.out.shape, dtype=torch.float32).pin_memory()
        nb = lambda t, e: tuple(s * e for s in t.stride()[::-1])
        if isinstance(w, C7):   # rows of the KV type's blocks (nb[0] = block or element bytes)
            kv_nb = lambda t: (w.bb,) + nb(t, 1)[1:]
            kv_type = w.kv_type
        else:
            kv_nb = lambda t: nb(t, 2)
            kv_type = mlz_b200.TYPE_F16
        desc = mlz_b200.make_fa_desc(q.data_ptr(), nb(q, 4), k.data_ptr(), kv_nb(k), v.data_ptr(), kv_nb(v),
                                     o.data_ptr(), nb(o, 4), (w.B, w.Hq, 1, w.Hkv, w.L, w.D),
                                     1.0 / math.sqrt(w.D), kv_len_ptr=kl.data_ptr(), kv_type=kv_type)
        # the hook copies the whole cache view it is given: here only the live keys count
        h2d = q.numel() * 4 + (k.numel() * k.element_size() + v.numel() * v.element_size()) + kl.numel() * 4
        d2h = o.numel() * 4
        step = lambda: mlz_b200.ggml_simd_try_flash_attn(desc)
    else:
        hws = w.host_weights()
        calls, h2d, d2h = w.e2e_calls(pinned)

        def make_step(pairs):
            views = []
            for (j, x, y) in pairs:
                hw, t, K = hws[j]
                views.append((mlz_b200.tensor_view(hw if t != 1 else hw.view(np.uint16), t, ne0=K),
                              mlz_b200.TensorView(), mlz_b200.TensorView()))
                sv = views[-1]
                for tv, arr in ((sv[1], x), (sv[2], y)):
                    tv.type = 0
                    tv.ne[:] = [arr.shape[1], arr.shape[0], 1, 1]
                    tv.nb[:] = [4, arr.stride(0) * 4, arr.stride(0) * 4 * arr.shape[0],
                                arr.stride(0) * 4 * arr.shape[0]]
                    tv.data = arr.data_ptr()

            def step_fn():
                r = 1
                for (s0, s1, d) in views:
                    r &= mlz_b200.ggml_simd_try_mul_mat(s0, s1, d)
                return r
            return step_fn
        step = make_step(calls)
        # the same calls with pageable (not page-locked) host buffers, as a ggml buffer is
        # unless the integration registers it (mlzc_host_register)
        pageable = [(j, x.clone(), y.clone()) for (j, x, y) in calls]
        step_pageable = make_step(pageable)

    def timed(fn):
        for _ in range(max(a.warmup, 2)):
            if fn() != 1:
                raise RuntimeError("plugin entry point declined the workload: " + mlz_b200.last_error())
        torch.cuda.synchronize()
        K = max(3, min(a.steps, 10))
        t0 = time.perf_counter()
        for _ in range(K):
            fn()
        return max_over_ranks(time.perf_counter() - t0, world) / K
    units = w.work_units() * world
    dt = timed(step)
    out = {"value": units / dt * w.unit_scale(), "unit": w.unit, "h2d_bytes_per_step": int(h2d),
           "d2h_bytes_per_step": int(d2h), "path": "mlzc_try_flash_attn" if fa else "mlzc_try_mul_mat",
           "host_buffers": "page-locked", "ms_per_step": 1e3 * dt}
    if not fa:
        dtp = timed(step_pageable)
        out["pageable"] = {"value": units / dtp * w.unit_scale(), "ms_per_step": 1e3 * dtp}
    return out


def main():
    a = parse_args()
    C7_TYPE["kv"] = a.kv_type
    if a.impl == "reference":
        reference_arm(a)
    else:
        mlz_arm(a)


if __name__ == "__main__":
    main()
