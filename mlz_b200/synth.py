"""Seeded synthetic operands in the shapes and value distributions of the benchmarked
workloads (no model files are involved: weights are random-init of the named shapes).

Host generators (numpy PCG64) feed the parity tests; the ``*_dev`` generators build the
large benchmark operands directly in device memory with torch's seeded CUDA generator.

Distributions:
  F16 weights  N(0, 0.02) rounded to f16;  activations N(0, 1) f32.
  Q4_K blocks  d, dmin = f16(|N(0, 0.01)|); 12 random scale bytes (every bit pattern is a
               valid set of 6-bit scales/mins); qs uniform nibbles 0..15.
  FA decode    q, k, v ~ N(0, 1)/sqrt(D) (k, v stored f16); kv lengths U{lo..hi}.
"""
from __future__ import annotations

import numpy as np

QK_K = 256
Q4K_BYTES = 144


def seed_for(config: int, n: int) -> int:
    """Per-row seed: 1000 + config*100 + N."""
    return 1000 + 100 * config + n


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def f16_weights(g: np.random.Generator, M: int, K: int, std: float = 0.02) -> np.ndarray:
    """(M, K) float16."""
    return (g.standard_normal((M, K), dtype=np.float32) * std).astype(np.float16)


def f32_acts(g: np.random.Generator, N: int, K: int) -> np.ndarray:
    return g.standard_normal((N, K), dtype=np.float32)


def q4k_blocks(g: np.random.Generator, M: int, K: int) -> np.ndarray:
    """(M, K/256*144) uint8 Q4_K super-blocks."""
    assert K % QK_K == 0
    nb = K // QK_K
    blk = g.integers(0, 256, size=(M, nb, Q4K_BYTES), dtype=np.uint8)
    d = np.abs(g.standard_normal((M, nb, 2), dtype=np.float32) * 0.01).astype(np.float16)
    blk[:, :, 0:4] = d.view(np.uint8).reshape(M, nb, 4)
    return blk.reshape(M, nb * Q4K_BYTES)


Q6K_BYTES = 210


def q6k_blocks(g: np.random.Generator, M: int, K: int) -> np.ndarray:
    """(M, K/256*210) uint8 Q6_K super-blocks: random ql / qh bits, int8 scales uniform in
    -128..127, d = f16(|N(0, 0.001)|)."""
    assert K % QK_K == 0
    nb = K // QK_K
    blk = g.integers(0, 256, size=(M, nb, Q6K_BYTES), dtype=np.uint8)
    d = np.abs(g.standard_normal((M, nb, 1), dtype=np.float32) * 0.001).astype(np.float16)
    blk[:, :, 208:210] = d.view(np.uint8).reshape(M, nb, 2)
    return blk.reshape(M, nb * Q6K_BYTES)


def fa_inputs(g: np.random.Generator, B: int, Hq: int, Hkv: int, L: int, D: int, NQ: int = 1):
    """q (B, Hq, NQ, D) f32; k, v (B, Hkv, L, D) f16."""
    s = 1.0 / np.sqrt(D)
    q = (g.standard_normal((B, Hq, NQ, D), dtype=np.float32) * s).astype(np.float32)
    k = (g.standard_normal((B, Hkv, L, D), dtype=np.float32) * s).astype(np.float16)
    v = (g.standard_normal((B, Hkv, L, D), dtype=np.float32) * s).astype(np.float16)
    return q, k, v


# ggml type -> (block bytes, typical |value / d|, offset m / d or None): Q8_0, Q4_0, Q4_1,
# Q5_0, Q5_1, IQ4_NL
KV_QUANT = {8: (34, 64.0, None), 2: (18, 4.0, None), 3: (20, 4.0, -7.5), 6: (22, 8.0, None),
            7: (24, 8.0, -15.5), 20: (18, 60.0, None)}


def kv_quant_rows(g: np.random.Generator, shape, D: int, kv_type: int) -> np.ndarray:
    """Quantised K/V rows of a KV-cache type of KV_QUANT (or F32 rows, kv_type 0, of N(0, 1)/
    sqrt(D) values): uint8 array of shape + (D/32*block_bytes,), random quants (and fifth bits),
    block scales d = f16(|N(0, 1)| /
    (typical |value / d| * sqrt(D))) so that the values have the spread of N(0, 1)/sqrt(D);
    the types with a block minimum (Q4_1, Q5_1) get m = f16(offset * d * (1 + N(0, 0.1)))."""
    if kv_type == 0:   # F32 rows: the values themselves, as bytes
        v = (g.standard_normal(tuple(shape) + (D,), dtype=np.float32) / np.sqrt(D)).astype(np.float32)
        return v.view(np.uint8)
    bb, qmag, moff = KV_QUANT[kv_type]
    nb = D // 32
    rows = g.integers(0, 256, size=tuple(shape) + (nb, bb), dtype=np.uint8)
    d32 = np.abs(g.standard_normal(tuple(shape) + (nb, 1), dtype=np.float32)) / (qmag * np.sqrt(D))
    rows[..., 0:2] = d32.astype(np.float16).view(np.uint8)
    if moff is not None:
        jit = 1.0 + 0.1 * g.standard_normal(tuple(shape) + (nb, 1), dtype=np.float32)
        rows[..., 2:4] = (moff * d32 * jit).astype(np.float16).view(np.uint8)
    return rows.reshape(tuple(shape) + (nb * bb,))


def kv_lengths(g: np.random.Generator, B: int, lo: int, hi: int) -> np.ndarray:
    return g.integers(lo, hi + 1, size=B, dtype=np.int64).astype(np.int32)


# ---------------------------------------------------------------- device side

def f16_weights_dev(gen, M: int, K: int, device, std: float = 0.02):
    import torch
    return (torch.randn((M, K), generator=gen, device=device, dtype=torch.float32) * std).to(torch.float16)


def f32_acts_dev(gen, N: int, K: int, device):
    import torch
    return torch.randn((N, K), generator=gen, device=device, dtype=torch.float32)


def q6k_blocks_dev(gen, M: int, K: int, device):
    import torch
    nb = K // QK_K
    blk = torch.randint(0, 256, (M, nb, Q6K_BYTES), generator=gen, device=device, dtype=torch.uint8)
    d = (torch.randn((M, nb, 1), generator=gen, device=device) * 0.001).abs().to(torch.float16)
    blk[:, :, 208:210] = d.view(torch.uint8).reshape(M, nb, 2)
    return blk.reshape(M, nb * Q6K_BYTES)


def q4k_blocks_dev(gen, M: int, K: int, device):
    import torch
    nb = K // QK_K
    blk = torch.randint(0, 256, (M, nb, Q4K_BYTES), generator=gen, device=device, dtype=torch.uint8)
    d = (torch.randn((M, nb, 2), generator=gen, device=device) * 0.01).abs().to(torch.float16)
    blk[:, :, 0:4] = d.view(torch.uint8).reshape(M, nb, 4)
    return blk.reshape(M, nb * Q4K_BYTES)
