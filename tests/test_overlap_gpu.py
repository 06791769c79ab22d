"""GPU: launch overlap (programmatic dependent launch) never changes a result.

Each case chains calls whose inputs are the previous call's outputs (ping-pong buffers,
so a kernel two steps back read what the next one overwrites; a shared workspace, so a
call's prep kernel rewrites what the previous call's main kernel read), eagerly and as
a replayed CUDA graph.  The kernels are deterministic, so every overlap mode must give
the same bits as plain stream order."""
import numpy as np
import pytest

import mlz_b200
from mlz_b200 import synth

pytestmark = pytest.mark.gpu
MODES = (mlz_b200.OVERLAP_OFF, mlz_b200.OVERLAP_SAFE, mlz_b200.OVERLAP_WEIGHTS)


def _weights(kind, gen, M, K, dev):
    import torch
    if kind == "f16":
        return synth.f16_weights_dev(gen, M, K, dev)
    if kind == "f32":
        return torch.randn((M, K), generator=gen, device=dev, dtype=torch.float32) * 0.02
    blk = synth.q4k_blocks_dev(gen, M, K, dev).view(M, K // 256, 144)
    # dmin = 7.5 d centres the weights (E[sc q] = 7.5 E[m]), so a chain of products stays finite
    r = torch.rand((M, K // 256, 1), generator=gen, device=dev) * 1e-4 + 1e-4
    d = torch.cat([r, 7.5 * r], dim=2).to(torch.float16)
    blk[:, :, 0:4] = d.view(torch.uint8).reshape(M, K // 256, 4)
    return blk.reshape(M, -1).contiguous()


def _in_mode(mode, fn):
    import torch
    torch.cuda.synchronize()
    mlz_b200.set_launch_overlap(mode)
    try:
        out = fn()
        torch.cuda.synchronize()
        return out
    finally:
        mlz_b200.set_launch_overlap(mlz_b200.OVERLAP_SAFE)


@pytest.mark.parametrize("kind", ["f16", "f32", "q4k"])
@pytest.mark.parametrize("N", [1, 4, 8, 16, 64])
def test_chained_mul_mat(dev, kind, N):
    import torch
    gen = torch.Generator(device=dev).manual_seed(9100 + N)
    M = K = 2048
    Ws = [_weights(kind, gen, M, K, dev) for _ in range(2)]
    x0 = synth.f32_acts_dev(gen, N, K, dev)
    wsb = mlz_b200.mul_mat_workspace_bytes(mlz_b200.weight_type_of(Ws[0]), M, K, N)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
    a = torch.empty_like(x0)
    b = torch.empty_like(x0)

    def chain():
        a.copy_(x0)
        for i in range(8):
            src, dst = (a, b) if i % 2 == 0 else (b, a)
            mlz_b200.mul_mat(Ws[i % 2], src, out=dst, workspace=ws)

    results = {}
    for mode in MODES:
        _in_mode(mode, chain)
        results[mode] = a.clone()
    ref = results[mlz_b200.OVERLAP_OFF]
    assert torch.isfinite(ref).all() and ref.abs().max() > 0
    for mode in MODES[1:]:
        assert torch.equal(results[mode], ref), f"mode {mode} differs from stream order"

    # the same chain captured once per mode and replayed
    for mode in MODES:
        def capture():
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                chain()   # warm-up outside capture (plans, attributes)
                torch.cuda.synchronize()
                with torch.cuda.graph(g, stream=s):
                    chain()
            return g
        g = _in_mode(mode, capture)
        for _ in range(3):
            a.zero_()
            b.fill_(float("nan"))
            g.replay()
        torch.cuda.synchronize()
        assert torch.equal(a, ref), f"graph replay in mode {mode} differs"
        del g


def test_chained_attention_block(dev):
    """x -> q = Wq x (skinny / GEMV) -> flash-attention (q from the previous kernel, a
    ragged batch) -> y = Wo attn -> next q ..., in every mode."""
    import torch
    gen = torch.Generator(device=dev).manual_seed(9200)
    B, Hq, Hkv, D, L = 8, 32, 8, 128, 1500
    E = 1024
    g = synth.rng(9201)
    kv_len = torch.from_numpy(synth.kv_lengths(g, B, 100, L)).to(dev)
    k = (torch.randn((B, Hkv, L, D), generator=gen, device=dev) * 0.1).to(torch.float16)
    v = (torch.randn((B, Hkv, L, D), generator=gen, device=dev) * 0.1).to(torch.float16)
    Wq = synth.f16_weights_dev(gen, Hq * D, E, dev)
    Wo = synth.f16_weights_dev(gen, E, Hq * D, dev, std=0.01)
    x0 = synth.f32_acts_dev(gen, B, E, dev)
    x = torch.empty_like(x0)
    q = torch.empty((B, Hq * D), dtype=torch.float32, device=dev)
    att = torch.empty((B, Hq, 1, D), dtype=torch.float32, device=dev)
    kv_nb = (2, 2 * D, 2 * L * D, 2 * Hkv * L * D)
    desc = mlz_b200.make_fa_desc(q.data_ptr(), (4, 4 * D, 4 * D, 4 * Hq * D), k.data_ptr(), kv_nb, v.data_ptr(),
                                 kv_nb, att.data_ptr(), (4, 4 * D, 4 * D, 4 * Hq * D), (B, Hq, 1, Hkv, L, D),
                                 1.0 / np.sqrt(D), kv_len_ptr=kv_len.data_ptr())
    fa_ws = torch.empty(mlz_b200.flash_attn_workspace_bytes(desc), dtype=torch.uint8, device=dev)

    def chain():
        x.copy_(x0)
        for _ in range(3):
            mlz_b200.mul_mat(Wq, x, out=q)
            mlz_b200.flash_attn_dispatch(q.view(B, Hq, 1, D), k, v, 1.0 / np.sqrt(D), kv_len=kv_len, out=att,
                                         workspace=fa_ws)
            mlz_b200.mul_mat(Wo, att.view(B, Hq * D), out=x)

    results = {}
    for mode in MODES:
        _in_mode(mode, chain)
        results[mode] = x.clone()
    ref = results[mlz_b200.OVERLAP_OFF]
    assert torch.isfinite(ref).all() and ref.abs().max() > 0
    for mode in MODES[1:]:
        assert torch.equal(results[mode], ref), f"mode {mode} differs from stream order"
