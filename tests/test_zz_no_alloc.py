"""The allocation-free attention entry point (b2_paged_attention_noalloc).

Some callers cannot allocate device memory when they run attention -- a plugin
whose host runtime owns all device memory through its own pool, or a hard
real-time decode loop that cannot take cudaMalloc's implicit device
synchronisation.  For them the library has an entry point whose workspace is a
fixed 4 MiB array compiled into the library.  These tests call it through the
C-ABI and check it against b2_paged_attention with a caller-provided workspace,
on two calls in a row with different inputs, within the attention tolerance of
the other GPU tests (max-abs 2e-3 for f16 K/V).  The file is named to be
collected last, so a run that stops at its first failure has already run
everything else; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-3  # the f16 attention tolerance used in tests/test_kernels_gpu.py


def _case(rng, b2, torch, batch, H, Dh, L, layer, ctx_hi):
    ctx = rng.integers(1, ctx_hi, size=batch).astype(np.int32)
    nbs = (ctx + 15) // 16
    mbps = int(nbs.max())
    nb = int(nbs.sum()) + 4
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((batch, mbps), np.int32)
    o = 0
    for b in range(batch):
        bt[b, : nbs[b]] = perm[o:o + nbs[b]]
        o += int(nbs[b])
    dev = torch.device("cuda:0")
    pool = torch.randn(nb * L * 2 * 16 * H * Dh, device=dev).half()
    q = torch.randn(batch, 3 * H * Dh, device=dev).half()  # q inside a fused QKV row
    btd = torch.from_numpy(bt).to(dev)
    sld = torch.from_numpy(ctx).to(dev)
    outs = [torch.full((batch, H, Dh), float("nan"), device=dev) for _ in range(2)]
    args = [b2.attn_args(q, 3 * H * Dh, pool, btd, sld, o, n_head=H, n_kv_head=H, head_dim=Dh,
                         max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, num_blocks=nb) for o in outs]
    return args, outs, (pool, q, btd, sld)


def test_noalloc_matches_workspace_entry_point_twice(b2, cuda):
    import torch
    lib = b2.load()
    lib.b2_paged_attention_noalloc.argtypes = [ctypes.POINTER(b2.PagedAttnArgs), ctypes.c_void_p]
    rng = np.random.Generator(np.random.PCG64(2026))
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # two calls in a row, different inputs: nothing stale may leak through
        (a_ref, a_na), (o_ref, o_na), keep = _case(rng, b2, torch, batch=24 + call, H=12, Dh=64, L=2, layer=1,
                                                   ctx_hi=700 + 300 * call)
        ws = b2.attention_workspace(a_ref)
        b2.paged_attention(a_ref, ws)
        rc = lib.b2_paged_attention_noalloc(ctypes.byref(a_na), stream)
        assert rc == 0, lib.b2_last_error_string().decode()
        torch.cuda.synchronize()
        assert torch.isfinite(o_na).all()
        err = (o_na - o_ref).abs().max().item()
        assert err <= TOL, f"call {call}: max-abs {err:.3g}"
    assert b2.device_errors() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch(b2, cuda):
    import torch
    lib = b2.load()
    lib.b2_paged_attention_noalloc.argtypes = [ctypes.POINTER(b2.PagedAttnArgs), ctypes.c_void_p]
    rng = np.random.Generator(np.random.PCG64(7))
    # 2048 sequences need ~15 MB of partials at 12 heads x 64 dims, far more than 4 MiB.
    (a_big, _), _, keep = _case(rng, b2, torch, batch=2048, H=12, Dh=64, L=1, layer=0, ctx_hi=3)
    assert lib.b2_paged_attention_workspace_bytes(ctypes.byref(a_big)) > 4 << 20
    rc = lib.b2_paged_attention_noalloc(ctypes.byref(a_big), torch.cuda.current_stream().cuda_stream)
    assert rc == -5  # B2_ERR_WORKSPACE, refused on the host before any launch
    assert "built-in scratch" in lib.b2_last_error_string().decode()
