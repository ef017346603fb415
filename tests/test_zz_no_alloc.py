"""The allocation-free attention entry point (b2_paged_attention_noalloc).

Some callers cannot allocate device memory when they run attention -- a plugin
whose host runtime owns all device memory through its own pool, or a hard
real-time decode loop that cannot take cudaMalloc's implicit device
synchronisation.  For them the library has an entry point whose workspace is a
fixed 4 MiB array compiled into the library.  These tests call it through the
C-ABI on two calls in a row with different inputs and check each output
against b2_paged_attention with a caller-provided workspace and against the
CPU oracle, within the attention tolerance of the other GPU tests (max-abs
2e-3 for 16-bit K/V, fp32 output).  They cover the CUDA-core kernel (with and
without the early-start flag) and the tensor-core grouped-query kernel.  The
file is named to be collected last, so a run that stops at its first failure
has already run everything else; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-3  # the 16-bit attention tolerance used in tests/test_kernels_gpu.py


def _case(rng, b2, torch, dt, batch, H, Hkv, Dh, L, layer, ctx_hi, flags=0):
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
    q_stride = (H + 2 * Hkv) * Dh  # q inside a fused QKV row
    pool = O.round_to(dt, rng.standard_normal(nb * L * 2 * 16 * Hkv * Dh, dtype=np.float32))
    q = O.round_to(dt, rng.standard_normal(batch * q_stride, dtype=np.float32))
    ref = O.paged_attention(dt, q, q_stride, pool, bt, ctx, n_head=H, n_kv_head=Hkv, head_dim=Dh,
                            max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, nthreads=8)
    tdt = torch.float16 if dt == O.F16 else torch.bfloat16
    dev = torch.device("cuda:0")
    pd = torch.from_numpy(pool.view(np.int16)).to(dev).view(tdt)
    qd = torch.from_numpy(q.view(np.int16)).to(dev).view(tdt)
    btd = torch.from_numpy(bt).to(dev)
    sld = torch.from_numpy(ctx).to(dev)
    outs = [torch.full((batch, H, Dh), float("nan"), device=dev) for _ in range(2)]
    args = [b2.attn_args(qd, q_stride, pd, btd, sld, o, n_head=H, n_kv_head=Hkv, head_dim=Dh,
                         max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, num_blocks=nb) for o in outs]
    for a in args:
        a.flags = flags
    return args, outs, ref, (pd, qd, btd, sld)


CASES = [
    # id, dtype, batch, H, Hkv, Dh, L, layer, ctx_hi, flags
    ("f16-mha-layer1", O.F16, 24, 12, 12, 64, 2, 1, 700, 0),
    ("f16-mha-inputs-ready", O.F16, 20, 12, 12, 64, 1, 0, 900, 1),  # B2_ATTN_INPUTS_READY
    ("bf16-gqa-tensor-cores", O.BF16, 4, 32, 8, 128, 1, 0, 1500, 0),  # 8 kv heads of 128: the tcgen05 kernel
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_noalloc_matches_workspace_entry_point_and_oracle_twice(b2, cuda, case):
    import torch
    name, dt, batch, H, Hkv, Dh, L, layer, ctx_hi, flags = case
    lib = b2.load()
    rng = np.random.Generator(np.random.PCG64(2026 + len(name)))
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # two calls in a row, different inputs: nothing stale may leak through
        (a_ref, a_na), (o_ref, o_na), ref, keep = _case(rng, b2, torch, dt, batch + call, H, Hkv, Dh, L, layer,
                                                        ctx_hi + 300 * call, flags)
        ws = b2.attention_workspace(a_ref)
        b2.paged_attention(a_ref, ws)
        rc = lib.b2_paged_attention_noalloc(ctypes.byref(a_na), stream)
        assert rc == 0, lib.b2_last_error_string().decode()
        torch.cuda.synchronize()
        got = o_na.cpu().numpy()
        assert np.isfinite(got).all()
        err_entry = float(np.max(np.abs(got - o_ref.cpu().numpy())))
        err_oracle = float(np.max(np.abs(got - ref.reshape(got.shape))))
        assert err_entry <= TOL, f"call {call}: max-abs {err_entry:.3g} against b2_paged_attention"
        assert err_oracle <= TOL, f"call {call}: max-abs {err_oracle:.3g} against the oracle"
    assert b2.device_errors() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch(b2, cuda):
    import torch
    lib = b2.load()
    rng = np.random.Generator(np.random.PCG64(7))
    # 2048 sequences need ~15 MB of partials at 12 heads x 64 dims, far more than 4 MiB.
    (a_big, _), _, _, keep = _case(rng, b2, torch, O.F16, 2048, 12, 12, 64, 1, 0, 3)
    assert lib.b2_paged_attention_workspace_bytes(ctypes.byref(a_big)) > 4 << 20
    rc = lib.b2_paged_attention_noalloc(ctypes.byref(a_big), torch.cuda.current_stream().cuda_stream)
    assert rc == -5  # B2_ERR_WORKSPACE, refused on the host before any launch
    assert "built-in scratch" in lib.b2_last_error_string().decode()
