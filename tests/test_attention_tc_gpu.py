"""The tensor-core decode-attention kernel (8 kv heads, head_dim 128, 16-bit K/V)
against the CPU oracle and, at the full grouped-query workload size, against a
torch fp32 restatement on the GPU (GPU).

Shapes with n_kv_head 8 and head_dim 128 are routed to paged_decode_tc_kernel
by the launcher; the cases below cover its block-boundary handling, pieces of
one sequence split across CTAs, q bias, 16-bit output, multi-layer pools and
NaN garbage past the end of each sequence.  Tolerance: max-abs 2e-3 with fp32
output, plus half an output ulp with 16-bit output (the bar of the CUDA-core
kernel's tests).
"""
from __future__ import annotations

import zlib

import numpy as np
import pytest

from oracle import oracle as O
from test_kernels_gpu import ULP_BITS, make_paged, run_attention

pytestmark = pytest.mark.gpu

NAN16 = {O.F16: 0x7E00, O.BF16: 0x7FC0}

TC_CASES = [
    # id, dtype, H, ctx (list or (B, lo, hi)), L, layer
    ("bf16-h32-boundaries", O.BF16, 32, [1, 2, 15, 16, 17, 31, 32, 33, 47, 48, 49, 64, 65, 300], 1, 0),
    ("f16-h32-random", O.F16, 32, (40, 1, 2000), 2, 1),
    ("bf16-h16", O.BF16, 16, (24, 1, 700), 1, 0),
    ("f16-h8", O.F16, 8, (17, 1, 900), 3, 2),
    ("bf16-one-long", O.BF16, 32, [20000], 1, 0),
    ("bf16-skew", O.BF16, 32, [9000] + list(range(1, 60, 3)), 1, 0),
    ("f16-empty", O.F16, 32, [0, 5, 0, 77, 0], 1, 0),
]


def _case_inputs(name, dt, H, ctx, L):
    rng = np.random.Generator(np.random.PCG64(zlib.crc32(name.encode())))
    if isinstance(ctx, tuple):
        B, lo, hi = ctx
        ctx = rng.integers(lo, hi + 1, size=B).tolist()
    pool, bt, mbps, nb = make_paged(rng, dt, ctx, 8, 128, L)
    q_stride = 3 * H * 128
    q = O.round_to(dt, rng.standard_normal(len(ctx) * q_stride, dtype=np.float32))
    return rng, ctx, pool, bt, mbps, nb, q, q_stride


@pytest.mark.parametrize("case", TC_CASES, ids=[c[0] for c in TC_CASES])
def test_tc_attention_matches_oracle(b2, cuda, case):
    name, dt, H, ctx, L, layer = case
    rng, ctx, pool, bt, mbps, nb, q, q_stride = _case_inputs(name, dt, H, ctx, L)
    ref = O.paged_attention(dt, q, q_stride, pool, np.where(bt < 0, 0, bt), ctx, n_head=H, n_kv_head=8, head_dim=128,
                            max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, nthreads=8)
    b2.device_errors()
    (got,), _ = run_attention(b2, dt, q, q_stride, pool, bt, ctx, H=H, Hkv=8, Dh=128, mbps=mbps, layer=layer, L=L,
                              nb=nb)
    err = np.max(np.abs(got - ref))
    assert np.isfinite(got).all()
    assert err <= 2e-3, f"max-abs {err:.3g}"
    assert b2.device_errors() == 0


@pytest.mark.parametrize("dt", [O.F16, O.BF16])
def test_tc_attention_bias_native_output_and_nan_tail(b2, cuda, dt):
    """q bias, 16-bit output, and NaN K/V rows past each sequence's end."""
    H, L, layer = 32, 2, 1
    rng, ctx, pool, bt, mbps, nb, q, q_stride = _case_inputs(f"bias-{dt}", dt, H, (30, 1, 400), L)
    pool = pool.reshape(nb, L, 2, 16, 8, 128)
    for b, c in enumerate(ctx):
        if c % 16:
            pool[bt[b, (c - 1) // 16], layer, :, c % 16:] = NAN16[dt]
    pool = pool.ravel()
    bias = O.round_to(dt, rng.standard_normal(H * 128, dtype=np.float32) * 0.5)
    qb = O.round_to(dt, O.widen(dt, q).reshape(len(ctx), -1)[:, : H * 128] + O.widen(dt, bias)[None, :])
    ref = O.paged_attention(dt, qb, H * 128, pool, bt, ctx, n_head=H, n_kv_head=8, head_dim=128,
                            max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, nthreads=8)
    (got,), _ = run_attention(b2, dt, q, q_stride, pool, bt, ctx, H=H, Hkv=8, Dh=128, mbps=mbps, layer=layer, L=L,
                              nb=nb, out_f32=False, q_bias=bias)
    bound = 2e-3 + np.abs(ref) * 2.0 ** -(ULP_BITS[dt] + 1)
    assert np.isfinite(got).all()
    assert np.all(np.abs(got - ref) <= bound)


def test_tc_attention_repeat_launches_are_identical(b2, cuda):
    dt = O.BF16
    rng, ctx, pool, bt, mbps, nb, q, q_stride = _case_inputs("repeat", dt, 32, [3000, 17, 2500, 900, 5], 1)
    outs, _ = run_attention(b2, dt, q, q_stride, pool, bt, ctx, H=32, Hkv=8, Dh=128, mbps=mbps, layer=0, L=1, nb=nb,
                            repeats=3)
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


def test_tc_attention_full_gqa_workload_sampled(b2, cuda):
    """Batch 256, 32 query / 8 kv heads, head_dim 128, bf16, contexts
    log-uniform in [512, 32768] (~7 GB of KV): every output finite, and 12
    sequences (the longest, the shortest, 10 random) checked against the
    oracle (the reference CPU attention, cpu_model.cpp:131-162, through a
    block table) on their own blocks, gathered into a compact host pool."""
    import torch
    from lis_b200.workloads import make_attention_workload
    wl = make_attention_workload(cuda, seed=3, n_sets=1, batch=256, n_head=32, n_kv_head=8, head_dim=128,
                                 ctx_lo=512, ctx_hi=32768, pool_blocks=140000, dtype=torch.bfloat16, log_uniform=True,
                                 out_dtype=torch.float32)
    s = wl.sets[0]
    ws = b2.attention_workspace(s.args)
    b2.device_errors()
    b2.paged_attention(s.args, ws)
    torch.cuda.synchronize()
    assert b2.device_errors() == 0
    out = s.d_out
    assert torch.isfinite(out).all()
    rng = np.random.default_rng(0)
    ctx = s.seq_lens
    pick = {int(np.argmax(ctx)), int(np.argmin(ctx))} | set(rng.choice(len(ctx), 10, replace=False).tolist())
    pool = wl.pool.view(wl.pool_blocks, 2 * 16 * 8 * 128)
    for b in sorted(pick):
        c = int(ctx[b])
        nblk = (c + 15) // 16
        blocks = torch.from_numpy(s.block_tables[b, :nblk].astype(np.int64)).cuda()
        mini = pool[blocks].contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
        qb = s.d_q[b].contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
        ref = O.paged_attention(O.BF16, qb, 32 * 128, mini, np.arange(nblk, dtype=np.int32)[None, :],
                                np.array([c], np.int32), n_head=32, n_kv_head=8, head_dim=128,
                                max_blocks_per_seq=nblk, layer_idx=0, n_layer=1, nthreads=8)
        err = float(np.max(np.abs(out[b].cpu().numpy().reshape(-1) - np.asarray(ref).reshape(-1))))
        assert err <= 2e-3, f"sequence {b} (ctx {c}): max-abs {err:.3g} against the oracle"
