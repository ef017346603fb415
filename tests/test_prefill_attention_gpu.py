"""b2_prefill_attention (tcgen05 causal prefill over the paged pool) against
the CPU oracle, through the C-ABI (GPU).

Row i of sequence b sits at position seq_lens_pre[b] + i and must equal the
oracle's decode attention (restatement of cpu_model.cpp:131-162) for that row
with seq_len = position + 1 -- what the reference computes when it walks the
prompt through Engine::decode_step one token at a time.  Tolerance: max-abs
2e-3 plus half an output ulp (16-bit output), the decode kernels' bar.
"""
from __future__ import annotations

import zlib

import numpy as np
import pytest

from oracle import oracle as O

from test_kernels_gpu import ULP_BITS, ints_dev, to_dev

pytestmark = pytest.mark.gpu

NAN16 = {O.F16: 0x7E00, O.BF16: 0x7FC0}


def _build(rng, dt, seqs, H, Hkv, L, layer, stale_nan):
    """seqs: [(pre, T)].  Pool with every sequence's keys, random block order;
    rows of each sequence's last block past its keys are NaN when stale_nan."""
    Dh = 64
    nb_seq = [(pre + t + 15) // 16 for pre, t in seqs]
    mbps = max(nb_seq)
    nb = sum(nb_seq) + 3
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.full((len(seqs), mbps), -1, np.int32)
    o = 0
    for b, n in enumerate(nb_seq):
        bt[b, :n] = perm[o:o + n]
        o += n
    pool = O.round_to(dt, rng.standard_normal(nb * L * 2 * 16 * Hkv * Dh, dtype=np.float32))
    if stale_nan:
        pv = pool.reshape(nb, L, 2, 16, Hkv, Dh)
        for b, (pre, t) in enumerate(seqs):
            end = pre + t
            if end % 16:
                pv[bt[b, (end - 1) // 16], layer, :, end % 16:, :, :] = NAN16[dt]
    return pool, bt, mbps, nb


CASES = [
    # id, dtype, H, Hkv, [(pre, T)], L, layer, bias
    ("f16-tile-edges", O.F16, 4, 4, [(0, 1), (0, 17), (0, 128), (0, 129), (0, 255)], 1, 0, False),
    ("bf16-cached-prefix", O.BF16, 6, 6, [(37, 50), (200, 256), (5, 300), (1000, 130)], 2, 1, True),
    ("f16-gpt2-medium-heads", O.F16, 16, 16, [(0, 512), (0, 33), (16, 100)], 1, 0, True),
    ("bf16-gqa4", O.BF16, 8, 2, [(0, 200), (64, 64), (3, 7)], 1, 0, False),
    # 480 (sequence, head, query tile) CTAs, ragged lengths and cached prefixes:
    # more than three waves of one CTA per SM
    ("f16-many-items-per-cta", O.F16, 16, 16,
     [(0, 512), (0, 300), (50, 256), (0, 140), (200, 384), (0, 64), (0, 512), (30, 129), (0, 400), (0, 200),
      (90, 96), (0, 256)], 2, 1, True),
]


@pytest.mark.parametrize("stale_nan", [False, True])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_prefill_attention_matches_oracle(b2, cuda, case, stale_nan):
    import torch
    name, dt, H, Hkv, seqs, L, layer, with_bias = case
    Dh = 64
    rng = np.random.Generator(np.random.PCG64(zlib.crc32(name.encode())))
    pool, bt, mbps, nb = _build(rng, dt, seqs, H, Hkv, L, layer, stale_nan)
    lens = [t for _, t in seqs]
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int32)
    rows = int(sum(lens))
    q_stride = 3 * H * Dh  # q inside a fused QKV row, like the engine's
    q = O.round_to(dt, rng.standard_normal(rows * q_stride, dtype=np.float32))
    bias = O.round_to(dt, rng.standard_normal(H * Dh, dtype=np.float32) * 0.5) if with_bias else None
    # oracle: one decode row per prompt row, seq_len = position + 1
    q_or = q.reshape(rows, q_stride)[:, :H * Dh]
    if with_bias:
        q_or = O.round_to(dt, O.widen(dt, q_or) + O.widen(dt, bias)[None, :])
    bt_rows = np.concatenate([np.repeat(np.where(bt[b:b + 1] < 0, 0, bt[b:b + 1]), t, axis=0)
                              for b, (_, t) in enumerate(seqs)])
    sl_rows = np.concatenate([np.arange(pre + 1, pre + t + 1) for pre, t in seqs]).astype(np.int32)
    ref = O.paged_attention(dt, np.ascontiguousarray(q_or), H * Dh, pool, bt_rows, sl_rows, n_head=H, n_kv_head=Hkv,
                            head_dim=Dh, max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, nthreads=8)
    tdt = torch.float16 if dt == O.F16 else torch.bfloat16
    out = torch.full((rows, H * Dh), float("nan"), dtype=tdt, device="cuda")
    b2.prefill_attention(out, to_dev(dt, q), q_stride, to_dev(dt, pool), ints_dev(bt),
                         ints_dev([pre for pre, _ in seqs]), ints_dev(starts), ints_dev(lens), n_head=H, n_kv_head=Hkv,
                         head_dim=Dh, max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, num_blocks=nb,
                         max_q_len=max(lens), q_bias=None if bias is None else to_dev(dt, bias))
    torch.cuda.synchronize()
    assert b2.device_errors() == 0
    got = out.float().cpu().numpy().reshape(rows, H, Dh)
    assert np.isfinite(got).all()
    bound = 2e-3 + np.abs(ref) * 2.0 ** -(ULP_BITS[dt] + 1)
    bad = np.abs(got - ref) > bound
    assert not bad.any(), f"{bad.sum()} outputs off; worst {np.max(np.abs(got - ref)):.3g}"


def test_prefill_attention_argument_errors(b2, cuda):
    import torch
    z = torch.zeros(16, 3 * 64, dtype=torch.float16, device="cuda")
    pool = torch.zeros(4 * 2 * 16 * 64, dtype=torch.float16, device="cuda")
    i = ints_dev([0])
    kw = dict(n_head=1, n_kv_head=1, head_dim=64, max_blocks_per_seq=1, layer_idx=0, n_layer=1, num_blocks=4,
              max_q_len=16)
    out = torch.zeros(16, 64, dtype=torch.float16, device="cuda")
    b2.prefill_attention(out, z, 3 * 64, pool, i, i, i, ints_dev([16]), **kw)  # valid
    with pytest.raises(b2.B2Error) as e:
        b2.prefill_attention(out.float(), z.float(), 3 * 64, pool.float(), i, i, i, ints_dev([16]), **kw)
    assert e.value.code == -2
    with pytest.raises(b2.B2Error) as e:
        b2.prefill_attention(out, z, 3 * 64, pool, i, i, i, ints_dev([16]), **{**kw, "head_dim": 128})
    assert e.value.code == -6
    torch.cuda.synchronize()
    assert b2.device_errors() == 0
