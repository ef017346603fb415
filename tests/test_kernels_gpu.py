"""Parity of the sm_100a kernels with the CPU oracle, through the C-ABI (GPU).

Tolerances (the bar stated for this path):
  * KV append, embedding, bias add, argmax, residual sums: bit-exact;
  * paged attention: max-abs 2e-3 for f16/bf16 K/V (fp32 output), 1e-5 for f32;
    with 16-bit output, 2e-3 plus half an output ulp of the oracle value;
  * LayerNorm / GELU: within one ulp of the output dtype of the oracle value
    (f32: 2e-6 relative + 1e-6 absolute; the GPU reduces in a different order);
  * the reference's own kernel KATs (tests/golden/kernel_kat.json): max-abs 5e-2,
    the reference's bar (gpu-engine/tests/test_kernels.cpp:89,152,194).
"""
from __future__ import annotations

import zlib

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

ULP_BITS = {O.F32: 23, O.F16: 10, O.BF16: 7}


def _torch():
    import torch
    return torch


def to_dev(dt, arr):
    torch = _torch()
    arr = np.ascontiguousarray(arr)
    if dt == O.F32:
        return torch.from_numpy(arr.astype(np.float32)).cuda()
    t = torch.from_numpy(arr.view(np.int16)).cuda()
    return t.view(torch.float16 if dt == O.F16 else torch.bfloat16)


def from_dev(dt, t):
    torch = _torch()
    t = t.detach().cpu().contiguous()
    if dt == O.F32:
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def ints_dev(a):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).cuda()


def make_paged(rng, dt, ctx, n_kv_head, head_dim, n_layer, slack=8, extra_slots=0):
    """Random pool holding exactly the blocks the contexts need (+ slack), random
    block permutation, block tables padded with -1 beyond each sequence."""
    nb_seq = [(c + 15) // 16 for c in ctx]
    mbps = max(1, max(nb_seq) + extra_slots)
    num_blocks = sum(nb_seq) + slack
    perm = rng.permutation(num_blocks).astype(np.int32)
    bt = np.full((len(ctx), mbps), -1, np.int32)
    o = 0
    for b, n in enumerate(nb_seq):
        bt[b, :n] = perm[o:o + n]
        o += n
    n_el = num_blocks * n_layer * 2 * 16 * n_kv_head * head_dim
    pool = O.round_to(dt, rng.standard_normal(n_el, dtype=np.float32))
    return pool, bt, mbps, num_blocks


def run_attention(b2, dt, q, q_stride, pool, bt, ctx, *, H, Hkv, Dh, mbps, layer, L, nb, out_f32=True, q_bias=None,
                  repeats=1, ws=None):
    torch = _torch()
    B = len(ctx)
    qd = to_dev(dt, q)
    pd = to_dev(dt, pool)
    btd, sld = ints_dev(bt), ints_dev(ctx)
    tdt = {O.F32: torch.float32, O.F16: torch.float16, O.BF16: torch.bfloat16}[dt]
    out = torch.full((B, H, Dh), float("nan"), dtype=torch.float32 if out_f32 else tdt, device="cuda")
    qb = None if q_bias is None else to_dev(dt, q_bias)
    args = b2.attn_args(qd, q_stride, pd, btd, sld, out, n_head=H, n_kv_head=Hkv, head_dim=Dh, max_blocks_per_seq=mbps,
                        layer_idx=layer, n_layer=L, num_blocks=nb, q_bias=qb)
    if ws is None:
        ws = b2.attention_workspace(args)
    outs = []
    for _ in range(repeats):
        b2.paged_attention(args, ws)
        torch.cuda.synchronize()
        outs.append(out.float().cpu().numpy().copy())
    return outs, ws


ATTN_CASES = [
    # id, dtype, Dh, H, Hkv, ctx (list or (B, lo, hi)), L, layer
    ("f16-mha-boundaries", O.F16, 64, 12, 12, [1, 15, 16, 17, 31, 32, 33, 200], 1, 0),
    ("f16-microbench-shape", O.F16, 64, 12, 12, (64, 128, 1024), 1, 0),
    ("f32-gpt2-small-shape", O.F32, 64, 12, 12, (8, 16, 192), 12, 5),
    ("bf16-xl-heads", O.BF16, 64, 25, 25, (9, 1, 300), 3, 2),
    ("bf16-gqa4-d128", O.BF16, 128, 32, 8, [512, 700, 33, 1000, 1], 1, 0),
    ("f16-gqa2-d128", O.F16, 128, 16, 8, (6, 1, 400), 2, 1),
    ("f16-d128-mha", O.F16, 128, 8, 8, (5, 1, 300), 1, 0),
    ("f32-gqa8", O.F32, 64, 16, 2, (4, 1, 100), 1, 0),
    ("f16-one-long-sequence", O.F16, 64, 12, 12, [5000], 1, 0),
    ("bf16-skew", O.BF16, 64, 12, 12, [6000] + list(range(1, 41)), 1, 0),
    ("f16-empty-sequences", O.F16, 64, 4, 4, [0, 7, 0, 100, 0], 1, 0),
    ("f16-gpt2-medium-heads", O.F16, 64, 16, 16, (40, 1, 1000), 1, 0),  # 3 token subgroups
    ("f32-xl-heads", O.F32, 64, 25, 25, (6, 1, 300), 2, 1),  # 6.4 KB rows: the 8-row-stage fallback plan
]


@pytest.mark.parametrize("case", ATTN_CASES, ids=[c[0] for c in ATTN_CASES])
def test_paged_attention_matches_oracle(b2, cuda, case):
    name, dt, Dh, H, Hkv, ctx, L, layer = case
    rng = np.random.Generator(np.random.PCG64(zlib.crc32(name.encode())))
    if isinstance(ctx, tuple):
        B, lo, hi = ctx
        ctx = rng.integers(lo, hi + 1, size=B).tolist()
    B = len(ctx)
    pool, bt, mbps, nb = make_paged(rng, dt, ctx, Hkv, Dh, L)
    q_stride = 3 * H * Dh  # q lives inside a fused QKV row, like the engine's
    q = O.round_to(dt, rng.standard_normal(B * q_stride, dtype=np.float32))
    bt_oracle = np.where(bt < 0, 0, bt)
    ref = O.paged_attention(dt, q, q_stride, pool, bt_oracle, ctx, n_head=H, n_kv_head=Hkv, head_dim=Dh,
                            max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, nthreads=8)
    (got,), _ = run_attention(b2, dt, q, q_stride, pool, bt, ctx, H=H, Hkv=Hkv, Dh=Dh, mbps=mbps, layer=layer, L=L,
                              nb=nb)
    tol = 1e-5 if dt == O.F32 else 2e-3
    err = np.max(np.abs(got - ref))
    assert np.isfinite(got).all()
    assert err <= tol, f"max-abs {err:.3g} > {tol}"
    assert b2.device_errors() == 0


@pytest.mark.parametrize("dt", [O.F16, O.BF16])
def test_paged_attention_native_output_and_bias(b2, cuda, dt):
    rng = np.random.Generator(np.random.PCG64(7))
    H, Dh, L = 12, 64, 2
    ctx = rng.integers(1, 600, size=20).tolist()
    pool, bt, mbps, nb = make_paged(rng, dt, ctx, H, Dh, L)
    q = O.round_to(dt, rng.standard_normal(len(ctx) * H * Dh, dtype=np.float32))
    bias = O.round_to(dt, rng.standard_normal(H * Dh, dtype=np.float32) * 0.5)
    # the kernel adds the bias and rounds q + bias to the storage dtype
    qb = O.round_to(dt, O.widen(dt, q).reshape(len(ctx), -1) + O.widen(dt, bias)[None, :])
    ref = O.paged_attention(dt, qb, H * Dh, pool, bt, ctx, n_head=H, n_kv_head=H, head_dim=Dh,
                            max_blocks_per_seq=mbps, layer_idx=1, n_layer=L, nthreads=8)
    (got,), _ = run_attention(b2, dt, q, H * Dh, pool, bt, ctx, H=H, Hkv=H, Dh=Dh, mbps=mbps, layer=1, L=L, nb=nb,
                              out_f32=False, q_bias=bias)
    bound = 2e-3 + np.abs(ref) * 2.0 ** -(ULP_BITS[dt] + 1)
    assert np.all(np.abs(got - ref) <= bound)


@pytest.mark.parametrize("dt,Dh,H,Hkv,packed,pinned_in,flags", [
    (O.F16, 64, 12, 12, True, True, 0), (O.F16, 64, 12, 12, False, True, 1), (O.F16, 64, 12, 12, True, False, 1),
    (O.BF16, 128, 32, 8, True, True, 0), (O.F32, 64, 8, 4, False, False, 0)])
def test_paged_attention_host_buffers(b2, cuda, dt, Dh, H, Hkv, packed, pinned_in, flags):
    """b2_paged_attention_host: uploads from host memory (page-locked: read by
    a kernel over the bus; pageable: copies, one when q | block tables |
    seq_lens are back to back on both sides), launch, output to the host
    (stored by the kernel into pinned memory, or copied into pageable memory),
    sync -- two calls with different inputs through the same device buffers,
    each against the oracle.  With B2_ATTN_INPUTS_READY set the call must
    still wait for its own uploads."""
    torch = _torch()
    rng = np.random.Generator(np.random.PCG64(11 + Dh + H))
    L, layer, B = 2, 1, 9
    ctx_a = rng.integers(1, 700, size=B).tolist()
    ctx_b = rng.integers(1, 700, size=B).tolist()
    ctx_b[0] = 0
    pool, _, mbps, nb = make_paged(rng, dt, [max(a, b) for a, b in zip(ctx_a, ctx_b)], Hkv, Dh, L)
    q_stride = 3 * H * Dh  # q inside a fused QKV row: the upload covers (B-1) strides + one row
    es = 4 if dt == O.F32 else 2
    qn = (B - 1) * q_stride + H * Dh
    q_bytes, bt_bytes = qn * es, B * mbps * 4
    pd = to_dev(dt, pool)
    if packed:
        d_in = torch.empty(q_bytes + bt_bytes + 4 * B, dtype=torch.uint8, device="cuda")
        qd, btd, sld = d_in[:q_bytes], d_in[q_bytes:q_bytes + bt_bytes], d_in[q_bytes + bt_bytes:]
    else:
        qd = torch.empty(q_bytes, dtype=torch.uint8, device="cuda")
        btd = torch.empty(bt_bytes, dtype=torch.uint8, device="cuda")
        sld = torch.empty(4 * B, dtype=torch.uint8, device="cuda")
    out = torch.empty(B, H, Dh, dtype=torch.float32, device="cuda")
    args = b2.attn_args(qd, q_stride, pd, btd.view(torch.int32).view(B, mbps), sld.view(torch.int32), out,
                        n_head=H, n_kv_head=Hkv, head_dim=Dh, max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L,
                        num_blocks=nb)
    args.flags = flags
    ws = b2.attention_workspace(args)
    perm = rng.permutation(nb).astype(np.int32)
    for ctx in (ctx_a, ctx_b):
        bt = np.full((B, mbps), -1, np.int32)
        o = 0
        for i, c in enumerate(ctx):
            n = (c + 15) // 16
            bt[i, :n] = perm[o:o + n]
            o += n
        q = O.round_to(dt, rng.standard_normal(qn, dtype=np.float32))
        host = torch.from_numpy(np.concatenate([np.ascontiguousarray(q).view(np.uint8), bt.view(np.uint8).reshape(-1),
                                                np.asarray(ctx, np.int32).view(np.uint8)]))
        if pinned_in:
            host = host.pin_memory()
        # pinned (mapped) output: the kernel stores into it; pageable: copied from args.out
        hout = torch.empty(B, H, Dh, dtype=torch.float32)
        if packed:
            hout = hout.pin_memory()
        b2.paged_attention_host(args, ws, q=host[:q_bytes], block_tables=host[q_bytes:q_bytes + bt_bytes],
                                seq_lens=host[q_bytes + bt_bytes:], out=hout)
        got = hout.numpy()  # the call has synchronised: no further sync before reading
        q_full = np.zeros(B * q_stride, q.dtype)
        q_full[:qn] = q
        ref = O.paged_attention(dt, q_full, q_stride, pool, np.where(bt < 0, 0, bt), ctx, n_head=H, n_kv_head=Hkv,
                                head_dim=Dh, max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, nthreads=8)
        tol = 1e-5 if dt == O.F32 else 2e-3
        assert np.isfinite(got).all()
        assert float(np.max(np.abs(got - ref))) <= tol
    assert b2.device_errors() == 0


def test_paged_attention_repeat_launches_are_identical(b2, cuda):
    """The merge counters are left at zero, so a reused workspace gives the same bits."""
    rng = np.random.Generator(np.random.PCG64(3))
    ctx = [3000, 17, 2500, 900]
    pool, bt, mbps, nb = make_paged(rng, O.F16, ctx, 12, 64, 1)
    q = O.round_to(O.F16, rng.standard_normal(len(ctx) * 768, dtype=np.float32))
    outs, _ = run_attention(b2, O.F16, q, 768, pool, bt, ctx, H=12, Hkv=12, Dh=64, mbps=mbps, layer=0, L=1, nb=nb,
                            repeats=4)
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


def test_paged_attention_flags_bad_block_ids(b2, cuda):
    rng = np.random.Generator(np.random.PCG64(5))
    ctx = [40, 20]
    pool, bt, mbps, nb = make_paged(rng, O.F16, ctx, 4, 64, 1)
    bt[0, 1] = nb + 100  # outside the pool
    b2.device_errors()
    q = O.round_to(O.F16, rng.standard_normal(len(ctx) * 256, dtype=np.float32))
    (got,), _ = run_attention(b2, O.F16, q, 256, pool, bt, ctx, H=4, Hkv=4, Dh=64, mbps=mbps, layer=0, L=1, nb=nb)
    assert b2.device_errors() & b2.DEVERR_BLOCK_ID
    assert np.isfinite(got).all()


def test_paged_attention_flags_overlong_seq_len(b2, cuda):
    rng = np.random.Generator(np.random.PCG64(6))
    ctx = [20, 10]
    pool, bt, mbps, nb = make_paged(rng, O.F16, ctx, 4, 64, 1)
    b2.device_errors()
    q = O.round_to(O.F16, rng.standard_normal(2 * 256, dtype=np.float32))
    run_attention(b2, O.F16, q, 256, pool, bt, [mbps * 16 + 5, 10], H=4, Hkv=4, Dh=64, mbps=mbps, layer=0, L=1, nb=nb)
    assert b2.device_errors() & b2.DEVERR_SEQ_LEN


# ------------------------------------------------------------------ append

APPEND_CASES = [
    ("f16-d64", O.F16, 64, 12, 1, 0, False),
    ("bf16-d128-gqa", O.BF16, 128, 8, 2, 1, False),
    ("f32-d64-layers", O.F32, 64, 12, 12, 7, False),
    ("f16-bias", O.F16, 64, 16, 3, 2, True),
    ("bf16-bias-d128", O.BF16, 128, 4, 1, 0, True),
]


@pytest.mark.parametrize("case", APPEND_CASES, ids=[c[0] for c in APPEND_CASES])
def test_kv_append_is_bit_exact(b2, cuda, case):
    torch = _torch()
    name, dt, Dh, Hkv, L, layer, with_bias = case
    rng = np.random.Generator(np.random.PCG64(zlib.crc32(name.encode())))
    pos = np.array([0, 1, 15, 16, 17, 31, 32, 100, 255, 3], np.int32)
    B = len(pos)
    pool, bt, mbps, nb = make_paged(rng, dt, (pos + 1).tolist(), Hkv, Dh, L)
    stride = 3 * Hkv * Dh + 16  # strided rows inside a fused buffer
    qkv = O.round_to(dt, rng.standard_normal(B * stride, dtype=np.float32)).reshape(B, stride)
    kb = vb = None
    if with_bias:
        kb = O.round_to(dt, rng.standard_normal(Hkv * Dh, dtype=np.float32))
        vb = O.round_to(dt, rng.standard_normal(Hkv * Dh, dtype=np.float32))
    # oracle on host
    ref_pool = pool.copy()
    kh = np.ascontiguousarray(qkv[:, Hkv * Dh:])
    vh = np.ascontiguousarray(qkv[:, 2 * Hkv * Dh:])
    kpad = np.zeros_like(qkv)
    vpad = np.zeros_like(qkv)
    kpad[:, : kh.shape[1]] = kh
    vpad[:, : vh.shape[1]] = vh
    if with_bias:
        kpad[:, : Hkv * Dh] = O.round_to(dt, O.widen(dt, kpad[:, : Hkv * Dh]) + O.widen(dt, kb)[None, :])
        vpad[:, : Hkv * Dh] = O.round_to(dt, O.widen(dt, vpad[:, : Hkv * Dh]) + O.widen(dt, vb)[None, :])
    O.kv_append(dt, ref_pool, kpad, vpad, stride, bt, pos, n_kv_head=Hkv, head_dim=Dh, max_blocks_per_seq=mbps,
                layer_idx=layer, n_layer=L, num_blocks=nb)
    # GPU
    pd = to_dev(dt, pool)
    qkvd = to_dev(dt, qkv.ravel()).view(B, stride)
    post = torch.zeros(B, dtype=torch.int32, device="cuda")
    b2.kv_append(pd, qkvd[:, Hkv * Dh:], qkvd[:, 2 * Hkv * Dh:], stride, ints_dev(bt), ints_dev(pos),
                 n_kv_head=Hkv, head_dim=Dh, max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, num_blocks=nb,
                 k_bias=None if kb is None else to_dev(dt, kb), v_bias=None if vb is None else to_dev(dt, vb),
                 seq_lens_post=post)
    torch.cuda.synchronize()
    assert np.array_equal(from_dev(dt, pd), ref_pool)
    assert post.cpu().numpy().tolist() == (pos + 1).tolist()


def test_kv_append_refuses_bad_block(b2, cuda):
    torch = _torch()
    rng = np.random.Generator(np.random.PCG64(9))
    pool, bt, mbps, nb = make_paged(rng, O.F16, [5, 5], 2, 64, 1)
    bt[1, 0] = -3
    before = pool.copy()
    pd = to_dev(O.F16, pool)
    kv = torch.randn(2, 128, device="cuda").half()
    b2.device_errors()
    b2.kv_append(pd, kv, kv, 128, ints_dev(bt), ints_dev([4, 4]), n_kv_head=2, head_dim=64, max_blocks_per_seq=mbps,
                 layer_idx=0, n_layer=1, num_blocks=nb)
    torch.cuda.synchronize()
    assert b2.device_errors() & b2.DEVERR_BLOCK_ID
    after = from_dev(O.F16, pd).reshape(nb, 2, 16, 2, 64)
    # sequence 0 was written, sequence 1 (bad block) was not
    assert np.array_equal(after[bt[0, 0], 0, 4].ravel(), kv[0].cpu().numpy().view(np.uint16))
    diff = np.argwhere(np.any(after != before.reshape(nb, 2, 16, 2, 64), axis=-1))
    assert all(int(d[0]) == int(bt[0, 0]) for d in diff)


# ------------------------------------------------------------ row kernels

def _ulp_close(dt, got, ref):
    if dt == O.F32:
        return np.all(np.abs(got - ref) <= 2e-6 * np.abs(ref) + 1e-6)
    return np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -ULP_BITS[dt] + 2.0 ** -24)


@pytest.mark.parametrize("dt", [O.F32, O.F16, O.BF16])
@pytest.mark.parametrize("D,B,with_x,with_bias", [(32, 3, True, False), (768, 8, True, True), (1024, 64, False, True),
                                                  (1600, 33, True, True), (2048, 2, True, False)])
def test_add_layernorm_matches_oracle(b2, cuda, dt, D, B, with_x, with_bias):
    torch = _torch()
    rng = np.random.Generator(np.random.PCG64(D + B))
    x = O.round_to(dt, rng.standard_normal((B, D), dtype=np.float32) * 2) if with_x else None
    r = O.round_to(dt, rng.standard_normal((B, D), dtype=np.float32) * 2)
    bias = O.round_to(dt, rng.standard_normal(D, dtype=np.float32)) if with_bias else None
    g = O.round_to(dt, 1 + 0.1 * rng.standard_normal(D, dtype=np.float32))
    be = O.round_to(dt, 0.1 * rng.standard_normal(D, dtype=np.float32))
    ref, _, ref_res = O.add_layernorm(dt, x, r, g, be, 1e-5, bias=bias)
    rd = to_dev(dt, r)
    xd = None if x is None else to_dev(dt, x)
    out = torch.empty_like(rd)
    b2.add_layernorm(out, rd, xd, rd, to_dev(dt, g), to_dev(dt, be), 1e-5,
                     bias=None if bias is None else to_dev(dt, bias))  # residual updated in place
    torch.cuda.synchronize()
    assert np.array_equal(from_dev(dt, rd), ref_res)
    assert _ulp_close(dt, O.widen(dt, from_dev(dt, out)), ref)


@pytest.mark.parametrize("dt", [O.F32, O.F16, O.BF16])
def test_bias_gelu_and_add_bias(b2, cuda, dt):
    torch = _torch()
    rng = np.random.Generator(np.random.PCG64(11))
    B, D = 13, 3072
    x = O.round_to(dt, rng.standard_normal((B, D), dtype=np.float32) * 3)
    bias = O.round_to(dt, rng.standard_normal(D, dtype=np.float32))
    xd, bd = to_dev(dt, x), to_dev(dt, bias)
    out = torch.empty_like(xd)
    b2.bias_gelu(out, xd, bd)
    torch.cuda.synchronize()
    assert _ulp_close(dt, O.widen(dt, from_dev(dt, out)), O.bias_gelu(dt, x, bias))
    b2.add_bias(xd, xd, bd)  # in place
    torch.cuda.synchronize()
    assert np.array_equal(from_dev(dt, xd), O.round_to(dt, O.add_bias(dt, x, bias)))


@pytest.mark.parametrize("dt", [O.F32, O.F16, O.BF16])
def test_embedding_and_argmax(b2, cuda, dt):
    torch = _torch()
    rng = np.random.Generator(np.random.PCG64(12))
    V, P, D, B = 1000, 64, 768, 9
    wte = O.round_to(dt, rng.standard_normal((V, D), dtype=np.float32))
    wpe = O.round_to(dt, rng.standard_normal((P, D), dtype=np.float32))
    tok = rng.integers(0, V, size=B).astype(np.int32)
    pos = rng.integers(0, P, size=B).astype(np.int32)
    out = torch.empty(B, D, device="cuda", dtype=to_dev(dt, wte[:1]).dtype)
    b2.embedding(out, to_dev(dt, wte), to_dev(dt, wpe), ints_dev(tok), ints_dev(pos))
    torch.cuda.synchronize()
    assert np.array_equal(from_dev(dt, out), O.round_to(dt, O.embedding(dt, wte, wpe, tok, pos)))
    logits = O.round_to(dt, rng.standard_normal((B, 50257), dtype=np.float32))
    lf = O.widen(dt, logits)
    for b in range(B):  # plant ties: the lowest index must win
        m = lf[b].max()
        idx = rng.choice(50257, size=3, replace=False)
        logits[b, idx] = O.round_to(dt, np.full(3, m + 1, np.float32))
    toks = torch.empty(B, dtype=torch.int32, device="cuda")
    b2.argmax(toks, to_dev(dt, logits))
    torch.cuda.synchronize()
    assert toks.cpu().numpy().tolist() == O.argmax(dt, logits).tolist()
    # padded rows (the engine's 16-byte row stride): vector path, padding ignored
    padded = np.zeros((B, 50264), dtype=logits.dtype)
    padded[:, :50257] = logits
    padded[:, 50257:] = O.round_to(dt, np.full((B, 7), 1e4, np.float32))  # larger than any logit
    toks2 = torch.empty(B, dtype=torch.int32, device="cuda")
    b2.argmax(toks2, to_dev(dt, padded.ravel()).view(B, 50264), vocab=50257)
    torch.cuda.synchronize()
    assert toks2.cpu().numpy().tolist() == O.argmax(dt, logits).tolist()


def test_add_one(b2, cuda):
    torch = _torch()
    a = ints_dev(np.arange(-3, 700))
    out = torch.empty_like(a)
    b2.add_one(out, a)
    torch.cuda.synchronize()
    assert out.cpu().numpy().tolist() == list(range(-2, 701))


def test_reference_kernel_kats(b2, cuda, golden):
    """gpu-engine/tests/test_kernels.cpp:50-228 on the sm_100a kernels (fp16, like the reference)."""
    torch = _torch()
    k = golden("kernel_kat.json")
    dt = O.F16
    e = k["embedding"]
    wte = O.round_to(dt, np.array(e["wte"], np.float32).reshape(-1, e["d"]))
    wpe = O.round_to(dt, np.array(e["wpe"], np.float32).reshape(-1, e["d"]))
    out = torch.empty(e["batch"], e["d"], dtype=torch.float16, device="cuda")
    b2.embedding(out, to_dev(dt, wte), to_dev(dt, wpe), ints_dev(e["token_ids"]), ints_dev(e["positions"]))
    torch.cuda.synchronize()
    assert np.max(np.abs(out.float().cpu().numpy().ravel() - np.array(e["expected"]))) < 5e-2

    ln = k["add_layernorm"]
    b, d = ln["batch"], ln["d"]
    x = to_dev(dt, O.round_to(dt, np.array(ln["x"], np.float32).reshape(b, d)))
    r = to_dev(dt, O.round_to(dt, np.array(ln["residual"], np.float32).reshape(b, d)))
    out = torch.empty_like(x)
    b2.add_layernorm(out, r, x, r, to_dev(dt, O.round_to(dt, np.array(ln["gamma"], np.float32))),
                     to_dev(dt, O.round_to(dt, np.array(ln["beta"], np.float32))), ln["eps"])
    torch.cuda.synchronize()
    assert np.max(np.abs(out.float().cpu().numpy().ravel() - np.array(ln["expected"]))) < 5e-2

    g = k["bias_gelu"]
    x = to_dev(dt, O.round_to(dt, np.array(g["x"], np.float32).reshape(g["batch"], g["d"])))
    out = torch.empty_like(x)
    b2.bias_gelu(out, x, to_dev(dt, O.round_to(dt, np.array(g["bias"], np.float32))))
    torch.cuda.synchronize()
    assert np.max(np.abs(out.float().cpu().numpy().ravel() - np.array(g["expected"]))) < 5e-2

    a = k["argmax"]
    logits = to_dev(dt, O.round_to(dt, np.array(a["logits"], np.float32).reshape(a["batch"], a["vocab"])))
    toks = torch.empty(a["batch"], dtype=torch.int32, device="cuda")
    b2.argmax(toks, logits)
    torch.cuda.synchronize()
    assert toks.cpu().numpy().tolist() == a["expected"]


@pytest.mark.parametrize("H", [12, 16])  # 16 heads x 64: the 8-row-stage plan (GPT-2 medium's)
@pytest.mark.parametrize("dt", [O.F16, O.BF16])
def test_attention_early_start_after_kv_append(b2, cuda, dt, H):
    """kv_append writes each sequence's newest row, then attention runs right
    behind it with B2_ATTN_NEWEST_ROW_PENDING (it may start before kv_append
    finishes and must still read the new rows); and with B2_ATTN_INPUTS_READY
    on inputs written long before.  Both against the oracle over the appended
    pool, several rounds."""
    torch = _torch()
    rng = np.random.Generator(np.random.PCG64(77 + H))
    Dh, L, layer = 64, 2, 1
    ctx_pre = rng.integers(0, 700, size=48).astype(np.int32)
    pool, bt, mbps, nb = make_paged(rng, dt, (ctx_pre + 1).tolist(), H, Dh, L)
    B = len(ctx_pre)
    stride = 3 * H * Dh
    qkv = O.round_to(dt, rng.standard_normal(B * stride, dtype=np.float32)).reshape(B, stride)
    ref_pool = pool.copy()
    kpad = np.zeros_like(qkv)
    vpad = np.zeros_like(qkv)
    kpad[:, : 2 * H * Dh] = qkv[:, H * Dh:]
    vpad[:, : H * Dh] = qkv[:, 2 * H * Dh:]
    O.kv_append(dt, ref_pool, kpad, vpad, stride, bt, ctx_pre, n_kv_head=H, head_dim=Dh, max_blocks_per_seq=mbps,
                layer_idx=layer, n_layer=L, num_blocks=nb)
    post = (ctx_pre + 1).tolist()
    ref = O.paged_attention(dt, qkv.ravel(), stride, ref_pool, np.where(bt < 0, 0, bt), post, n_head=H, n_kv_head=H,
                            head_dim=Dh, max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, nthreads=8)
    qkvd = to_dev(dt, qkv.ravel()).view(B, stride)
    btd, pre_d = ints_dev(bt), ints_dev(ctx_pre)
    post_d = torch.zeros(B, dtype=torch.int32, device="cuda")
    out = torch.empty(B, H, Dh, dtype=torch.float32, device="cuda")
    for flags in (b2.ATTN_NEWEST_ROW_PENDING, b2.ATTN_INPUTS_READY):
        pd = to_dev(dt, pool)  # fresh pool without the new rows
        args = b2.attn_args(qkvd, stride, pd, btd, post_d, out, n_head=H, n_kv_head=H, head_dim=Dh,
                            max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, num_blocks=nb, flags=flags)
        ws = b2.attention_workspace(args)
        for _ in range(3):
            out.fill_(float("nan"))
            b2.kv_append(pd, qkvd[:, H * Dh:], qkvd[:, 2 * H * Dh:], stride, btd, pre_d, n_kv_head=H, head_dim=Dh,
                         max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, num_blocks=nb, seq_lens_post=post_d)
            if flags == b2.ATTN_INPUTS_READY:
                torch.cuda.synchronize()  # READY promises nothing is written by the kernel just before
            b2.paged_attention(args, ws)
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            assert np.isfinite(got).all()
            assert np.max(np.abs(got - ref)) <= 2e-3
    assert b2.device_errors() == 0
