"""Synthetic paged-decode workloads on the device, with their algorithmic byte counts.

The paged-attention microbench is batch 64, 12 heads, head_dim 64, fp16 K/V and q
drawn N(0,1) from a seed, per-sequence context U[128, 1024], block size 16,
block tables taken from a random permutation of a 65536-block pool (one layer
per block), scale 1/sqrt(64), fp32 softmax.  The pool is carved into disjoint
input SETS (each its own 64 sequences and block tables) so consecutive
launches touch different memory: with 16 sets, ~1.8 GB of KV rotates through a
126 MB L2, and every launch reads from HBM.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import BLOCK_TOKENS, F16, BF16, F32, attn_args, dtype_code


@dataclass
class AttnSet:
    seq_lens: np.ndarray           # host copy
    block_tables: np.ndarray       # host copy [B, mbps]
    d_seq_lens: object = None      # torch int32 [B]
    d_block_tables: object = None  # torch int32 [B, mbps]
    d_q: object = None
    d_out: object = None
    args: object = None
    bytes: int = 0                 # algorithmic bytes of one launch on this set


@dataclass
class AttnWorkload:
    batch: int
    n_head: int
    n_kv_head: int
    head_dim: int
    dtype: object
    pool_blocks: int
    mbps: int
    pool: object
    sets: list[AttnSet] = field(default_factory=list)
    workspace: object = None

    @property
    def elem(self) -> int:
        return 4 if dtype_code(self.dtype) == F32 else 2


def attention_bytes(seq_lens, n_head, n_kv_head, head_dim, s_kv, s_q, s_out) -> int:
    """Algorithmic bytes of one decode-attention launch:
    sum_b C_b*Hkv*Dh*2*s_kv (K and V rows read once) + B*H*Dh*(s_q + s_out)
    + sum_b ceil(C_b/16)*4 (block-table entries) + 4*B (seq_lens)."""
    c = np.asarray(seq_lens, dtype=np.int64)
    return int(c.sum() * n_kv_head * head_dim * 2 * s_kv + len(c) * n_head * head_dim * (s_q + s_out)
               + ((c + BLOCK_TOKENS - 1) // BLOCK_TOKENS).sum() * 4 + 4 * len(c))


def make_attention_workload(device, seed: int = 0, n_sets: int = 16, batch: int = 64, n_head: int = 12,
                            n_kv_head: int = 12, head_dim: int = 64, ctx_lo: int = 128, ctx_hi: int = 1024,
                            pool_blocks: int = 65536, dtype=None, log_uniform: bool = False,
                            out_dtype=None) -> AttnWorkload:
    import torch

    dtype = dtype or torch.float16
    out_dtype = out_dtype or dtype
    rng = np.random.Generator(np.random.PCG64(seed))
    mbps = (ctx_hi + BLOCK_TOKENS - 1) // BLOCK_TOKENS
    perm = rng.permutation(pool_blocks).astype(np.int32)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    row = n_kv_head * head_dim
    pool = torch.empty(pool_blocks * 2 * BLOCK_TOKENS * row, dtype=dtype, device=device)
    chunk = 1 << 28
    for o in range(0, pool.numel(), chunk):  # N(0,1) in pieces to bound temporaries
        n = min(chunk, pool.numel() - o)
        pool[o:o + n] = torch.randn(n, generator=gen, device=device, dtype=torch.float32).to(dtype)
    wl = AttnWorkload(batch, n_head, n_kv_head, head_dim, dtype, pool_blocks, mbps, pool)
    es = wl.elem
    used = 0
    for _ in range(n_sets):
        if log_uniform:
            ctx = np.exp(rng.uniform(np.log(ctx_lo), np.log(ctx_hi), size=batch)).astype(np.int64)
        else:
            ctx = rng.integers(ctx_lo, ctx_hi + 1, size=batch)
        nb = (ctx + BLOCK_TOKENS - 1) // BLOCK_TOKENS
        if used + int(nb.sum()) > pool_blocks:
            break
        bt = np.zeros((batch, mbps), np.int32)
        for b in range(batch):
            bt[b, : nb[b]] = perm[used: used + nb[b]]
            used += int(nb[b])
        s = AttnSet(ctx.astype(np.int32), bt)
        s.d_seq_lens = torch.from_numpy(s.seq_lens).to(device)
        s.d_block_tables = torch.from_numpy(bt).to(device)
        s.d_q = torch.randn(batch, n_head * head_dim, generator=gen, device=device, dtype=torch.float32).to(dtype)
        s.d_out = torch.empty(batch, n_head, head_dim, dtype=out_dtype, device=device)
        s.args = attn_args(s.d_q, n_head * head_dim, pool, s.d_block_tables, s.d_seq_lens, s.d_out, n_head=n_head,
                           n_kv_head=n_kv_head, head_dim=head_dim, max_blocks_per_seq=mbps, layer_idx=0, n_layer=1,
                           num_blocks=pool_blocks)
        s.bytes = attention_bytes(ctx, n_head, n_kv_head, head_dim, es, es, 4 if out_dtype == torch.float32 else es)
        wl.sets.append(s)
    return wl


def make_layered_workload(device, layout: str, seed: int = 0, batch: int = 128, n_head: int = 25, head_dim: int = 64,
                          ctx_lo: int = 256, ctx_hi: int = 1011, n_layer: int = 48, dtype=None) -> AttnWorkload:
    """One batch of sequences whose KV cache holds n_layer layers, one set per
    layer (launch l reads layer l), in one of two layouts:
      "blocks"      -- the reference's pool (kv_cache.h:6-8): one block holds
                       all layers, [block][layer][K|V][16][H][Dh]; launch l
                       passes layer_idx = l, n_layer = n_layer;
      "layer-major" -- the engine's: one [blocks][K|V][16][H][Dh] arena per
                       layer; launch l addresses layer l's arena (its block ids
                       offset by l * blocks), n_layer = 1.
    Same block permutation, same bytes per launch: the two differ only in where
    one layer's slabs sit (a block apart, or packed)."""
    import torch

    dtype = dtype or torch.bfloat16
    rng = np.random.Generator(np.random.PCG64(seed))
    ctx = rng.integers(ctx_lo, ctx_hi + 1, size=batch)
    nb = (ctx + BLOCK_TOKENS - 1) // BLOCK_TOKENS
    nblk = int(nb.sum())
    mbps = (ctx_hi + BLOCK_TOKENS - 1) // BLOCK_TOKENS
    perm = rng.permutation(nblk).astype(np.int32)
    bt = np.zeros((batch, mbps), np.int32)
    o = 0
    for b in range(batch):
        bt[b, : nb[b]] = perm[o:o + nb[b]]
        o += int(nb[b])
    row = n_head * head_dim
    pool_blocks = nblk if layout == "blocks" else nblk * n_layer
    n_el = pool_blocks * (n_layer if layout == "blocks" else 1) * 2 * BLOCK_TOKENS * row
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    pool = torch.empty(n_el, dtype=dtype, device=device)
    chunk = 1 << 28
    for i in range(0, n_el, chunk):
        n = min(chunk, n_el - i)
        pool[i:i + n] = torch.randn(n, generator=gen, device=device, dtype=torch.float32).to(dtype)
    wl = AttnWorkload(batch, n_head, n_head, head_dim, dtype, pool_blocks, mbps, pool)
    es = wl.elem
    d_sl = torch.from_numpy(ctx.astype(np.int32)).to(device)
    q = torch.randn(batch, row, generator=gen, device=device, dtype=torch.float32).to(dtype)
    out = torch.empty(batch, n_head, head_dim, dtype=dtype, device=device)
    for l in range(n_layer):
        tab = bt if layout == "blocks" else bt + l * nblk
        s = AttnSet(ctx.astype(np.int32), tab)
        s.d_seq_lens = d_sl
        s.d_block_tables = torch.from_numpy(np.ascontiguousarray(tab)).to(device)
        s.d_q, s.d_out = q, out
        s.args = attn_args(q, row, pool, s.d_block_tables, d_sl, out, n_head=n_head, n_kv_head=n_head,
                           head_dim=head_dim, max_blocks_per_seq=mbps, layer_idx=l if layout == "blocks" else 0,
                           n_layer=n_layer if layout == "blocks" else 1, num_blocks=pool_blocks)
        s.bytes = attention_bytes(ctx, n_head, n_head, head_dim, es, es, es)
        wl.sets.append(s)
    return wl


def host_subset(wl: AttnWorkload, set_index: int, n_seq: int | None = None):
    """Copies one set's blocks to host as a compact pool (for the CPU leg).
    Returns (pool uint16/float32 array, block tables remapped, seq_lens, q)."""
    import torch

    s = wl.sets[set_index]
    n_seq = n_seq or wl.batch
    ctx = s.seq_lens[:n_seq]
    bt = s.block_tables[:n_seq]
    ids = np.concatenate([bt[b, : (ctx[b] + 15) // 16] for b in range(n_seq)])
    remap = {int(v): i for i, v in enumerate(ids)}
    bt2 = np.zeros_like(bt)
    for b in range(n_seq):
        for j in range((ctx[b] + 15) // 16):
            bt2[b, j] = remap[int(bt[b, j])]
    blk_elems = 2 * BLOCK_TOKENS * wl.n_kv_head * wl.head_dim
    pv = wl.pool.view(wl.pool_blocks, blk_elems)
    sub = pv[torch.from_numpy(ids.astype(np.int64)).to(wl.pool.device)].contiguous().cpu()
    q = s.d_q[:n_seq].contiguous().cpu()
    if wl.elem == 2:
        sub = sub.view(torch.int16).numpy().view(np.uint16)
        q = q.view(torch.int16).numpy().view(np.uint16)
    else:
        sub, q = sub.numpy(), q.numpy()
    return sub.ravel(), bt2, ctx, q.ravel()
