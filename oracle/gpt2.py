"""Greedy GPT-2 decode composed from the oracle's primitives over a PAGED KV
cache, token by token -- the CPU restatement of the reference's decode path.

TEST INFRASTRUCTURE ONLY.  It follows CPUModel::forward_step
(gpu-engine/src/reference/cpu_model.cpp:92-180) operation for operation, but
feeds the prompt one token at a time through the paged layout the GPU
engine uses (blocks of 16 positions, all layers per block, kv_cache.h:6-8),
with keys addressed through a block table.  Per-row arithmetic is the same
as the reference's T-token prompt pass, so the two must agree bit for bit;
tests/test_oracle_pin.py checks the tokens against the reference itself.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O


def greedy_generate(cfg: dict, tensors: dict, prompt: list[int], n_new: int, block_order_seed: int = 0,
                    nthreads: int = 8) -> list[int]:
    D, H, L = cfg["d_model"], cfg["n_head"], cfg["n_layer"]
    Dh = cfg["head_dim"]
    eps = float(cfg["layer_norm_epsilon"])
    eos = int(cfg["eos_token_id"])
    total = len(prompt) + n_new
    nblk = (total + 15) // 16
    # Blocks come from a shuffled pool so the block table is not the identity.
    rng = np.random.default_rng(block_order_seed)
    num_blocks = nblk + 3
    table = rng.permutation(num_blocks)[:nblk].astype(np.int32)
    pool = np.zeros(num_blocks * L * 2 * 16 * H * Dh, dtype=np.float32)
    wte, wpe = tensors["wte"], tensors["wpe"]
    zero_ff = np.zeros(4 * D, dtype=np.float32)

    def step(tok: int, pos: int) -> int:
        hidden = O.embedding(O.F32, wte, wpe, [tok], [pos])  # [1, D]
        for l in range(L):
            p = f"layer{l}."
            x, _, _ = O.add_layernorm(O.F32, None, hidden, tensors[p + "ln1_g"], tensors[p + "ln1_b"], eps)
            qkv = O.linear(x, tensors[p + "qkv_w"], tensors[p + "qkv_b"], nthreads)
            O.kv_append(O.F32, pool, qkv[:, D:2 * D].copy(), qkv[:, 2 * D:].copy(), D, table[None, :],
                        np.array([pos], np.int32), n_kv_head=H, head_dim=Dh, max_blocks_per_seq=nblk,
                        layer_idx=l, n_layer=L, num_blocks=num_blocks)
            attn = O.paged_attention(O.F32, qkv, 3 * D, pool, table[None, :], np.array([pos + 1], np.int32),
                                     n_head=H, n_kv_head=H, head_dim=Dh, max_blocks_per_seq=nblk, layer_idx=l,
                                     n_layer=L)
            attn_out = O.linear(attn.reshape(1, D), tensors[p + "proj_w"], tensors[p + "proj_b"], nthreads)
            hidden = (hidden + attn_out).astype(np.float32)
            x, _, _ = O.add_layernorm(O.F32, None, hidden, tensors[p + "ln2_g"], tensors[p + "ln2_b"], eps)
            ff = O.linear(x, tensors[p + "fc_w"], tensors[p + "fc_b"], nthreads)
            ff = O.bias_gelu(O.F32, ff, zero_ff)  # x + 0 is exact: gelu of the biased GEMM output
            ff_out = O.linear(ff, tensors[p + "fc_proj_w"], tensors[p + "fc_proj_b"], nthreads)
            hidden = (hidden + ff_out).astype(np.float32)
        normed, _, _ = O.add_layernorm(O.F32, None, hidden, tensors["lnf_g"], tensors["lnf_b"], eps)
        return O.tied_lm_head_argmax(wte, normed[0])

    out: list[int] = []
    nxt = 0
    for pos, tok in enumerate(prompt):
        nxt = step(tok, pos)
    out.append(nxt)
    if nxt == eos:
        return out
    pos = len(prompt)
    while len(out) < n_new:
        nxt = step(nxt, pos)
        pos += 1
        out.append(nxt)
        if nxt == eos:
            break
    return out
