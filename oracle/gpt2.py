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


class PagedDecoder:
    """One sequence's decode state over a paged KV cache: step(tok, pos) runs
    CPUModel::forward_step (cpu_model.cpp:92-180) for one position and returns
    the final LayerNorm's output row [D] (fp32)."""

    def __init__(self, cfg: dict, tensors: dict, total: int, block_order_seed: int = 0, nthreads: int = 8):
        self.cfg, self.t, self.nthreads = cfg, tensors, nthreads
        D, H, L = cfg["d_model"], cfg["n_head"], cfg["n_layer"]
        Dh = cfg["head_dim"]
        self.nblk = (total + 15) // 16
        # Blocks come from a shuffled pool so the block table is not the identity.
        rng = np.random.default_rng(block_order_seed)
        self.num_blocks = self.nblk + 3
        self.table = rng.permutation(self.num_blocks)[: self.nblk].astype(np.int32)
        self.pool = np.zeros(self.num_blocks * L * 2 * 16 * H * Dh, dtype=np.float32)
        self.zero_ff = np.zeros(4 * D, dtype=np.float32)

    def step(self, tok: int, pos: int) -> np.ndarray:
        cfg, tensors, nthreads = self.cfg, self.t, self.nthreads
        D, H, L = cfg["d_model"], cfg["n_head"], cfg["n_layer"]
        Dh = cfg["head_dim"]
        eps = float(cfg["layer_norm_epsilon"])
        table, nblk, pool = self.table, self.nblk, self.pool
        hidden = O.embedding(O.F32, tensors["wte"], tensors["wpe"], [tok], [pos])  # [1, D]
        for l in range(L):
            p = f"layer{l}."
            x, _, _ = O.add_layernorm(O.F32, None, hidden, tensors[p + "ln1_g"], tensors[p + "ln1_b"], eps)
            qkv = O.linear(x, tensors[p + "qkv_w"], tensors[p + "qkv_b"], nthreads)
            O.kv_append(O.F32, pool, qkv[:, D:2 * D].copy(), qkv[:, 2 * D:].copy(), D, table[None, :],
                        np.array([pos], np.int32), n_kv_head=H, head_dim=Dh, max_blocks_per_seq=nblk,
                        layer_idx=l, n_layer=L, num_blocks=self.num_blocks)
            attn = O.paged_attention(O.F32, qkv, 3 * D, pool, table[None, :], np.array([pos + 1], np.int32),
                                     n_head=H, n_kv_head=H, head_dim=Dh, max_blocks_per_seq=nblk, layer_idx=l,
                                     n_layer=L)
            attn_out = O.linear(attn.reshape(1, D), tensors[p + "proj_w"], tensors[p + "proj_b"], nthreads)
            hidden = (hidden + attn_out).astype(np.float32)
            x, _, _ = O.add_layernorm(O.F32, None, hidden, tensors[p + "ln2_g"], tensors[p + "ln2_b"], eps)
            ff = O.linear(x, tensors[p + "fc_w"], tensors[p + "fc_b"], nthreads)
            ff = O.bias_gelu(O.F32, ff, self.zero_ff)  # x + 0 is exact: gelu of the biased GEMM output
            ff_out = O.linear(ff, tensors[p + "fc_proj_w"], tensors[p + "fc_proj_b"], nthreads)
            hidden = (hidden + ff_out).astype(np.float32)
        normed, _, _ = O.add_layernorm(O.F32, None, hidden, tensors["lnf_g"], tensors["lnf_b"], eps)
        return normed[0]


def greedy_generate(cfg: dict, tensors: dict, prompt: list[int], n_new: int, block_order_seed: int = 0,
                    nthreads: int = 8) -> list[int]:
    eos = int(cfg["eos_token_id"])
    dec = PagedDecoder(cfg, tensors, len(prompt) + n_new, block_order_seed, nthreads)
    wte = tensors["wte"]

    def step(tok: int, pos: int) -> int:
        return O.tied_lm_head_argmax(wte, dec.step(tok, pos))

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


def teacher_forced(cfg: dict, tensors: dict, tokens: list[int], nthreads: int = 8) -> tuple[np.ndarray, np.ndarray]:
    """Feeds `tokens` one position at a time (the input at position p is
    tokens[p], whatever was predicted) and returns the final LayerNorm output
    [T, D] and the tied lm_head logits [T, vocab] (fp32, wte . h as the
    reference's argmax scans them, cpu_model.cpp:170-180)."""
    dec = PagedDecoder(cfg, tensors, len(tokens), 0, nthreads)
    hidden = np.stack([dec.step(int(t), p) for p, t in enumerate(tokens)]).astype(np.float32)
    logits = O.linear(hidden, tensors["wte"], None, nthreads)
    return hidden, logits
