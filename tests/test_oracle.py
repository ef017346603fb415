"""The CPU oracle against the reference's own known answers (CPU only).

Pins: gpu-engine/tests/test_kernels.cpp:50-228 (kernel KATs, via
tests/golden/kernel_kat.json), gpu-engine/tests/test_kv_cache.cpp:80-83
(block_bytes), and straightforward float64 restatements for attention.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O


def test_half_and_bf16_conversions_are_exact(oracle, rng):
    x = np.concatenate([rng.standard_normal(4096).astype(np.float32) * 3,
                        np.array([0.0, -0.0, 65504.0, 1e-7, -6.1e-5, 5.96e-8, 1e5], np.float32)])
    h = O.round_to(O.F16, x)
    assert np.array_equal(h, x.astype(np.float16).view(np.uint16))
    assert np.array_equal(O.widen(O.F16, h), x.astype(np.float16).astype(np.float32))
    b = O.round_to(O.BF16, x)
    # round-to-nearest-even on the top 16 bits
    u = x.view(np.uint32).astype(np.uint64)
    ref = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    assert np.array_equal(b, ref)
    assert np.array_equal(O.widen(O.BF16, b), (b.astype(np.uint32) << 16).view(np.float32))


def test_block_bytes_matches_reference_kat(oracle):
    # gpu-engine/tests/test_kv_cache.cpp:80-83
    assert O.block_bytes(12, 12, 64, 2) == 589824
    if O.ref_available():
        assert O.load_ref().ref_block_bytes(12, 12, 64) == 589824
        assert O.load_ref().ref_block_tokens() == 16


def test_embedding_kat(oracle, golden):
    k = golden("kernel_kat.json")["embedding"]
    d = k["d"]
    wte = np.array(k["wte"], np.float32).reshape(-1, d)
    wpe = np.array(k["wpe"], np.float32).reshape(-1, d)
    out = O.embedding(O.F32, wte, wpe, k["token_ids"], k["positions"])
    assert np.array_equal(out.ravel(), np.array(k["expected"], np.float32))


def test_add_layernorm_kat(oracle, golden):
    k = golden("kernel_kat.json")["add_layernorm"]
    b, d = k["batch"], k["d"]
    x = np.array(k["x"], np.float32).reshape(b, d)
    r = np.array(k["residual"], np.float32).reshape(b, d)
    out, _, res = O.add_layernorm(O.F32, x, r, np.array(k["gamma"], np.float32), np.array(k["beta"], np.float32),
                                  k["eps"])
    assert np.array_equal(res, (x + r).astype(np.float32))
    # the reference test forms inv_std in float, the oracle (cpu_model.cpp) in double
    assert np.max(np.abs(out.ravel() - np.array(k["expected"], np.float32))) < 1e-5


def test_bias_gelu_kat(oracle, golden):
    k = golden("kernel_kat.json")["bias_gelu"]
    x = np.array(k["x"], np.float32).reshape(k["batch"], k["d"])
    out = O.bias_gelu(O.F32, x, np.array(k["bias"], np.float32))
    assert np.max(np.abs(out.ravel() - np.array(k["expected"], np.float32))) < 1e-6


def test_argmax_kat_and_lowest_index_ties(oracle, golden):
    k = golden("kernel_kat.json")["argmax"]
    logits = np.array(k["logits"], np.float32).reshape(k["batch"], k["vocab"])
    assert O.argmax(O.F32, logits).tolist() == k["expected"]
    tie = np.zeros((1, 50), np.float32)
    tie[0, [7, 3, 40]] = 2.0
    assert O.argmax(O.F32, tie).tolist() == [3]


def _random_paged(rng, dt, B, H, Hkv, Dh, L, ctx, extra_blocks=5):
    mbps = max(1, max((c + 15) // 16 for c in ctx))
    nblocks_needed = sum((c + 15) // 16 for c in ctx)
    num_blocks = nblocks_needed + extra_blocks
    perm = rng.permutation(num_blocks).astype(np.int32)
    bt = np.zeros((B, mbps), np.int32)
    o = 0
    for b, c in enumerate(ctx):
        n = (c + 15) // 16
        bt[b, :n] = perm[o:o + n]
        o += n
    pool = O.round_to(dt, rng.standard_normal(num_blocks * L * 2 * 16 * Hkv * Dh).astype(np.float32))
    return pool, bt, mbps, num_blocks


@pytest.mark.parametrize("dt", [O.F32, O.F16, O.BF16])
@pytest.mark.parametrize("H,Hkv", [(4, 4), (8, 2)])
def test_paged_attention_oracle_matches_float64_softmax(oracle, rng, dt, H, Hkv):
    B, Dh, L, layer = 3, 64, 2, 1
    ctx = [1, 17, 40]
    pool, bt, mbps, nb = _random_paged(rng, dt, B, H, Hkv, Dh, L, ctx)
    stride = H * Dh + 32
    q = O.round_to(dt, rng.standard_normal(B * stride).astype(np.float32))
    out = O.paged_attention(dt, q, stride, pool, bt, ctx, n_head=H, n_kv_head=Hkv, head_dim=Dh,
                            max_blocks_per_seq=mbps, layer_idx=layer, n_layer=L, nthreads=2)
    poolf = O.widen(dt, pool).reshape(nb, L, 2, 16, Hkv, Dh).astype(np.float64)
    qf = O.widen(dt, q).reshape(B, stride)[:, :H * Dh].reshape(B, H, Dh).astype(np.float64)
    for b in range(B):
        rows = [poolf[bt[b, j // 16], layer, :, j % 16] for j in range(ctx[b])]
        K = np.stack([r[0] for r in rows])  # [C, Hkv, Dh]
        V = np.stack([r[1] for r in rows])
        for h in range(H):
            hk = h // (H // Hkv)
            s = K[:, hk] @ qf[b, h] / np.sqrt(Dh)
            w = np.exp(s - s.max())
            w /= w.sum()
            assert np.max(np.abs(w @ V[:, hk] - out[b, h])) < 2e-5


def test_paged_attention_oracle_empty_sequence_is_zero(oracle, rng):
    pool, bt, mbps, nb = _random_paged(rng, O.F16, 2, 2, 2, 64, 1, [0, 5])
    q = O.round_to(O.F16, rng.standard_normal(2 * 128).astype(np.float32))
    out = O.paged_attention(O.F16, q, 128, pool, bt, [0, 5], n_head=2, n_kv_head=2, head_dim=64,
                            max_blocks_per_seq=mbps, layer_idx=0, n_layer=1)
    assert np.all(out[0] == 0) and np.any(out[1] != 0)


def test_kv_append_oracle_places_rows(oracle, rng):
    dt, B, Hkv, Dh, L, layer = O.F16, 3, 2, 64, 3, 2
    pos = np.array([0, 15, 33], np.int32)
    pool, bt, mbps, nb = _random_paged(rng, dt, B, Hkv, Hkv, Dh, L, [int(p) + 1 for p in pos])
    before = pool.copy()
    stride = 3 * Hkv * Dh
    qkv = O.round_to(dt, rng.standard_normal(B * stride).astype(np.float32)).reshape(B, stride)
    k = np.ascontiguousarray(qkv[:, Hkv * Dh:])
    v = np.ascontiguousarray(qkv[:, 2 * Hkv * Dh:])
    # k / v are views into the fused row: pass the fused buffer offsets via copies with the same stride
    kbuf = np.zeros((B, stride), np.uint16)
    vbuf = np.zeros((B, stride), np.uint16)
    kbuf[:, : 2 * Hkv * Dh] = k
    vbuf[:, : Hkv * Dh] = v
    O.kv_append(dt, pool, kbuf, vbuf, stride, bt, pos, n_kv_head=Hkv, head_dim=Dh, max_blocks_per_seq=mbps,
                layer_idx=layer, n_layer=L, num_blocks=nb)
    P = pool.reshape(nb, L, 2, 16, Hkv, Dh)
    Pb = before.reshape(nb, L, 2, 16, Hkv, Dh)
    changed = np.argwhere(np.any(P != Pb, axis=-1))
    assert len(changed) <= B * 2 * Hkv
    for b in range(B):
        blk, t = bt[b, pos[b] // 16], pos[b] % 16
        assert np.array_equal(P[blk, layer, 0, t].ravel(), kbuf[b, : Hkv * Dh])
        assert np.array_equal(P[blk, layer, 1, t].ravel(), vbuf[b, : Hkv * Dh])


def test_kv_append_oracle_rejects_bad_block(oracle, rng):
    pool, bt, mbps, nb = _random_paged(rng, O.F16, 1, 1, 1, 64, 1, [3])
    bt[0, 0] = nb + 7
    k = np.zeros((1, 64), np.uint16)
    with pytest.raises(ValueError):
        O.kv_append(O.F16, pool, k, k, 64, bt, [2], n_kv_head=1, head_dim=64, max_blocks_per_seq=mbps,
                    layer_idx=0, n_layer=1, num_blocks=nb)
