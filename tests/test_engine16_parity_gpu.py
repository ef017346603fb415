"""The 16-bit engine against the oracle, teacher-forced (GPU).

The f16 / bf16 engines behind every GPT-2 decode tokens/s number run the
reference's forward step (CPUModel::forward_step, cpu_model.cpp:92-180) with
16-bit weights, activations and KV cache.  Here each is fed fixed random token
streams as prompts (decode_step consumes a prompt one position per step, so
the stream is teacher-forced) and, after every step, its final LayerNorm rows
and logits (b2_engine_last_step_outputs) are compared with the oracle's
forward step in fp32 on the same weights rounded to the engine's dtype
(oracle/gpt2.py teacher_forced).  The difference is the engine's 16-bit
activation rounding, so the bar is a stated tolerance, not bit equality:

  * final LayerNorm output: max-abs <= HIDDEN_TOL[dtype] (the rows are ~N(0,1));
  * logits: max-abs <= LOGIT_TOL[dtype];
  * greedy choice: the engine's argmax equals the oracle's at every position
    where the oracle's top-2 margin exceeds 2 * LOGIT_TOL (elsewhere a flip is
    within the tolerance).

Models: small synthetic GPT-2s with the medium head shape (16 x 64) and the
XL head shape (25 x 64), two layers, weights N(0, 0.02); four streams of 40
tokens decoded together (batch 4); the decode GEMMs on cublasGemmEx, on
cuBLASLt with timed algorithm choice and the FC bias + GELU in its epilogue
(b2_engine_set_gemm_mode 3), and on b2_linear.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import gpt2, oracle as O

pytestmark = pytest.mark.gpu

HIDDEN_TOL = {O.F16: 0.02, O.BF16: 0.1}
LOGIT_TOL = {O.F16: 0.01, O.BF16: 0.05}
SHAPES = {"medium-heads": dict(n_layer=2, n_head=16, d_model=1024, vocab_size=2048, n_ctx=256),
          "xl-heads": dict(n_layer=2, n_head=25, d_model=1600, vocab_size=2048, n_ctx=256)}
T, STREAMS = 40, 4


def _rounded(dt, tensors):
    return {k: O.widen(dt, O.round_to(dt, v)) for k, v in tensors.items()}


@pytest.fixture(scope="module")
def models(b2, tmp_path_factory):
    from lis_b200 import model_files as MF
    out = {}
    for name, shp in SHAPES.items():
        d = MF.write_model_dir(tmp_path_factory.mktemp(name), MF.GPT2Shape(**shp), seed=21, std=0.02)
        out[name] = (d, *MF.load_model_dir(d))
    return out


@pytest.mark.parametrize("gemm", ["cublas", "cublaslt", "b2_linear"])
@pytest.mark.parametrize("dt", [O.F16, O.BF16], ids=["f16", "bf16"])
@pytest.mark.parametrize("shape", list(SHAPES))
def test_16bit_engine_matches_oracle_teacher_forced(b2, cuda, models, shape, dt, gemm):
    from lis_b200 import engine as E
    d, cfg, tensors = models[shape]
    rng = np.random.Generator(np.random.PCG64(7 + len(shape)))
    streams = [rng.integers(0, cfg["vocab_size"], size=T).tolist() for _ in range(STREAMS)]
    eng = E.Engine()
    assert eng.init(str(d), E.Config(max_batch=STREAMS, max_seq_len=256, kv_block_budget=64, dtype=dt, device=0))
    if gemm == "b2_linear":
        eng.set_linear_tensor_cores(True)
    elif gemm == "cublaslt":
        eng.set_gemm_mode(3)
    ids = [eng.add_sequence(s) for s in streams]
    hid = np.empty((T, STREAMS, cfg["d_model"]), np.float32)
    lg = np.empty((T, STREAMS, cfg["vocab_size"]), np.float32)
    for t in range(T):
        eng.decode_step(ids)
        h, l = eng.last_step_outputs(STREAMS)
        hid[t], lg[t] = O.widen(dt, h), O.widen(dt, l)
    eng.close()
    ref_t = _rounded(dt, tensors)
    worst_h = worst_l = 0.0
    checked = agree = 0
    for i, s in enumerate(streams):
        rh, rl = gpt2.teacher_forced(cfg, ref_t, s, nthreads=8)
        worst_h = max(worst_h, float(np.abs(hid[:, i] - rh).max()))
        worst_l = max(worst_l, float(np.abs(lg[:, i] - rl).max()))
        top2 = np.sort(rl, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 2 * LOGIT_TOL[dt]
        checked += int(clear.sum())
        agree += int((np.argmax(lg[:, i], axis=1) == np.argmax(rl, axis=1))[clear].sum())
    print(f"{shape} dt={dt} gemm={gemm}: hidden max-abs {worst_h:.4g}, logits max-abs {worst_l:.4g}, "
          f"argmax agrees at {agree}/{checked} clear positions")
    assert worst_h <= HIDDEN_TOL[dt], f"final LayerNorm max-abs {worst_h:.4g} > {HIDDEN_TOL[dt]}"
    assert worst_l <= LOGIT_TOL[dt], f"logits max-abs {worst_l:.4g} > {LOGIT_TOL[dt]}"
    assert checked > 0 and agree == checked


@pytest.mark.parametrize("dt", [O.F16, O.BF16], ids=["f16", "bf16"])
@pytest.mark.parametrize("shape", list(SHAPES))
def test_fused_lm_head_engine_tokens_match_oracle(b2, cuda, models, shape, dt):
    """b2_engine_set_lm_head_fused: the tokens decode_step and prefill return
    (now from b2_lm_head_argmax, no logits formed) equal the oracle's greedy
    choice at every position where the oracle's top-2 margin exceeds
    2 * LOGIT_TOL, and the unfused engine's tokens wherever its own logits'
    top two are more than two ulps apart."""
    from lis_b200 import engine as E
    d, cfg, tensors = models[shape]
    rng = np.random.Generator(np.random.PCG64(11 + len(shape)))
    streams = [rng.integers(0, cfg["vocab_size"], size=T).tolist() for _ in range(STREAMS)]
    toks, logits = {}, None
    for fused in (False, True):
        eng = E.Engine()
        assert eng.init(str(d), E.Config(max_batch=STREAMS, max_seq_len=256, kv_block_budget=64, dtype=dt, device=0))
        eng.set_lm_head_fused(fused)
        ids = [eng.add_sequence(s) for s in streams]
        out = np.empty((T, STREAMS), np.int64)
        lg = np.empty((T, STREAMS, cfg["vocab_size"]), np.float32)
        for t in range(T):
            out[t] = eng.decode_step(ids)
            if not fused:
                lg[t] = O.widen(dt, eng.last_step_outputs(STREAMS)[1])
        toks[fused] = out
        if not fused:
            logits = lg
        # the same prompts through the batched prefill: each stream's first token
        eng2 = E.Engine()
        assert eng2.init(str(d), E.Config(max_batch=STREAMS, max_seq_len=256, kv_block_budget=64, dtype=dt, device=0))
        eng2.set_lm_head_fused(fused)
        toks[("prefill", fused)] = eng2.prefill([eng2.add_sequence(s) for s in streams])
        eng2.close()
        eng.close()
    ref_t = _rounded(dt, tensors)
    checked = 0
    mant = 7 if dt == O.BF16 else 10
    for i, s in enumerate(streams):
        _, rl = gpt2.teacher_forced(cfg, ref_t, s, nthreads=8)
        top2 = np.sort(rl, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 2 * LOGIT_TOL[dt]
        want = np.argmax(rl, axis=1)
        assert np.array_equal(toks[True][clear, i], want[clear]), f"stream {i}: fused tokens differ from the oracle"
        checked += int(clear.sum())
        if clear[-1]:
            assert toks[("prefill", True)][i] == want[-1], f"stream {i}: fused prefill token differs from the oracle"
        u2 = np.sort(logits[:, i], axis=1)[:, -2:]
        ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(u2[:, 1]), 2.0 ** -14))) - mant)
        apart = (u2[:, 1] - u2[:, 0]) > 2 * ulp
        assert np.array_equal(toks[True][apart, i], toks[False][apart, i]), f"stream {i}: fused vs unfused engine"
    assert checked > T
