"""b2_lm_head_argmax (tied lm_head GEMM + greedy argmax in one tensor-core
kernel) against the oracle: the reference CPU path's logits
(cpu_model.cpp:182-196, fp32 dot products, oracle.linear) of the 16-bit x and
w, rounded to the dtype as the unfused engine stores them
(engine.cu:202-203), then the first maximum (oracle.argmax, logits.cu:18-57 /
cpu_model.cpp:190).

The kernel sums each dot product in a different order (tensor-core K
blocks), so its fp32 logit differs from the oracle's by at most
eps = K * 2^-21 * sum|x||w| (a generous bound).  Where the oracle's winner
leads every other logit by more than two ulps of the dtype at its magnitude
plus 2 eps, no rounding can reorder them and the tokens must be identical;
elsewhere (near-ties) the kernel's token must be within that margin of the
best logit.  Planted exact ties must go to the lowest index, NaN logits must
never win, and rows of w past the vocabulary must never count."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _ulp(dt, v):
    mant = 7 if dt == O.BF16 else 10
    e = np.floor(np.log2(np.maximum(np.abs(v), 2.0 ** -14)))
    return 2.0 ** (e - mant)


def _run(b2, torch, dt, x16, w16, vocab, workspace=None):
    tdt = torch.bfloat16 if dt == O.BF16 else torch.float16
    dev = torch.device("cuda:0")
    xd = torch.from_numpy(x16.view(np.int16)).to(dev).view(tdt)
    wd = torch.from_numpy(w16.view(np.int16)).to(dev).view(tdt)
    tok = torch.full((x16.shape[0],), -7, dtype=torch.int32, device=dev)
    ws = workspace if workspace is not None else b2.lm_head_argmax_workspace(x16.shape[0], dev)
    b2.lm_head_argmax(tok, xd, wd, vocab=vocab, workspace=ws)
    torch.cuda.synchronize()
    return tok.cpu().numpy(), ws


def _check(dt, x16, w16, vocab, got):
    xf, wf = O.widen(dt, x16), O.widen(dt, w16[:vocab])
    lf = O.linear(xf, wf, None)                      # fp32 logits, the reference CPU path's dot
    want = O.argmax(dt, O.round_to(dt, lf))         # rounded as stored, first maximum
    l64 = xf.astype(np.float64) @ wf.astype(np.float64).T
    eps = xf.shape[1] * 2.0 ** -21 * (np.abs(xf).astype(np.float64) @ np.abs(wf).astype(np.float64).T)
    robust = 0
    for b in range(x16.shape[0]):
        row = np.where(np.isnan(l64[b]), -np.inf, l64[b])
        top = int(want[b])
        margin = 2 * _ulp(dt, row[top]) + 2 * np.nanmax(eps[b])
        others = np.delete(row, top)
        if row[top] - others.max() > margin:
            robust += 1
            assert got[b] == top, f"row {b}: token {got[b]} vs oracle {top} (lead {row[top] - others.max():.3g})"
        else:
            assert 0 <= got[b] < vocab and row[got[b]] >= row.max() - margin, f"row {b}: token {got[b]} not near-best"
    return robust


CASES = [
    # id, dtype, batch, d_model, vocab, w_rows
    ("bf16-one-row", O.BF16, 1, 64, 128, 128),
    ("f16-ragged-vocab", O.F16, 7, 768, 1000, 1000),
    ("bf16-xl-width-padded-rows", O.BF16, 130, 1600, 5003, 5008),
    ("f16-two-batch-chunks", O.F16, 300, 1024, 2048, 2048),
    ("bf16-gpt2-vocab", O.BF16, 48, 1600, 50257, 50264),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_lm_head_argmax_matches_oracle(b2, cuda, case):
    import torch
    name, dt, batch, d, vocab, w_rows = case
    rng = np.random.Generator(np.random.PCG64(71 + batch))
    # final LayerNorm output, ~N(0, 1), shifted so that a constant row's logit is large and positive
    x = rng.standard_normal((batch, d), dtype=np.float32) + 0.5
    w = rng.normal(0.0, 0.02, size=(w_rows, d)).astype(np.float32)
    w[vocab:] = 5.0  # rows past the vocabulary would win every row if they counted
    x16, w16 = O.round_to(dt, x), O.round_to(dt, w)
    got, ws = _run(b2, torch, dt, x16, w16, vocab)
    robust = _check(dt, x16, w16, vocab, got)
    assert robust >= batch // 2, f"only {robust} of {batch} rows were decisive: the case does not test much"
    assert int(ws.count_nonzero()) == 0, "the launch must leave its workspace zeroed"


def test_lm_head_argmax_ties_nan_and_back_to_back(b2, cuda):
    import torch
    dt, batch, d, vocab = O.BF16, 4, 256, 700
    rng = np.random.Generator(np.random.PCG64(5))
    x = rng.standard_normal((batch, d), dtype=np.float32)
    w = rng.normal(0.0, 0.02, size=(vocab, d)).astype(np.float32)
    # row 0: rows 150 (tile 1) and 600 (tile 4) identical and far ahead -> 150
    w[150] = w[600] = 0.25 * np.sign(x[0])
    # row 1: a NaN row with the largest magnitude never wins; row 420 does
    w[9] = 0.3 * np.sign(x[1])
    w[9, 5] = np.nan
    w[420] = 0.2 * np.sign(x[1])
    # row 2: three equal winners in one tile -> the lowest
    w[260] = w[300] = w[261] = 0.3 * np.sign(x[2])
    x16, w16 = O.round_to(dt, x), O.round_to(dt, w)
    got, ws = _run(b2, torch, dt, x16, w16, vocab)
    assert got[0] == 150 and got[1] == 420 and got[2] == 260, got
    # launch twice back to back on one workspace with other inputs, no sync between
    tdt = torch.bfloat16
    dev = torch.device("cuda:0")
    x2 = O.round_to(dt, rng.standard_normal((batch, d), dtype=np.float32))
    wd = torch.from_numpy(w16.view(np.int16)).to(dev).view(tdt)
    xa = torch.from_numpy(x16.view(np.int16)).to(dev).view(tdt)
    xb = torch.from_numpy(x2.view(np.int16)).to(dev).view(tdt)
    ta = torch.zeros(batch, dtype=torch.int32, device=dev)
    tb = torch.zeros(batch, dtype=torch.int32, device=dev)
    b2.lm_head_argmax(ta, xa, wd, vocab=vocab, workspace=ws)
    b2.lm_head_argmax(tb, xb, wd, vocab=vocab, workspace=ws)
    torch.cuda.synchronize()
    assert np.array_equal(ta.cpu().numpy(), got)
    _check(dt, x2, w16, vocab, tb.cpu().numpy())
    assert int(ws.count_nonzero()) == 0
    assert b2.device_errors() == 0


def test_lm_head_argmax_matches_unfused_gpu_path(b2, cuda):
    """Against the engine's unfused path on the same GPU (cuBLAS GEMM into
    dtype logits, then b2_argmax_rows): identical wherever the unfused
    logits' top two are more than two ulps apart."""
    import torch
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(3)
    for tdt in (torch.float16, torch.bfloat16):
        x = torch.randn(96, 1024, generator=g, device=dev).to(tdt)
        w = (torch.randn(8000, 1024, generator=g, device=dev) * 0.02).to(tdt)
        logits = x @ w.T
        ref = torch.empty(96, dtype=torch.int32, device=dev)
        b2.argmax(ref, logits)
        tok = torch.empty(96, dtype=torch.int32, device=dev)
        b2.lm_head_argmax(tok, x, w)
        top2 = logits.float().topk(2, dim=1).values
        mant = 7 if tdt == torch.bfloat16 else 10
        ulp = torch.exp2(torch.floor(torch.log2(top2[:, 0].abs().clamp_min(2.0 ** -14))) - mant)
        decisive = (top2[:, 0] - top2[:, 1] > 2 * ulp).cpu()  # two ulps: rounding cannot swap them
        assert int(decisive.sum()) >= 48
        assert torch.equal(tok.cpu()[decisive], ref.cpu()[decisive])
