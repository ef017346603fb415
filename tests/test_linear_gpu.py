"""b2_linear (tcgen05 weight-streaming linear layer) against a torch fp32
restatement of the reference's unfused sequence, through the C-ABI (GPU).

The reference runs gemm_rowmajor (cuBLAS, gpu-engine/src/engine.cu:124-131,
fp32 accumulation, output rounded to T) and then add_bias / bias_gelu
(kernels.h:35-49) on the rounded output.  The fp32 restatement here does the
same: y_ref = T(x.float() @ w.float().T), then + bias in fp32, GELU(tanh) in
fp32, rounded to T.  The kernel accumulates in fp32 in another order, so
its T(x.W^T) may land one rounding step away from the reference's, a step
the bias add and GELU (slope up to ~1.13) carry into the output; the output
rounding adds one more; and near zero the two fp32 sums may differ by their
accumulation error, a few units of 2^-24 * sum_k |x_k w_k|:
    |y - y_ref| <= 1.2 ulp_T(|x.W^T|) + ulp_T(max(|y|, |y_ref|))
                   + 2^-20 * (|x| . |w|^T) + 1e-6.
A wrong or missing K block would be off by ~ (|x| . |w|^T) / blocks, far
outside this.  Measured against a float64 product, the kernel's rounding
error is the same as cuBLAS's (both round a near-exact fp32 sum once).
"""
from __future__ import annotations

import math

import pytest

pytestmark = pytest.mark.gpu

# (batch, in_features, out_features): the engine's decode shapes (GPT-2 medium
# / XL at batch 1-512), ragged K and N, and a batch that needs two chunks.
SHAPES = [
    (1, 64, 128),
    (3, 1024, 3072),
    (128, 1024, 1024),
    (128, 4096, 1024),
    (128, 1600, 4800),
    (200, 1600, 6400),
    (17, 136, 200),
    (300, 256, 130),
    (512, 1600, 1600),
]


def _ref(torch, x, w, bias, epilogue, dtype):
    y = (x.float() @ w.float().T).to(dtype).float()
    if bias is not None:
        y = y + bias.float()
    if epilogue == 1:
        k = math.sqrt(2.0 / math.pi)
        y = 0.5 * y * (1.0 + torch.tanh(k * (y + 0.044715 * y * y * y)))
    return y.to(dtype)


def _ulp(torch, v, mant):
    """ulp of T at |v|: 2^(floor(log2|v|) - mant), floored at the subnormal step."""
    return torch.pow(2.0, torch.floor(torch.log2(v.abs().clamp_min(2.0 ** -14))) - mant)


def _check_close(torch, got, want, dtype, x, w):
    mant = 10 if dtype == torch.float16 else 7
    pre = x.float() @ w.float().T
    acc_slack = (x.float().abs() @ w.float().abs().T) * 2.0 ** -20
    g, r = got.float(), want.float()
    tol = 1.2 * _ulp(torch, pre, mant) + _ulp(torch, torch.maximum(g.abs(), r.abs()), mant) + acc_slack + 1e-6
    bad = (g - r).abs() > tol
    assert not bool(bad.any()), (
        f"{int(bad.sum())} of {bad.numel()} outputs outside the tolerance; "
        f"worst {(g - r).abs().max().item():.3e} at {torch.nonzero(bad)[0].tolist()}")


@pytest.mark.parametrize("dtype_name", ["f16", "bf16"])
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("epilogue,with_bias", [(0, False), (0, True), (1, True)])
def test_linear_matches_fp32_restatement(b2, cuda, dtype_name, shape, epilogue, with_bias):
    import torch
    dtype = torch.float16 if dtype_name == "f16" else torch.bfloat16
    batch, k, n = shape
    g = torch.Generator(device="cuda").manual_seed(batch * 7919 + k * 31 + n)
    x = torch.randn(batch, k, generator=g, device="cuda").to(dtype)
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).to(dtype)
    bias = (torch.randn(n, generator=g, device="cuda") * 0.02).to(dtype) if with_bias else None
    # output rows padded to a multiple of 8 elements (the TMA store's stride rule)
    y = torch.full((batch, (n + 7) // 8 * 8), float("nan"), device="cuda", dtype=dtype)[:, :n]
    b2.linear(y, x, w, bias, epilogue)
    torch.cuda.synchronize()
    assert b2.device_errors() == 0
    _check_close(torch, y, _ref(torch, x, w, bias, epilogue, dtype), dtype, x, w)


def test_linear_strided_rows_and_padding_untouched(b2, cuda):
    """x and y as column windows of wider buffers: the kernel reads only the
    window's columns and writes only [batch, out_features]."""
    import torch
    dtype = torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(5)
    xbuf = torch.randn(64, 3 * 1024, generator=g, device="cuda").to(dtype)
    x = xbuf[:, 1024:2048]
    w = (torch.randn(1000, 1024, generator=g, device="cuda") * 0.02).to(dtype)
    ybuf = torch.full((64, 1024 + 24), 7.0, device="cuda", dtype=dtype)
    y = ybuf[:, :1000]
    b2.linear(y, x, w)
    torch.cuda.synchronize()
    _check_close(torch, y, _ref(torch, x, w, None, 0, dtype), dtype, x, w)
    assert bool((ybuf[:, 1000:] == 7.0).all())


def test_linear_back_to_back_on_one_stream(b2, cuda):
    """Chained launches (programmatic dependent launch): each layer reads the
    previous layer's output, as the engine's FC -> FC-proj pair does."""
    import torch
    dtype = torch.float16
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(128, 1024, generator=g, device="cuda").to(dtype)
    w1 = (torch.randn(4096, 1024, generator=g, device="cuda") * 0.02).to(dtype)
    b1 = (torch.randn(4096, generator=g, device="cuda") * 0.02).to(dtype)
    w2 = (torch.randn(1024, 4096, generator=g, device="cuda") * 0.02).to(dtype)
    h = torch.empty(128, 4096, device="cuda", dtype=dtype)
    y = torch.empty(128, 1024, device="cuda", dtype=dtype)
    for _ in range(3):
        b2.linear(h, x, w1, b1, b2.LINEAR_GELU)
        b2.linear(y, h, w2)
    torch.cuda.synchronize()
    assert b2.device_errors() == 0
    h_ref = _ref(torch, x, w1, b1, 1, dtype)
    _check_close(torch, h, h_ref, dtype, x, w1)
    _check_close(torch, y, _ref(torch, h, w2, None, 0, dtype), dtype, h, w2)


def test_linear_argument_errors(b2, cuda):
    import torch
    x = torch.zeros(4, 64, device="cuda", dtype=torch.float16)
    w = torch.zeros(128, 64, device="cuda", dtype=torch.float16)
    y = torch.zeros(4, 128, device="cuda", dtype=torch.float16)
    with pytest.raises(b2.B2Error) as e:
        b2.linear(y.float(), x.float(), w.float())
    assert e.value.code == -2  # F32 stays on cuBLAS
    xs = torch.zeros(4, 72, device="cuda", dtype=torch.float16)[:, 4:68]  # rows start 8 bytes in
    with pytest.raises(b2.B2Error) as e:
        b2.linear(y, xs, w)
    assert e.value.code == -4
    w60 = torch.zeros(128, 60, device="cuda", dtype=torch.float16)
    with pytest.raises(b2.B2Error) as e:
        b2.linear(y, x[:, :60], w60)
    assert e.value.code == -4  # in_features not a multiple of 8
    y130 = torch.zeros(4, 130, device="cuda", dtype=torch.float16)
    with pytest.raises(b2.B2Error) as e:
        b2.linear(y130, x, torch.zeros(130, 64, device="cuda", dtype=torch.float16))
    assert e.value.code == -4  # y_row_stride not a multiple of 8
