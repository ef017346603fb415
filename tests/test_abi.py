"""The C-ABI library loads, exports every declared symbol, and rejects bad
arguments on the host before any launch (CPU only: no call here reaches the GPU)."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT


def declared_functions(header: str) -> list[str]:
    text = (ROOT / "include" / header).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b2_\w+)\s*\(", text)))


def test_decode_library_exports_every_declared_symbol(b2):
    lib = b2.load()
    names = declared_functions("b2_decode.h")
    assert set(names) == set(b2.DECODE_SYMBOLS), "binding list out of date with include/b2_decode.h"
    for n in names:
        assert hasattr(lib, n), f"{n} not exported"
    assert "sm_100a" in b2.version()


def test_library_has_no_cpu_fallback_symbols(b2):
    # The product library must not carry the oracle.
    lib = b2.load()
    for n in ("oracle_paged_attention", "oracle_kv_append"):
        with pytest.raises(AttributeError):
            getattr(lib, n)


def _attn_args(b2, **kw):
    base = dict(dtype=b2.F16, out_dtype=b2.F32, q=16, q_row_stride=768, q_bias=None, kv_pool=32, block_tables=48,
                seq_lens=64, out=80, batch=4, n_head=12, n_kv_head=12, head_dim=64, max_blocks_per_seq=8,
                layer_idx=0, n_layer=1, num_blocks=100, scale=0.0)
    base.update(kw)
    return b2.PagedAttnArgs(**base)


@pytest.mark.parametrize("kw,code", [
    (dict(dtype=7), -2),
    (dict(out_dtype=2), -2),
    (dict(head_dim=96), -6),
    (dict(n_kv_head=5), -3),
    (dict(n_head=96, n_kv_head=12), -6),
    (dict(layer_idx=1), -3),
    (dict(num_blocks=0), -3),
    (dict(q=None), -1),
    (dict(q=17), -4),
    (dict(q_row_stride=700), -3),
    (dict(q_row_stride=772), -4),
])
def test_paged_attention_host_checks(b2, kw, code):
    lib = b2.load()
    args = _attn_args(b2, **kw)
    ws = ctypes.create_string_buffer(64)
    assert lib.b2_paged_attention(ctypes.byref(args), ctypes.addressof(ws), 64, None) == code
    assert lib.b2_last_error_string().decode() != ""


def test_paged_attention_host_checks_before_any_copy(b2):
    # The host-buffer entry point validates everything before its first copy.
    lib = b2.load()
    assert lib.b2_paged_attention_host(ctypes.byref(_attn_args(b2)), None, None, 0, None) == -1  # io NULL
    io = b2.AttnHostIO(None, None, None, None)
    for kw, code in ((dict(dtype=7), -2), (dict(q=17), -4), (dict(head_dim=96), -6), (dict(q=None), -1)):
        args = _attn_args(b2, **kw)
        assert lib.b2_paged_attention_host(ctypes.byref(args), ctypes.byref(io), None, 0, None) == code
        assert lib.b2_last_error_string().decode() != ""


def test_paged_attention_empty_batch_is_a_no_op(b2):
    args = _attn_args(b2, batch=0, q=None, kv_pool=None)
    assert b2.load().b2_paged_attention(ctypes.byref(args), None, 0, None) == 0


def _append_args(b2, **kw):
    base = dict(dtype=b2.BF16, kv_pool=16, k=32, v=48, kv_row_stride=3 * 512, k_bias=None, v_bias=None,
                block_tables=64, seq_lens=80, seq_lens_post=None, batch=2, n_kv_head=4, head_dim=128,
                max_blocks_per_seq=4, layer_idx=0, n_layer=1, num_blocks=10)
    base.update(kw)
    return b2.KvAppendArgs(**base)


@pytest.mark.parametrize("kw,code", [
    (dict(dtype=3), -2),
    (dict(k=None), -1),
    (dict(head_dim=80), -6),
    (dict(kv_row_stride=100), -3),
    (dict(seq_lens_post=80), -3),
    (dict(v=50), -4),
    (dict(layer_idx=-1), -3),
])
def test_kv_append_host_checks(b2, kw, code):
    args = _append_args(b2, **kw)
    assert b2.load().b2_kv_append(ctypes.byref(args), None) == code


def test_row_kernel_host_checks(b2):
    lib = b2.load()
    assert lib.b2_add_layernorm(5, 16, 16, 16, None, 16, 16, 16, 4, 768, 1e-5, None) == -2
    assert lib.b2_add_layernorm(1, 16, 16, 16, None, 16, 16, 16, 4, 770, 1e-5, None) == -3
    assert lib.b2_add_layernorm(1, 16, 16, 16, None, 16, 16, 16, 4, 8 * 4097, 1e-5, None) == -6  # > 4096 chunks
    assert lib.b2_add_layernorm(1, None, 16, 16, None, 16, 16, 16, 4, 768, 1e-5, None) == -1
    assert lib.b2_bias_gelu(1, 16, 16, 18, 2, 3072, None) == -4
    assert lib.b2_add_bias(0, 16, 16, 16, 2, 6, None) == -3
    assert lib.b2_add_one(None, 16, 3, None) == -1
    assert lib.b2_embedding(1, 16, 16, 16, 16, 16, 2, 768, 0, 1024, None) == -3
    assert lib.b2_argmax(1, None, 16, 2, 100, None) == -1
    for fn in (lib.b2_bias_gelu, lib.b2_add_bias):
        assert fn(1, 16, 16, 16, 0, 768, None) == 0  # empty batch


def test_barrier_limit_is_checked_on_the_host(b2):
    lib = b2.load()
    assert lib.b2_tp_barrier_timed(16, 32, 0, 2, 48, 0, 0, None) == -3  # zero limit: B2_ERR_SHAPE, no launch
    assert lib.b2_tp_barrier_timed(16, 32, 0, 2, 48, 0, 61 * 10**9, None) == -3
    assert lib.b2_tp_barrier_timed(16, 32, 2, 2, 48, 0, 10**6, None) == -3  # rank out of range


def _lm_args(b2, **kw):
    base = dict(dtype=b2.BF16, x=16, x_row_stride=1600, w=32, batch=4, d_model=1600, vocab=50257, out_tokens=48,
                workspace=64, workspace_bytes=1 << 20)
    base.update(kw)
    return b2.LmHeadArgmaxArgs(**base)


@pytest.mark.parametrize("kw,code", [
    (dict(dtype=0), -2),  # F32
    (dict(vocab=0), -3),
    (dict(x=None), -1),
    (dict(workspace=None), -1),
    (dict(x_row_stride=1000), -3),
    (dict(d_model=1604, x_row_stride=1604), -4),
    (dict(x=24), -4),
    (dict(workspace_bytes=16), -5),
    (dict(workspace=72), -5),
])
def test_lm_head_argmax_host_checks(b2, kw, code):
    lib = b2.load()
    assert lib.b2_lm_head_argmax(ctypes.byref(_lm_args(b2, **kw)), None) == code
    assert lib.b2_last_error_string().decode() != ""


def test_lm_head_argmax_workspace_size_and_empty_batch(b2):
    lib = b2.load()
    assert lib.b2_lm_head_argmax_workspace_bytes(512) >= 16 + 8 * 512
    assert lib.b2_lm_head_argmax_workspace_bytes(512) % 256 == 0
    assert lib.b2_lm_head_argmax(ctypes.byref(_lm_args(b2, batch=0, x=None, w=None)), None) == 0
