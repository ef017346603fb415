"""Python binding of the sm_100a decode hot path (libb2decode.so, include/b2_decode.h).

This is a thin ctypes layer over the C-ABI, used by the tests and the bench.
It mirrors the reference's kernel launchers (gpu-engine/include/engine/kernels.h):
``kv_append``, ``paged_attention``, ``add_layernorm``, ``bias_gelu``, ``add_bias``,
``add_one``, ``embedding``, ``argmax`` -- same argument meaning, plus the dtype,
n_kv_head and num_blocks fields of the C-ABI.  Tensors are torch CUDA tensors;
only their data pointers cross the boundary.

There is no CPU fallback: if the native library is missing, loading it raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_DIR = PKG_DIR / "lib"
ROOT_DIR = PKG_DIR.parent

F32, F16, BF16 = 0, 1, 2
BLOCK_TOKENS = 16

B2_OK = 0
ATTN_INPUTS_READY, ATTN_NEWEST_ROW_PENDING = 1, 2  # B2PagedAttnArgs.flags
LINEAR_STORE, LINEAR_GELU = 0, 1  # B2LinearArgs.epilogue
DEVERR_BLOCK_ID, DEVERR_SEQ_LEN, DEVERR_TIMEOUT, DEVERR_TOKEN = 1, 2, 4, 8

# Every symbol include/b2_decode.h declares.
DECODE_SYMBOLS = (
    "b2_version", "b2_last_error_string", "b2_device_errors", "b2_kv_append",
    "b2_paged_attention_workspace_bytes", "b2_paged_attention",
    "b2_add_layernorm", "b2_bias_gelu", "b2_add_bias", "b2_add_one", "b2_embedding", "b2_argmax",
    "b2_paged_attention_noalloc", "b2_argmax_rows", "b2_paged_attention_gather", "b2_tp_barrier",
    "b2_tp_epoch_bump", "b2_linear", "b2_prefill_attention", "b2_paged_attention_host",
    "b2_tp_barrier_timed", "b2_device_error_word", "b2_raise_device_error",
    "b2_lm_head_argmax_workspace_bytes", "b2_lm_head_argmax",
)

_c_int, _c_float, _vp = ctypes.c_int32, ctypes.c_float, ctypes.c_void_p


class KvAppendArgs(ctypes.Structure):
    _fields_ = [("dtype", _c_int), ("kv_pool", _vp), ("k", _vp), ("v", _vp), ("kv_row_stride", _c_int),
                ("k_bias", _vp), ("v_bias", _vp), ("block_tables", _vp), ("seq_lens", _vp),
                ("seq_lens_post", _vp), ("batch", _c_int), ("n_kv_head", _c_int), ("head_dim", _c_int),
                ("max_blocks_per_seq", _c_int), ("layer_idx", _c_int), ("n_layer", _c_int),
                ("num_blocks", _c_int)]


class PagedAttnArgs(ctypes.Structure):
    _fields_ = [("dtype", _c_int), ("out_dtype", _c_int), ("q", _vp), ("q_row_stride", _c_int), ("q_bias", _vp),
                ("kv_pool", _vp), ("block_tables", _vp), ("seq_lens", _vp), ("out", _vp), ("batch", _c_int),
                ("n_head", _c_int), ("n_kv_head", _c_int), ("head_dim", _c_int), ("max_blocks_per_seq", _c_int),
                ("layer_idx", _c_int), ("n_layer", _c_int), ("num_blocks", _c_int), ("scale", _c_float),
                ("flags", _c_int), ("max_ctas", _c_int)]


class AttnHostIO(ctypes.Structure):
    _fields_ = [("q", _vp), ("block_tables", _vp), ("seq_lens", _vp), ("out", _vp)]


class LinearArgs(ctypes.Structure):
    _fields_ = [("dtype", _c_int), ("x", _vp), ("x_row_stride", ctypes.c_int64), ("w", _vp), ("bias", _vp),
                ("y", _vp), ("y_row_stride", ctypes.c_int64), ("batch", _c_int), ("in_features", _c_int),
                ("out_features", _c_int), ("epilogue", _c_int)]


class LmHeadArgmaxArgs(ctypes.Structure):
    _fields_ = [("dtype", _c_int), ("x", _vp), ("x_row_stride", ctypes.c_int64), ("w", _vp), ("batch", _c_int),
                ("d_model", _c_int), ("vocab", _c_int), ("out_tokens", _vp), ("workspace", _vp),
                ("workspace_bytes", ctypes.c_size_t)]


class PrefillAttnArgs(ctypes.Structure):
    _fields_ = [("dtype", _c_int), ("q", _vp), ("q_row_stride", _c_int), ("q_bias", _vp), ("kv_pool", _vp),
                ("block_tables", _vp), ("seq_lens_pre", _vp), ("q_start", _vp), ("q_len", _vp), ("out", _vp),
                ("out_row_stride", _c_int), ("n_seqs", _c_int), ("n_head", _c_int), ("n_kv_head", _c_int),
                ("head_dim", _c_int), ("max_blocks_per_seq", _c_int), ("layer_idx", _c_int), ("n_layer", _c_int),
                ("num_blocks", _c_int), ("max_q_len", _c_int), ("scale", _c_float)]


class B2Error(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"b2 status {code}: {what}")
        self.code = code


_lib = None


def lib_path() -> Path:
    return LIB_DIR / "libb2decode.so"


def load() -> ctypes.CDLL:
    """Loads libb2decode.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not path.exists():
        raise FileNotFoundError(f"{path} is missing: run llm-inference-server_b200/build.py (nvcc, sm_100a)")
    lib = ctypes.CDLL(str(path))
    lib.b2_version.restype = ctypes.c_char_p
    lib.b2_last_error_string.restype = ctypes.c_char_p
    lib.b2_device_errors.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
    lib.b2_kv_append.argtypes = [ctypes.POINTER(KvAppendArgs), _vp]
    lib.b2_paged_attention_workspace_bytes.argtypes = [ctypes.POINTER(PagedAttnArgs)]
    lib.b2_paged_attention_workspace_bytes.restype = ctypes.c_size_t
    lib.b2_paged_attention.argtypes = [ctypes.POINTER(PagedAttnArgs), _vp, ctypes.c_size_t, _vp]
    lib.b2_paged_attention_host.argtypes = [ctypes.POINTER(PagedAttnArgs), ctypes.POINTER(AttnHostIO), _vp,
                                            ctypes.c_size_t, _vp]
    lib.b2_add_layernorm.argtypes = [_c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_float, _vp]
    lib.b2_bias_gelu.argtypes = [_c_int, _vp, _vp, _vp, _c_int, _c_int, _vp]
    lib.b2_add_bias.argtypes = [_c_int, _vp, _vp, _vp, _c_int, _c_int, _vp]
    lib.b2_add_one.argtypes = [_vp, _vp, _c_int, _vp]
    lib.b2_embedding.argtypes = [_c_int, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp]
    lib.b2_argmax.argtypes = [_c_int, _vp, _vp, _c_int, _c_int, _vp]
    lib.b2_argmax_rows.argtypes = [_c_int, _vp, _vp, ctypes.c_int64, _c_int, _c_int, _vp]
    lib.b2_linear.argtypes = [ctypes.POINTER(LinearArgs), _vp]
    lib.b2_lm_head_argmax_workspace_bytes.argtypes = [_c_int]
    lib.b2_lm_head_argmax_workspace_bytes.restype = ctypes.c_size_t
    lib.b2_lm_head_argmax.argtypes = [ctypes.POINTER(LmHeadArgmaxArgs), _vp]
    lib.b2_prefill_attention.argtypes = [ctypes.POINTER(PrefillAttnArgs), _vp]
    lib.b2_paged_attention_noalloc.argtypes = [ctypes.POINTER(PagedAttnArgs), _vp]
    lib.b2_tp_barrier.argtypes = [_vp, _vp, _c_int, _c_int, _vp, _c_int, _vp]
    lib.b2_tp_barrier_timed.argtypes = [_vp, _vp, _c_int, _c_int, _vp, _c_int, ctypes.c_uint64, _vp]
    lib.b2_tp_epoch_bump.argtypes = [_vp, _vp]
    lib.b2_device_error_word.argtypes = [ctypes.POINTER(ctypes.c_void_p)]
    lib.b2_raise_device_error.argtypes = [ctypes.c_uint32, _vp]
    _lib = lib
    return lib


def _check(rc: int) -> None:
    if rc != B2_OK:
        raise B2Error(rc, load().b2_last_error_string().decode())


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


def dtype_code(torch_dtype) -> int:
    import torch
    return {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}[torch_dtype]


def version() -> str:
    return load().b2_version().decode()


def device_errors() -> int:
    v = ctypes.c_uint32(0)
    _check(load().b2_device_errors(ctypes.byref(v)))
    return int(v.value)


# --------------------------------------------------------------- launchers

def kv_append(kv_pool, k, v, kv_row_stride, block_tables, seq_lens, *, n_kv_head, head_dim, max_blocks_per_seq,
              layer_idx, n_layer, num_blocks, k_bias=None, v_bias=None, seq_lens_post=None, stream=None):
    """kernels::launch_kv_append (kernels.h:51-60): write this step's K/V into slot seq_lens[b]."""
    a = KvAppendArgs(dtype_code(kv_pool.dtype), _ptr(kv_pool), _ptr(k), _ptr(v), kv_row_stride, _ptr(k_bias),
                     _ptr(v_bias), _ptr(block_tables), _ptr(seq_lens), _ptr(seq_lens_post), block_tables.shape[0],
                     n_kv_head, head_dim, max_blocks_per_seq, layer_idx, n_layer, num_blocks)
    _check(load().b2_kv_append(ctypes.byref(a), _stream(stream)))


def attn_args(q, q_row_stride, kv_pool, block_tables, seq_lens, out, *, n_head, n_kv_head, head_dim,
              max_blocks_per_seq, layer_idx, n_layer, num_blocks, scale=0.0, q_bias=None, flags=0,
              max_ctas=0) -> PagedAttnArgs:
    return PagedAttnArgs(dtype_code(kv_pool.dtype), dtype_code(out.dtype), _ptr(q), q_row_stride, _ptr(q_bias),
                         _ptr(kv_pool), _ptr(block_tables), _ptr(seq_lens), _ptr(out), block_tables.shape[0], n_head,
                         n_kv_head, head_dim, max_blocks_per_seq, layer_idx, n_layer, num_blocks, scale, flags,
                         max_ctas)


def attention_workspace(args: PagedAttnArgs):
    """Allocates (torch) a zeroed workspace for launches shaped like args (the
    per-sequence piece counters in it must start at zero; launches leave them
    at zero)."""
    import torch
    n = load().b2_paged_attention_workspace_bytes(ctypes.byref(args))
    if n == 0:
        raise B2Error(-3, load().b2_last_error_string().decode() or "workspace size query failed")
    return torch.zeros(n, dtype=torch.uint8, device="cuda")


def paged_attention(args: PagedAttnArgs, workspace, stream=None) -> None:
    """kernels::launch_paged_attention (kernels.h:67-87) with the C-ABI's argument struct."""
    _check(load().b2_paged_attention(ctypes.byref(args), workspace.data_ptr(), workspace.numel(), _stream(stream)))


def paged_attention_host(args: PagedAttnArgs, workspace, *, q=None, block_tables=None, seq_lens=None, out=None,
                         stream=None) -> None:
    """One synchronous attention call from host buffers (pinned torch CPU
    tensors or None): upload q / block_tables / seq_lens into the device
    arrays args names, launch, download args.out into `out`, wait -- the host
    side of Engine::decode_step (engine.cu:343-368) around one attention."""
    io = AttnHostIO(_ptr(q), _ptr(block_tables), _ptr(seq_lens), _ptr(out))
    _check(load().b2_paged_attention_host(ctypes.byref(args), ctypes.byref(io), workspace.data_ptr(),
                                          workspace.numel(), _stream(stream)))


def add_layernorm(out, residual_out, x, residual_in, gamma, beta, eps, bias=None, stream=None):
    b, d = residual_in.shape
    _check(load().b2_add_layernorm(dtype_code(residual_in.dtype), _ptr(out), _ptr(residual_out), _ptr(x), _ptr(bias),
                                   _ptr(residual_in), _ptr(gamma), _ptr(beta), b, d, eps, _stream(stream)))


def bias_gelu(out, x, bias, stream=None):
    b, d = x.shape
    _check(load().b2_bias_gelu(dtype_code(x.dtype), _ptr(out), _ptr(x), _ptr(bias), b, d, _stream(stream)))


def add_bias(out, x, bias, stream=None):
    b, d = x.shape
    _check(load().b2_add_bias(dtype_code(x.dtype), _ptr(out), _ptr(x), _ptr(bias), b, d, _stream(stream)))


def add_one(out, inp, stream=None):
    _check(load().b2_add_one(_ptr(out), _ptr(inp), inp.numel(), _stream(stream)))


def embedding(out, wte, wpe, token_ids, positions, stream=None):
    _check(load().b2_embedding(dtype_code(wte.dtype), _ptr(out), _ptr(wte), _ptr(wpe), _ptr(token_ids),
                               _ptr(positions), token_ids.numel(), wte.shape[1], wte.shape[0], wpe.shape[0],
                               _stream(stream)))


def argmax(out_tokens, logits, stream=None, vocab=None):
    """Row-wise greedy argmax.  A contiguous [batch, vocab] tensor goes through
    b2_argmax; with vocab < logits.shape[1] (padded rows) or a strided view,
    through b2_argmax_rows."""
    b, v = logits.shape
    vocab = v if vocab is None else vocab
    if vocab == v and logits.is_contiguous():
        _check(load().b2_argmax(dtype_code(logits.dtype), _ptr(out_tokens), _ptr(logits), b, v, _stream(stream)))
    else:
        _check(load().b2_argmax_rows(dtype_code(logits.dtype), _ptr(out_tokens), _ptr(logits), logits.stride(0), b,
                                     vocab, _stream(stream)))


def linear(y, x, w, bias=None, epilogue=LINEAR_STORE, stream=None):
    """y = epilogue(x @ w.T) on the tensor cores (b2_linear): x [batch, in],
    w [out, in] contiguous, y [batch, out] (x and y rows may be strided)."""
    if not w.is_contiguous() or x.stride(1) != 1 or y.stride(1) != 1:
        raise ValueError("w must be contiguous and x, y must have unit column stride")
    a = LinearArgs(dtype_code(w.dtype), _ptr(x), x.stride(0), _ptr(w), _ptr(bias), _ptr(y), y.stride(0), x.shape[0],
                   w.shape[1], w.shape[0], epilogue)
    _check(load().b2_linear(ctypes.byref(a), _stream(stream)))


def lm_head_argmax_workspace(batch: int, device=None):
    """A zeroed workspace for lm_head_argmax at up to `batch` rows (every
    launch leaves it zeroed again)."""
    import torch
    n = int(load().b2_lm_head_argmax_workspace_bytes(batch))
    return torch.zeros(n, dtype=torch.uint8, device=device if device is not None else "cuda")


def lm_head_argmax(out_tokens, x, w, vocab=None, workspace=None, stream=None):
    """out_tokens[b] = argmax_v dtype(x[b] . w[v]) over v < vocab
    (b2_lm_head_argmax: the tied lm_head GEMM and the greedy argmax in one
    tensor-core kernel).  x [batch, d_model] (rows may be strided), w
    [>= vocab, d_model] contiguous, out_tokens int32 [batch]."""
    if not w.is_contiguous() or x.stride(1) != 1:
        raise ValueError("w must be contiguous and x must have unit column stride")
    batch, d = x.shape
    vocab = w.shape[0] if vocab is None else vocab
    if workspace is None:
        workspace = lm_head_argmax_workspace(batch, x.device)
    a = LmHeadArgmaxArgs(dtype_code(w.dtype), _ptr(x), x.stride(0), _ptr(w), batch, d, vocab, _ptr(out_tokens),
                         _ptr(workspace), workspace.numel() * workspace.element_size())
    _check(load().b2_lm_head_argmax(ctypes.byref(a), _stream(stream)))


def prefill_attention(out, q, q_row_stride, kv_pool, block_tables, seq_lens_pre, q_start, q_len, *, n_head, n_kv_head,
                      head_dim, max_blocks_per_seq, layer_idx, n_layer, num_blocks, max_q_len, q_bias=None, scale=0.0,
                      stream=None):
    """b2_prefill_attention: causal attention of each sequence's new rows over
    the paged pool (rows q_start[b] .. q_start[b] + q_len[b] - 1 of q / out)."""
    a = PrefillAttnArgs(dtype_code(kv_pool.dtype), _ptr(q), q_row_stride, _ptr(q_bias), _ptr(kv_pool),
                        _ptr(block_tables), _ptr(seq_lens_pre), _ptr(q_start), _ptr(q_len), _ptr(out), out.stride(0),
                        seq_lens_pre.numel(), n_head, n_kv_head, head_dim, max_blocks_per_seq, layer_idx, n_layer,
                        num_blocks, max_q_len, scale)
    _check(load().b2_prefill_attention(ctypes.byref(a), _stream(stream)))
