"""ctypes binding of the CPU oracle (liboracle.so, built from b2_oracle.c) and of
the reference's own CPU path (_ref/libref_cpu.so, built from the reference
sources by oracle/Makefile).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU legs of bench.py, never by the product.  Arrays are numpy; dtype codes are
0 = f32, 1 = f16, 2 = bf16 (stored as uint16 bit patterns for the 16-bit types).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
F32, F16, BF16 = 0, 1, 2

_lib = None
_ref = None


def _reference_checkout() -> Path | None:
    """The reference checkout: $B2_REFERENCE, else /root/reference where it exists
    (the build container; GPU boxes use the prebuilt _ref files)."""
    import os
    for c in (os.environ.get("B2_REFERENCE"), "/root/reference"):
        if c and (Path(c) / "gpu-engine" / "src" / "reference" / "cpu_model.cpp").exists():
            return Path(c)
    return None


def _json_include() -> Path | None:
    """A directory holding nlohmann/json.hpp ($B2_JSON_INCLUDE, system include
    dirs, then copies vendored by installed Python packages)."""
    import os
    import site
    cands = [Path(os.environ["B2_JSON_INCLUDE"])] if os.environ.get("B2_JSON_INCLUDE") else []
    cands += [Path("/usr/include"), Path("/usr/local/include")]
    for sp in site.getsitepackages():
        cands += sorted(Path(sp).glob("include/*/thirdparty"))
        cands += sorted(Path(sp).glob("*/include"))
    for c in cands:
        if (c / "nlohmann" / "json.hpp").exists():
            return c
    return None


def build() -> None:
    """Builds liboracle.so, and -- when the reference checkout is present -- the
    reference's CPU path and scheduler harnesses under _ref/."""
    cmd = ["make", "-s", "-C", str(HERE), "all"]
    ref, js = _reference_checkout(), _json_include()
    if ref is not None and js is not None:
        cmd += [f"REF={ref}", f"JSON={js}"]
    subprocess.run(cmd, check=True)


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = HERE / "liboracle.so"
        if not path.exists():
            build()
        _lib = ctypes.CDLL(str(path))
        _lib.oracle_paged_attention.restype = ctypes.c_int
        _lib.oracle_kv_append.restype = ctypes.c_int
        _lib.oracle_block_bytes.restype = ctypes.c_size_t
        _lib.oracle_tied_lm_head_argmax.restype = ctypes.c_int
    return _lib


def ref_available() -> bool:
    return (HERE / "_ref" / "libref_cpu.so").exists()


def load_ref() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        path = HERE / "_ref" / "libref_cpu.so"
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: build it with `make -C oracle ref` where the reference exists")
        _ref = ctypes.CDLL(str(path))
        _ref.ref_last_error.restype = ctypes.c_char_p
        _ref.ref_greedy_generate_many.restype = ctypes.c_double
        _ref.ref_block_bytes.restype = ctypes.c_size_t
        _ref.ref_pool_create.restype = ctypes.c_void_p
        _ref.ref_pool_destroy.argtypes = [ctypes.c_void_p]
        _ref.ref_pool_allocate.argtypes = [ctypes.c_void_p]
        _ref.ref_pool_num_free.argtypes = [ctypes.c_void_p]
        _ref.ref_pool_free.argtypes = [ctypes.c_void_p, ctypes.c_int]
    return _ref


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


# ------------------------------------------------------------- conversions

def round_to(dt: int, x: np.ndarray) -> np.ndarray:
    """float32 array -> storage of dtype dt (float32, or uint16 bit patterns)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.float32 if dt == F32 else np.uint16)
    load().oracle_round_to_dtype(dt, _p(x), _p(out), ctypes.c_size_t(x.size))
    return out


def widen(dt: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x)
    out = np.empty(x.shape, dtype=np.float32)
    load().oracle_widen_from_dtype(dt, _p(x), _p(out), ctypes.c_size_t(x.size))
    return out


# ------------------------------------------------------------------ kernels

def paged_attention(dt, q, q_row_stride, pool, block_tables, seq_lens, *, n_head, n_kv_head, head_dim,
                    max_blocks_per_seq, layer_idx, n_layer, scale=0.0, nthreads=1) -> np.ndarray:
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    batch = sl.shape[0]
    out = np.zeros((batch, n_head, head_dim), dtype=np.float32)
    rc = load().oracle_paged_attention(dt, _p(np.ascontiguousarray(q)), q_row_stride, _p(np.ascontiguousarray(pool)),
                                       _p(bt), _p(sl), _p(out), batch, n_head, n_kv_head, head_dim,
                                       max_blocks_per_seq, layer_idx, n_layer, ctypes.c_float(scale), nthreads)
    if rc != 0:
        raise ValueError(f"oracle_paged_attention rejected its inputs (rc={rc})")
    return out


def kv_append(dt, pool, k, v, kv_row_stride, block_tables, seq_lens, *, n_kv_head, head_dim, max_blocks_per_seq,
              layer_idx, n_layer, num_blocks) -> None:
    """In place on pool (numpy)."""
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    rc = load().oracle_kv_append(dt, _p(pool), _p(np.ascontiguousarray(k)), _p(np.ascontiguousarray(v)),
                                 kv_row_stride, _p(bt), _p(sl), sl.shape[0], n_kv_head, head_dim,
                                 max_blocks_per_seq, layer_idx, n_layer, num_blocks)
    if rc != 0:
        raise ValueError("oracle_kv_append rejected its inputs")


def add_layernorm(dt, x, residual_in, gamma, beta, eps, bias=None):
    """Returns (out fp32, out rounded to dt, residual_out in dt); x and bias may be None."""
    b, d = residual_in.shape
    out = np.empty((b, d), dtype=np.float32)
    out_dt = np.empty((b, d), dtype=np.float32 if dt == F32 else np.uint16)
    res_out = np.empty_like(out_dt)
    xx = None if x is None else np.ascontiguousarray(x)
    bb = None if bias is None else np.ascontiguousarray(bias)
    load().oracle_add_layernorm(dt, _p(out), _p(out_dt), _p(res_out), _p(xx), _p(bb),
                                _p(np.ascontiguousarray(residual_in)), _p(np.ascontiguousarray(gamma)),
                                _p(np.ascontiguousarray(beta)), b, d, ctypes.c_float(eps))
    return out, out_dt, res_out


def bias_gelu(dt, x, bias) -> np.ndarray:
    b, d = x.shape
    out = np.empty((b, d), dtype=np.float32)
    load().oracle_bias_gelu(dt, _p(out), _p(np.ascontiguousarray(x)), _p(np.ascontiguousarray(bias)), b, d)
    return out


def add_bias(dt, x, bias) -> np.ndarray:
    b, d = x.shape
    out = np.empty((b, d), dtype=np.float32)
    load().oracle_add_bias(dt, _p(out), _p(np.ascontiguousarray(x)), _p(np.ascontiguousarray(bias)), b, d)
    return out


def embedding(dt, wte, wpe, token_ids, positions) -> np.ndarray:
    tok = np.ascontiguousarray(token_ids, dtype=np.int32)
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    d = wte.shape[1]
    out = np.empty((tok.shape[0], d), dtype=np.float32)
    load().oracle_embedding(dt, _p(out), _p(np.ascontiguousarray(wte)), _p(np.ascontiguousarray(wpe)), _p(tok),
                            _p(pos), tok.shape[0], d)
    return out


def argmax(dt, logits) -> np.ndarray:
    b, v = logits.shape
    out = np.empty((b,), dtype=np.int32)
    load().oracle_argmax(dt, _p(out), _p(np.ascontiguousarray(logits)), b, v)
    return out


def linear(x: np.ndarray, W: np.ndarray, b: np.ndarray | None, nthreads: int = 8) -> np.ndarray:
    """cpu_model.cpp:11-25 on float32 arrays: x [T,I], W [O,I] -> [T,O]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    W = np.ascontiguousarray(W, dtype=np.float32)
    T, I = x.shape
    O = W.shape[0]
    out = np.empty((T, O), dtype=np.float32)
    load().oracle_linear(_p(out), _p(x), T, I, O, _p(W), _p(None if b is None else np.ascontiguousarray(b, np.float32)),
                         nthreads)
    return out


def tied_lm_head_argmax(wte: np.ndarray, hidden: np.ndarray) -> int:
    v, d = wte.shape
    return int(load().oracle_tied_lm_head_argmax(_p(np.ascontiguousarray(wte, np.float32)),
                                                 _p(np.ascontiguousarray(hidden, np.float32)), v, d))


def block_bytes(n_layer, n_heads, head_dim, elem_bytes=2) -> int:
    return int(load().oracle_block_bytes(n_layer, n_heads, head_dim, elem_bytes))


# ------------------------------------------------- reference CPU forward path

def ref_greedy_generate(model_dir: str, prompts: list[list[int]], n_new: int, n_threads: int = 1):
    """CPUModel::greedy_generate of the reference (cpu_model.cpp:198-216), one
    CPUModel per thread.  Returns (list of token lists, elapsed seconds)."""
    lib = load_ref()
    flat = np.array([t for p in prompts for t in p], dtype=np.int32)
    lens = np.array([len(p) for p in prompts], dtype=np.int32)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int32)
    out = np.zeros((len(prompts), n_new), dtype=np.int32)
    counts = np.zeros((len(prompts),), dtype=np.int32)
    secs = lib.ref_greedy_generate_many(str(model_dir).encode(), _p(flat), _p(offs), _p(lens), len(prompts), n_new,
                                        n_threads, _p(out), _p(counts))
    if secs < 0:
        raise RuntimeError(lib.ref_last_error().decode())
    return [out[i, : counts[i]].tolist() for i in range(len(prompts))], float(secs)
