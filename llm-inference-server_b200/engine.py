"""Python binding of the GPT-2 decode engine (libb2engine.so, include/b2_engine.h).

``Engine`` mirrors the reference's ``Engine`` (gpu-engine/include/engine/engine_api.h:15-48):
``init(weights_dir, cfg) -> bool``, ``add_sequence(prompt) -> id`` (-1 when the KV
pool is exhausted), ``decode_step(seq_ids) -> next tokens``, ``free_sequence(id)``,
``free_blocks()``, ``set_use_cuda_graphs(bool)``.  ``BlockPool`` exposes the
engine's allocator with the reference BlockPool's behaviour
(gpu-engine/src/kv_cache_pool.cpp:6-28): free() raises IndexError for an id out
of range and RuntimeError for one that is not allocated, where the C++ class
throws std::out_of_range / std::logic_error.

There is no CPU fallback: if the native library is missing, loading it raises.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path
from typing import Sequence

from . import F16, LIB_DIR, B2Error, load as load_decode

ENGINE_SYMBOLS = (
    "b2_engine_create", "b2_engine_create_synthetic", "b2_engine_destroy", "b2_engine_add_sequence",
    "b2_engine_add_sequence_cached", "b2_engine_decode_step", "b2_engine_free_sequence",
    "b2_engine_free_blocks", "b2_engine_set_use_cuda_graphs", "b2_engine_set_prefill_tensor_cores",
    "b2_engine_shape", "b2_engine_stream",
    "b2_engine_last_error", "b2_block_pool_create", "b2_block_pool_destroy", "b2_block_pool_allocate",
    "b2_block_pool_free", "b2_block_pool_num_free", "b2_engine_tp_handle", "b2_engine_tp_connect",
    "b2_engine_prefill", "b2_engine_tp_nccl_id", "b2_engine_tp_connect_nccl", "b2_engine_set_linear_tensor_cores",
    "b2_engine_last_step_outputs", "b2_engine_set_gemm_mode", "b2_engine_set_lm_head_fused",
)

TP_HANDLE_BYTES = 128
TP_NCCL_ID_BYTES = 128

ERR_POOL, ERR_IO, ERR_KERNEL = -8, -9, -10

_i32, _vp = ctypes.c_int32, ctypes.c_void_p


class EngineConfig(ctypes.Structure):
    """gpu-engine/include/engine/engine_api.h:9-13 plus dtype, graphs and device."""
    _fields_ = [("max_batch", _i32), ("max_seq_len", _i32), ("kv_block_budget", _i32), ("dtype", _i32),
                ("use_cuda_graphs", _i32), ("device", _i32), ("tp_rank", _i32), ("tp_size", _i32),
                ("max_prefill_tokens", _i32), ("tp_allgather", _i32)]


class ModelShape(ctypes.Structure):
    """gpu-engine/include/engine/model.h:7-18."""
    _fields_ = [("n_layer", _i32), ("n_head", _i32), ("d_model", _i32), ("vocab_size", _i32), ("n_ctx", _i32),
                ("layer_norm_epsilon", ctypes.c_float), ("eos_token_id", _i32)]


_lib = None


def lib_path() -> Path:
    return LIB_DIR / "libb2engine.so"


def load() -> ctypes.CDLL:
    """Loads libb2engine.so (and libb2decode.so, which it links); raises if unbuilt."""
    global _lib
    if _lib is not None:
        return _lib
    load_decode()
    path = lib_path()
    if not path.exists():
        raise FileNotFoundError(f"{path} is missing: run llm-inference-server_b200/build.py")
    lib = ctypes.CDLL(str(path))
    P = ctypes.POINTER
    lib.b2_engine_create.argtypes = [ctypes.c_char_p, P(EngineConfig), P(_vp)]
    lib.b2_engine_create_synthetic.argtypes = [P(ModelShape), ctypes.c_uint64, ctypes.c_float, P(EngineConfig),
                                               P(_vp)]
    lib.b2_engine_destroy.argtypes = [_vp]
    lib.b2_engine_destroy.restype = None
    lib.b2_engine_add_sequence.argtypes = [_vp, P(_i32), _i32]
    lib.b2_engine_add_sequence_cached.argtypes = [_vp, _i32, _i32]
    lib.b2_engine_decode_step.argtypes = [_vp, P(_i32), _i32, P(_i32)]
    lib.b2_engine_free_sequence.argtypes = [_vp, _i32]
    lib.b2_engine_free_blocks.argtypes = [_vp]
    lib.b2_engine_free_blocks.restype = ctypes.c_int64
    lib.b2_engine_set_use_cuda_graphs.argtypes = [_vp, _i32]
    lib.b2_engine_set_prefill_tensor_cores.argtypes = [_vp, _i32]
    lib.b2_engine_shape.argtypes = [_vp, P(ModelShape)]
    lib.b2_engine_stream.argtypes = [_vp, P(_vp)]
    lib.b2_engine_last_error.restype = ctypes.c_char_p
    lib.b2_block_pool_create.argtypes = [_i32]
    lib.b2_block_pool_create.restype = _vp
    lib.b2_block_pool_destroy.argtypes = [_vp]
    lib.b2_block_pool_destroy.restype = None
    lib.b2_block_pool_allocate.argtypes = [_vp]
    lib.b2_block_pool_free.argtypes = [_vp, _i32]
    lib.b2_block_pool_num_free.argtypes = [_vp]
    lib.b2_engine_tp_handle.argtypes = [_vp, ctypes.c_char_p]
    lib.b2_engine_tp_connect.argtypes = [_vp, ctypes.c_char_p]
    lib.b2_engine_prefill.argtypes = [_vp, P(_i32), _i32, P(_i32)]
    lib.b2_engine_tp_nccl_id.argtypes = [ctypes.c_char_p]
    lib.b2_engine_set_linear_tensor_cores.argtypes = [_vp, _i32]
    lib.b2_engine_last_step_outputs.argtypes = [_vp, _i32, _vp, _vp]
    lib.b2_engine_set_gemm_mode.argtypes = [_vp, _i32]
    lib.b2_engine_set_lm_head_fused.argtypes = [_vp, _i32]
    lib.b2_engine_tp_connect_nccl.argtypes = [_vp, ctypes.c_char_p]
    _lib = lib
    return lib


def _check(rc: int) -> None:
    if rc != 0:
        raise B2Error(rc, load().b2_engine_last_error().decode())


def _ints(values: Sequence[int]):
    arr = (_i32 * max(1, len(values)))()
    for i, v in enumerate(values):
        arr[i] = int(v)
    return arr


@dataclass
class Config:
    """EngineConfig (engine_api.h:9-13) with the reference's defaults."""
    max_batch: int = 8
    max_seq_len: int = 1024
    kv_block_budget: int = 4096
    dtype: int = F16
    use_cuda_graphs: bool = True
    device: int = -1
    tp_rank: int = 0   # head-sharded engines: this rank
    tp_size: int = 1   # > 1: heads split over tp_size GPUs (see include/b2_engine.h)
    max_prefill_tokens: int = 0  # prompt tokens per prefill call; 0 = 2048
    tp_allgather: int = 0  # head-sharded: 0 peer stores fused into attention, 1 ncclAllGather

    def to_c(self) -> EngineConfig:
        return EngineConfig(self.max_batch, self.max_seq_len, self.kv_block_budget, self.dtype,
                            1 if self.use_cuda_graphs else 0, self.device, self.tp_rank, self.tp_size,
                            self.max_prefill_tokens, self.tp_allgather)


class Engine:
    """The reference Engine's calls over b2_engine_* (engine.cu:240-388)."""

    def __init__(self) -> None:
        self._h = None
        self.cfg = None
        self._lib = load()

    def init(self, weights_dir: str | Path, cfg: Config) -> bool:
        """Engine::init: False (and last_error()) on failure, like the reference."""
        self.close()
        h = _vp()
        rc = self._lib.b2_engine_create(str(weights_dir).encode(), ctypes.byref(cfg.to_c()), ctypes.byref(h))
        if rc != 0:
            return False
        self._h = h
        self.cfg = cfg
        return True

    def init_synthetic(self, shape: ModelShape, cfg: Config, seed: int = 0, std: float = 0.02) -> None:
        self.close()
        h = _vp()
        _check(self._lib.b2_engine_create_synthetic(ctypes.byref(shape), seed, std, ctypes.byref(cfg.to_c()),
                                                    ctypes.byref(h)))
        self._h = h
        self.cfg = cfg

    def last_error(self) -> str:
        return self._lib.b2_engine_last_error().decode()

    def _handle(self):
        if self._h is None:
            raise RuntimeError("engine is not initialised")
        return self._h

    def add_sequence(self, prompt: Sequence[int]) -> int:
        rc = self._lib.b2_engine_add_sequence(self._handle(), _ints(prompt), len(prompt))
        if rc < -1:
            _check(rc)
        return rc

    def add_sequence_cached(self, ctx_len: int, last_token: int) -> int:
        rc = self._lib.b2_engine_add_sequence_cached(self._handle(), ctx_len, last_token)
        if rc < -1:
            _check(rc)
        return rc

    def decode_step(self, seq_ids: Sequence[int]) -> list[int]:
        out = (_i32 * max(1, len(seq_ids)))()
        _check(self._lib.b2_engine_decode_step(self._handle(), _ints(seq_ids), len(seq_ids), out))
        return list(out[:len(seq_ids)])

    def prefill(self, seq_ids: Sequence[int]) -> list[int]:
        """Batched prefill: every remaining prompt token of each sequence in one
        pass; returns each sequence's first generated token."""
        out = (_i32 * max(1, len(seq_ids)))()
        _check(self._lib.b2_engine_prefill(self._handle(), _ints(seq_ids), len(seq_ids), out))
        return list(out[:len(seq_ids)])

    def free_sequence(self, seq_id: int) -> None:
        _check(self._lib.b2_engine_free_sequence(self._handle(), seq_id))

    def free_blocks(self) -> int:
        return int(self._lib.b2_engine_free_blocks(self._handle()))

    def set_use_cuda_graphs(self, enabled: bool) -> None:
        _check(self._lib.b2_engine_set_use_cuda_graphs(self._handle(), 1 if enabled else 0))

    def last_step_outputs(self, rows: int):
        """(final LayerNorm rows [rows, d_model], logits [rows, vocab]) of the last
        decode_step as numpy arrays in the engine dtype (uint16 bit patterns for
        f16 / bf16)."""
        import numpy as np
        s = self.shape()
        dt = np.float32 if self.cfg.dtype == 0 else np.uint16
        h = np.empty((rows, s.d_model), dtype=dt)
        lg = np.empty((rows, s.vocab_size), dtype=dt)
        _check(self._lib.b2_engine_last_step_outputs(self._handle(), rows, h.ctypes.data, lg.ctypes.data))
        return h, lg

    def set_gemm_mode(self, mode: int) -> None:
        """Bit 1: cuBLASLt with timed algorithm choice; bit 2: FC bias + GELU in its epilogue."""
        _check(self._lib.b2_engine_set_gemm_mode(self._handle(), mode))

    def set_lm_head_fused(self, enabled: bool) -> None:
        """b2_engine_set_lm_head_fused: lm_head GEMM + argmax in one tensor-core launch (f16 / bf16)."""
        _check(self._lib.b2_engine_set_lm_head_fused(self._handle(), 1 if enabled else 0))

    def set_linear_tensor_cores(self, enabled: bool) -> None:
        _check(self._lib.b2_engine_set_linear_tensor_cores(self._handle(), 1 if enabled else 0))

    def set_prefill_tensor_cores(self, enabled: bool) -> None:
        _check(self._lib.b2_engine_set_prefill_tensor_cores(self._handle(), 1 if enabled else 0))

    def tp_handle(self) -> bytes:
        """This head-sharded rank's IPC handles, to be shared with every rank."""
        buf = ctypes.create_string_buffer(TP_HANDLE_BYTES)
        _check(self._lib.b2_engine_tp_handle(self._handle(), buf))
        return buf.raw

    @staticmethod
    def tp_nccl_id() -> bytes:
        """A new NCCL unique id (one rank makes it, every rank connects with it)."""
        buf = ctypes.create_string_buffer(TP_NCCL_ID_BYTES)
        _check(load().b2_engine_tp_nccl_id(buf))
        return buf.raw

    def tp_connect_nccl(self, nccl_id: bytes) -> None:
        """Joins the NCCL communicator of the head-sharded ranks (tp_allgather = 1)."""
        if len(nccl_id) != TP_NCCL_ID_BYTES:
            raise ValueError("the NCCL id is TP_NCCL_ID_BYTES bytes")
        _check(self._lib.b2_engine_tp_connect_nccl(self._handle(), nccl_id))

    def tp_connect(self, handles: Sequence[bytes]) -> None:
        """Maps every rank's buffers (handles in rank order, this rank's included)."""
        blob = b"".join(handles)
        if any(len(h) != TP_HANDLE_BYTES for h in handles):
            raise ValueError("each handle is TP_HANDLE_BYTES bytes")
        _check(self._lib.b2_engine_tp_connect(self._handle(), blob))

    def shape(self) -> ModelShape:
        s = ModelShape()
        _check(self._lib.b2_engine_shape(self._handle(), ctypes.byref(s)))
        return s

    def stream_handle(self) -> int:
        p = _vp()
        _check(self._lib.b2_engine_stream(self._handle(), ctypes.byref(p)))
        return p.value or 0

    def close(self) -> None:
        if self._h is not None:
            self._lib.b2_engine_destroy(self._h)
            self._h = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


class BlockPool:
    """The engine's block allocator (block_pool.h), reference BlockPool semantics."""

    def __init__(self, num_blocks: int) -> None:
        self._lib = load()
        self._h = self._lib.b2_block_pool_create(num_blocks)
        if not self._h:
            raise ValueError("num_blocks must be >= 0")

    def allocate(self) -> int:
        return int(self._lib.b2_block_pool_allocate(self._h))

    def free(self, block_id: int) -> None:
        rc = self._lib.b2_block_pool_free(self._h, block_id)
        if rc == 1:
            raise IndexError(f"block id {block_id} out of range")
        if rc == 2:
            raise RuntimeError(f"block id {block_id} is not allocated")

    def num_free(self) -> int:
        return int(self._lib.b2_block_pool_num_free(self._h))

    def __del__(self) -> None:
        h, self._h = getattr(self, "_h", None), None
        if h:
            self._lib.b2_block_pool_destroy(h)
