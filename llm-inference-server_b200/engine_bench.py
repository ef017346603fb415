"""GPT-2 decode throughput (tokens/s) through the engine's public API.

Used by bench.py for its engine workloads.  One step = one
b2_engine_decode_step over every running sequence of a wave: host block-table
build, one upload, the captured CUDA graph of the whole model step (embedding,
48 x [LN, QKV GEMM, KV append, paged attention, proj GEMM, LN, FC GEMM,
GELU, FC-proj GEMM], final LN, lm_head GEMM, argmax), the download of the
next tokens and a stream synchronisation -- the reference's
Engine::decode_step (gpu-engine/src/engine.cu:309-377).

GPT-2 XL shape (48 layers, 25 heads, d_model 1600, vocab 50257, n_ctx 1024),
bf16, weights N(0, 0.02) drawn on the device, global batch 1024 sequences
whose cached contexts are uniform in [256, 1024 - steps] (positions stay
below n_ctx); the cached keys and values are N(0, 1).  Sequences are sharded
over the ranks (one engine and one KV pool per GPU, no collective on the data
path).  A rank whose share of the KV cache would not fit next to the weights
runs its sequences in waves of at most 512 (one GPU: 2 waves).
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass

import numpy as np

from . import BF16, F16, F32, BLOCK_TOKENS


@dataclass(frozen=True)
class EngineWorkload:
    name: str
    n_layer: int
    n_head: int
    d_model: int
    vocab: int
    n_ctx: int
    dtype: int
    global_batch: int
    ctx_lo: int
    wave_cap: int
    description: str
    head_sharded: bool = False  # every rank holds every sequence and ceil(H / ranks) of the heads


ENGINE_WORKLOADS = {
    "gpt2-xl": EngineWorkload(
        "gpt2-xl", 48, 25, 1600, 50257, 1024, BF16, 1024, 256, 512,
        "GPT-2 XL-shaped decode: 48 layers, 25 heads, d_model 1600, head_dim 64, bf16, weights N(0,0.02); global "
        "batch 1024 sequences, cached contexts U[256, 1024-steps], KV N(0,1), block 16, sequence-sharded "
        "(one engine and KV pool per GPU), waves of <= 512 sequences per GPU"),
    "gpt2-medium": EngineWorkload(
        "gpt2-medium", 24, 16, 1024, 50257, 1024, F16, 128, 32, 128,
        "GPT-2 medium-shaped decode: 24 layers, 16 heads, d_model 1024, head_dim 64, fp16, weights N(0,0.02); "
        "batch 128 sequences per GPU, cached contexts U[32, 1024-steps], KV N(0,1), block 16"),
    "gpt2-xl-heads": EngineWorkload(
        "gpt2-xl-heads", 48, 25, 1600, 50257, 1024, BF16, 1024, 256, 1024,
        "GPT-2 XL-shaped decode, head-sharded: 48 layers, 25 heads split ceil(25/N) per GPU, d_model 1600, "
        "head_dim 64, bf16, weights N(0,0.02); global batch 1024 sequences on every GPU, cached contexts "
        "U[256, 1024-steps], KV N(0,1) (each GPU holds its heads' slice), attention output all-gathered in the "
        "attention epilogue over NVLink, flag barrier per layer; LN, projections, MLP and lm_head replicated",
        head_sharded=True),
}


def weight_elems(w: EngineWorkload) -> int:
    D, V, L = w.d_model, w.vocab, w.n_layer
    per_layer = 2 * D + 3 * D * D + 3 * D + D * D + D + 2 * D + 4 * D * D + 4 * D + 4 * D * D + D
    return V * D + w.n_ctx * D + L * per_layer + 2 * D


def elem_bytes(dt: int) -> int:
    return 4 if dt == F32 else 2


def step_bytes(w: EngineWorkload, ctx: np.ndarray, world: int = 1) -> float:
    """Algorithmic HBM bytes of one decode step (on one GPU) over sequences
    with cached contexts ctx (before the step): every weight it reads once,
    every cached K/V row of every layer once, the new K/V rows written once.
    A head-sharded GPU reads its QKV slice, a zero-padded output projection
    and the replicated rest, and only its heads' K/V."""
    es = elem_bytes(w.dtype)
    D, L = w.d_model, w.n_layer
    if w.head_sharded and world > 1:
        hd = D // w.n_head
        qd = -(-w.n_head // world) * hd  # this GPU's heads x head_dim
        weights = weight_elems(w) - L * (3 * D * D + 3 * D + D * D) + L * (3 * qd * D + 3 * qd + D * world * qd)
        kv_row = L * 2 * qd * es
    else:
        weights = weight_elems(w)
        kv_row = L * 2 * D * es
    return float(weights * es + (ctx.astype(np.float64) + 1).sum() * kv_row)


@dataclass(frozen=True)
class ShardPlan:
    """One rank's share of an engine workload."""
    sharded: bool    # head-sharded: every rank holds every sequence and a slice of the heads
    per_rank: int    # sequences this rank decodes
    wave: int        # sequences per wave (one engine batch)
    waves: int       # waves this rank runs one after the other
    seed: int        # contexts and last tokens of this rank's sequences
    token_div: int   # ranks that produce each of this rank's tokens (a head-sharded token counts once)

    def tokens(self, steps: int) -> float:
        """Tokens of the job this rank accounts for over `steps` steps of every wave."""
        return self.per_rank * steps / self.token_div


def shard_plan(w: EngineWorkload, rank: int, world: int, per_rank_batch: int | None = None) -> ShardPlan:
    """Sequence-sharded: the global batch split evenly, each rank its own
    sequences (its own seed); head-sharded: every rank the whole batch (the
    same seed on every rank) and its slice of the heads.  per_rank_batch
    overrides the sequences per rank (profiling one GPU's share of a larger
    job).  A rank runs its sequences in waves of at most w.wave_cap."""
    sharded = w.head_sharded and world > 1
    if w.head_sharded and world == 1:
        raise ValueError("the head-sharded workload needs 2 or more GPUs")
    if w.global_batch % world:
        raise ValueError(f"global batch {w.global_batch} does not split over {world} ranks")
    per_rank = w.global_batch if sharded else w.global_batch // world
    if per_rank_batch:
        per_rank = per_rank_batch
    wave = min(per_rank, w.wave_cap)
    return ShardPlan(sharded=sharded, per_rank=per_rank, wave=wave, waves=(per_rank + wave - 1) // wave,
                     seed=20_000 + (0 if sharded else rank), token_div=world if sharded else 1)


def run(w: EngineWorkload, steps: int, warmup: int, rank: int, world: int, dist, device, timed_region=None,
        per_rank_batch: int | None = None, allgather: int = 0, linear: bool = False, gemm_mode: int = 0) -> dict:
    """Runs the workload's waves on this rank; timed_region() (optional) gives a
    context manager entered around each wave's timed steps.  per_rank_batch
    overrides the sequences per rank (profiling one GPU's share of a larger
    job).  allgather (head-sharded only): 0 = the attention epilogue stores
    into every rank's gathered buffer over NVLink; 1 = ncclAllGather."""
    import torch

    from . import engine as E

    plan = shard_plan(w, rank, world, per_rank_batch)
    sharded, per_rank, wave, n_waves = plan.sharded, plan.per_rank, plan.wave, plan.waves
    total = warmup + steps
    if w.ctx_lo + total > w.n_ctx:
        raise ValueError("too many steps for the context range")
    rng = np.random.Generator(np.random.PCG64(plan.seed))
    ctx = rng.integers(w.ctx_lo, w.n_ctx - total + 1, size=per_rank)
    last_tok = rng.integers(0, w.vocab, size=per_rank)
    blocks_needed = max(int(((ctx[i:i + wave] + total + BLOCK_TOKENS - 1) // BLOCK_TOKENS).sum())
                        for i in range(0, per_rank, wave))
    shape = E.ModelShape(n_layer=w.n_layer, n_head=w.n_head, d_model=w.d_model, vocab_size=w.vocab, n_ctx=w.n_ctx,
                         layer_norm_epsilon=1e-5, eos_token_id=-1)
    eng = E.Engine()
    eng.init_synthetic(shape, E.Config(max_batch=wave, max_seq_len=w.n_ctx, kv_block_budget=blocks_needed + 64,
                                       dtype=w.dtype, use_cuda_graphs=True, device=device.index,
                                       tp_rank=rank if sharded else 0, tp_size=world if sharded else 1,
                                       tp_allgather=allgather if sharded else 0),
                       seed=1, std=0.02)
    if linear:
        eng.set_linear_tensor_cores(True)
    if gemm_mode:
        eng.set_gemm_mode(gemm_mode)
    if sharded and allgather:
        ids_box = [E.Engine.tp_nccl_id() if rank == 0 else None]
        dist.broadcast_object_list(ids_box, src=0)
        eng.tp_connect_nccl(ids_box[0])
    elif sharded:
        handles = [None] * world
        dist.all_gather_object(handles, eng.tp_handle())
        eng.tp_connect(handles)
    stream = torch.cuda.ExternalStream(eng.stream_handle(), device=device)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(device)

    timed_ms = 0.0
    bytes_timed = 0.0
    for wv in range(n_waves):
        lo, hi = wv * wave, min(per_rank, (wv + 1) * wave)
        ids = [eng.add_sequence_cached(int(ctx[i]), int(last_tok[i])) for i in range(lo, hi)]
        if min(ids) < 0:
            raise RuntimeError("KV pool exhausted while adding sequences")
        for _ in range(warmup):
            eng.decode_step(ids)
        barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with (timed_region() if timed_region else contextlib.nullcontext()):
            ev0.record(stream)
            for _ in range(steps):
                eng.decode_step(ids)
            ev1.record(stream)
            torch.cuda.synchronize(device)
        barrier()
        timed_ms += ev0.elapsed_time(ev1)
        c0 = ctx[lo:hi] + warmup
        bytes_timed += sum(step_bytes(w, c0 + s, world) for s in range(steps))
        for i in ids:
            eng.free_sequence(i)
    eng.close()
    return {"ms": timed_ms, "tokens": plan.tokens(steps), "bytes": bytes_timed, "waves": n_waves, "wave": wave,
            "per_rank": per_rank}
