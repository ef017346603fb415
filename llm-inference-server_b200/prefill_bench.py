"""Prefill throughput through the engine: prompt tokens per second of
b2_engine_prefill on a GPT-2 medium-shaped fp16 model (24 layers, 16 heads,
d_model 1024, weights N(0, 0.02) drawn on the device).

The reference has no batched prefill -- GpuEngineGenerator walks every prompt
token through Engine::decode_step at batch 1
(cpp-engine/src/gpu_engine_generator.cpp:28-42).  Two attention paths of the
same b2_engine_prefill call are timed on identical prompts:
  * "tensor_cores": b2_prefill_attention, 128-row query tiles on tcgen05;
  * "decode_rows":  one decode-attention row per prompt token (each row reads
                    its whole key prefix).
A step is one call over n_prompts fresh sequences of prompt_len uniform random
tokens; its time includes the host-side preparation, the upload, every
kernel, the download of the first generated tokens and the synchronisation
(the call blocks), i.e. it is measured end to end through the engine API.
"""
from __future__ import annotations

import time

import numpy as np

from . import F16

MEDIUM = dict(n_layer=24, n_head=16, d_model=1024, vocab_size=50257, n_ctx=1024, layer_norm_epsilon=1e-5,
              eos_token_id=-1)


def run(n_prompts: int = 8, prompt_len: int = 512, steps: int = 5, warmup: int = 3, device_index: int = 0,
        modes=("tensor_cores", "decode_rows")) -> dict:
    from . import engine as E
    shape = E.ModelShape(**MEDIUM)
    blocks_per_seq = (prompt_len + 16) // 16 + 1
    cfg = E.Config(max_batch=max(8, n_prompts), max_seq_len=shape.n_ctx,
                   kv_block_budget=n_prompts * blocks_per_seq + 16, dtype=F16, use_cuda_graphs=True,
                   device=device_index, max_prefill_tokens=n_prompts * prompt_len)
    eng = E.Engine()
    eng.init_synthetic(shape, cfg, seed=3, std=0.02)
    rng = np.random.Generator(np.random.PCG64(1))
    prompts = [rng.integers(0, shape.vocab_size, size=prompt_len).tolist() for _ in range(n_prompts)]
    out = {"n_prompts": n_prompts, "prompt_len": prompt_len, "steps": steps, "warmup": warmup}
    try:
        for mode in modes:
            eng.set_prefill_tensor_cores(mode == "tensor_cores")
            times = []
            for i in range(warmup + steps):
                ids = [eng.add_sequence(p) for p in prompts]
                t0 = time.perf_counter()
                eng.prefill(ids)
                dt = time.perf_counter() - t0
                for sid in ids:
                    eng.free_sequence(sid)
                if i >= warmup:
                    times.append(dt)
            ms = float(np.median(times)) * 1e3
            out[mode] = {"ms_per_call": round(ms, 3), "prompt_tok_s": round(n_prompts * prompt_len / ms * 1e3, 1)}
    finally:
        eng.close()
    return out
