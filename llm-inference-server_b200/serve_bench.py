"""Continuous-batching serving benchmark over the engine (GPT-2 medium shape).

Replays the loop of the reference's ContinuousBatchScheduler
(cpp-engine/src/scheduler.cpp:48-73): admit waiting requests into free batch
slots, prefill the newly admitted ones, one decode step for every running
sequence, evict the finished ones -- driving the engine the way
GpuEngineGenerator does (cpp-engine/src/gpu_engine_generator.cpp:16-56).

Two prefill modes on the same request trace:
  * "token": every new prompt is walked token by token through decode_step at
    batch 1, inside the scheduler's prefill phase -- the reference's behaviour;
  * "batched": the new prompts of an iteration go through b2_engine_prefill
    in one pass (split by max_prefill_tokens).

Traffic (the serving config): Poisson arrivals at 50 requests/s, prompt lengths
U[32, 512] (token ids uniform), output lengths U[16, 512], max batch 128, block
16, GPT-2 medium shape (24 layers, 16 heads, d_model 1024) fp16 with weights
N(0, 0.02) drawn on the device.  eos_token_id is -1, so every request runs to
its output length.  Reported: output tokens/s over the whole run (first
arrival to last completion) and time-to-first-token percentiles.
"""
from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field

import numpy as np

from . import F16


@dataclass
class Request:
    arrival: float
    prompt: list
    out_len: int
    first_token: float = -1.0
    done: float = -1.0
    generated: list = field(default_factory=list)


def make_trace(n: int, rate: float = 50.0, seed: int = 7, vocab: int = 50257, prompt_lo: int = 32,
               prompt_hi: int = 512, out_lo: int = 16, out_hi: int = 512) -> list[Request]:
    rng = np.random.Generator(np.random.PCG64(seed))
    gaps = rng.exponential(1.0 / rate, size=n)
    arrivals = np.cumsum(gaps) - gaps[0]
    reqs = []
    for i in range(n):
        plen = int(rng.integers(prompt_lo, prompt_hi + 1))
        reqs.append(Request(float(arrivals[i]), rng.integers(0, vocab, size=plen).tolist(),
                            int(rng.integers(out_lo, out_hi + 1))))
    return reqs


def serve(eng, reqs: list[Request], mode: str, max_batch: int = 128, max_prefill_tokens: int = 4096) -> dict:
    """Runs the scheduler loop over `reqs` (arrival times relative to start)."""
    waiting: deque[int] = deque()
    active: dict[int, int] = {}   # engine sequence id -> request index
    state: dict[int, str] = {}    # engine sequence id -> "prefill" | "decode"
    nxt, finished = 0, 0
    t0 = time.perf_counter()
    steps = 0
    while finished < len(reqs):
        now = time.perf_counter() - t0
        while nxt < len(reqs) and reqs[nxt].arrival <= now:
            waiting.append(nxt)
            nxt += 1
        if not active and not waiting:
            time.sleep(max(0.0, min(0.001, reqs[nxt].arrival - now)))
            continue
        # admit
        while waiting and len(active) < max_batch:
            r = waiting.popleft()
            sid = eng.add_sequence(reqs[r].prompt)
            if sid < 0:
                waiting.appendleft(r)
                break
            active[sid] = r
            state[sid] = "prefill"
        # prefill
        new = [sid for sid in active if state[sid] == "prefill"]
        if new:
            if mode == "batched":
                chunk, budget = [], 0
                groups = []
                for sid in new:
                    plen = len(reqs[active[sid]].prompt)
                    if chunk and budget + plen > max_prefill_tokens:
                        groups.append(chunk)
                        chunk, budget = [], 0
                    chunk.append(sid)
                    budget += plen
                groups.append(chunk)
                firsts = {}
                for g in groups:
                    firsts.update(zip(g, eng.prefill(g)))
            else:
                firsts = {}
                for sid in new:
                    tok = 0
                    for _ in reqs[active[sid]].prompt:
                        tok = eng.decode_step([sid])[0]
                    firsts[sid] = tok
            now = time.perf_counter() - t0
            for sid in new:
                req = reqs[active[sid]]
                req.generated.append(firsts[sid])
                req.first_token = now
                state[sid] = "decode"
        # decode
        dec = [sid for sid in active if state[sid] == "decode" and len(reqs[active[sid]].generated) <
               reqs[active[sid]].out_len]
        if dec:
            toks = eng.decode_step(dec)
            steps += 1
            for sid, tok in zip(dec, toks):
                reqs[active[sid]].generated.append(tok)
        # evict
        now = time.perf_counter() - t0
        for sid in list(active):
            req = reqs[active[sid]]
            if state[sid] == "decode" and len(req.generated) >= req.out_len:
                req.done = now
                eng.free_sequence(sid)
                del active[sid], state[sid]
                finished += 1
    makespan = max(r.done for r in reqs) - reqs[0].arrival
    ttft = np.array([r.first_token - r.arrival for r in reqs])
    out_tokens = sum(r.out_len for r in reqs)
    return {"mode": mode, "requests": len(reqs), "output_tokens": out_tokens, "makespan_s": round(makespan, 3),
            "output_tok_s": round(out_tokens / makespan, 1), "ttft_p50_ms": round(float(np.percentile(ttft, 50)) * 1e3, 2),
            "ttft_p99_ms": round(float(np.percentile(ttft, 99)) * 1e3, 2), "decode_steps": steps}


def run(n_requests: int, n_compare: int, device_index: int = 0) -> dict:
    """Batched prefill on the whole trace, then both modes on its first
    n_compare requests (token-by-token prefill is far slower), each on a fresh
    engine."""
    from . import engine as E
    shape = E.ModelShape(n_layer=24, n_head=16, d_model=1024, vocab_size=50257, n_ctx=1024, layer_norm_epsilon=1e-5,
                         eos_token_id=-1)
    cfg = E.Config(max_batch=128, max_seq_len=1024, kv_block_budget=128 * 64 + 64, dtype=F16, use_cuda_graphs=True,
                   device=device_index, max_prefill_tokens=4096)
    out = {}
    for key, mode, n in (("batched", "batched", n_requests), ("batched_small", "batched", n_compare),
                         ("token_small", "token", n_compare)):
        eng = E.Engine()
        eng.init_synthetic(shape, cfg, seed=3, std=0.02)
        serve(eng, make_trace(4, seed=99), "batched")  # capture graphs and warm the prefill path
        out[key] = serve(eng, make_trace(n), mode)
        eng.close()
    return out
