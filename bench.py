#!/usr/bin/env python3
"""Paged-attention decode benchmark (HBM GB/s) and GPT-2 decode tokens/s for the sm_100a hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload mha|gqa|...]

One step = one paged-attention call over one batch.  The default run's line
also carries the GPT-2 XL-shaped decode step through the engine at the same N
(`gpt2_xl`: global batch 1024, sequence-sharded; at N >= 2 also
`gpt2_xl_heads`: head-sharded with the all-gather fused into the attention
epilogue and with ncclAllGather, plus a greedy-token check of both against one
GPU) and, at N = 1, the GPT-2 small fp32 greedy job with the reference's own
CPU path timed on the host cores (`gpt2_small`).  Workloads:

  mha (default, the headline): batch 64 per GPU, 12 heads, head_dim 64, fp16
      K/V and q ~ N(0,1) from a seed, context U[128,1024], block size 16,
      block tables from a random permutation of a 65536-block pool, scale 1/8,
      fp32 softmax.  Consecutive steps rotate through 16 disjoint input sets
      (~1.8 GB of KV) so no launch is served from the 126 MB L2.
  gqa: batch 256 per GPU, 32 query heads over 8 kv heads, head_dim 128, bf16
      K/V and q ~ N(0,1), context log-uniform in [512, 32768] (~7.2 GB of KV
      per launch, far larger than L2), pool of 140000 blocks; runs on the
      tensor-core kernel.

Under torchrun every rank runs its own batch stream on its own GPU (weak
scaling, no collective on the data path); the job's time is the max over
ranks.

The line also carries: the same metric end to end through the C-ABI with
host buffers (e2e), the roofline of the attention kernel against the measured
HBM copy bandwidth, the CPU baseline (the oracle's restatement of the
reference CPU attention, multi-threaded, on a bounded sample), clocks sampled
during the timed region, and the number of our kernel launches timed.

--impl reference times the reference's CPU implementation of the path (the
oracle restatement of gpu-engine/src/reference/cpu_model.cpp:131-162 through
the block table; the reference exposes no standalone attention call) on the
host cores, same metric and config.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import sys
import threading
import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged-attn decode HBM GB/s"
SPIN_CYCLES = 100_000  # ~0.05 ms at B200 clocks


@dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    n_head: int
    n_kv_head: int
    head_dim: int
    dtype: str          # "f16" | "bf16"
    ctx_lo: int
    ctx_hi: int
    log_uniform: bool
    n_sets: int
    pool_blocks: int
    profile: str        # committed ncu summary holding traffic_bytes_per_launch
    description: str
    layout: str = ""    # "blocks" / "layer-major": 48-layer KV cache, one launch per layer


WORKLOADS = {
    "mha": Workload("mha", 64, 12, 12, 64, "f16", 128, 1024, False, 16, 65536, "paged_decode_microbench.md",
                    "paged-attention decode microbench: batch 64 per GPU, 12 heads, head_dim 64, fp16 K/V and q "
                    "N(0,1), context U[128,1024], block 16, random permutation of a 65536-block pool, scale 1/8"),
    "mha-medium": Workload("mha-medium", 128, 16, 16, 64, "f16", 32, 1024, False, 16, 81920,
                           "paged_decode_medium_heads.md",
                           "paged-attention decode at the GPT-2 medium engine's shape: batch 128 per GPU, 16 heads, "
                           "head_dim 64, fp16 K/V and q N(0,1), context U[32,1024], block 16, random permutation of "
                           "an 81920-block pool, scale 1/8"),
    "gqa": Workload("gqa", 256, 32, 8, 128, "bf16", 512, 32768, True, 1, 140000, "paged_decode_tc_gqa.md",
                    "grouped-query paged-attention decode: batch 256 per GPU, 32 query / 8 kv heads, head_dim 128, "
                    "bf16 K/V and q N(0,1), context log-uniform [512,32768], block 16, random permutation of a "
                    "140000-block pool, scale 1/sqrt(128)"),
    "xl-blocks": Workload("xl-blocks", 128, 25, 25, 64, "bf16", 256, 1011, False, 48, 0, "",
                          "paged-attention decode over the reference's all-layers-per-block pool (kv_cache.h:6-8): "
                          "GPT-2 XL shape, batch 128, 25 heads x 64, bf16, 48 layers per 4.9 MB block, launch l reads "
                          "layer l, context U[256,1011], random block permutation", "blocks"),
    "xl-layers": Workload("xl-layers", 128, 25, 25, 64, "bf16", 256, 1011, False, 48, 0, "",
                          "paged-attention decode over the engine's layer-major KV cache: GPT-2 XL shape, batch 128, "
                          "25 heads x 64, bf16, one arena per layer (48), launch l reads layer l, context "
                          "U[256,1011], the same random block permutation", "layer-major"),
}
WL = WORKLOADS["mha"]  # set by main()


def import_package(name: str = "lis_b200"):
    import importlib.util
    if name in sys.modules:
        return sys.modules[name]
    pkg = ROOT / "llm-inference-server_b200"
    spec = importlib.util.spec_from_file_location(name, pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def workload_config(n_gpus: int, n_sets: int | None = None) -> dict:
    n_sets = WL.n_sets if n_sets is None else n_sets
    l2 = (f"inputs larger than L2: {n_sets} disjoint input sets rotated between launches" if n_sets > 1 else
          "inputs larger than L2: one input set of several GB per launch")
    return {"workload": WL.description, "name": WL.name, "global_batch": WL.batch * n_gpus, "accumulate": "f32",
            "out_dtype": WL.dtype, "l2": l2, "parallelism": f"sequence-sharded x{n_gpus}, no collective"}


def torch_dtype():
    import torch
    return torch.float16 if WL.dtype == "f16" else torch.bfloat16


def oracle_dtype():
    from oracle import oracle as O
    return O.F16 if WL.dtype == "f16" else O.BF16


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic():
    """dram bytes per launch of the attention kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / WL.profile
    if not WL.profile or not p.is_file():
        return None, None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
    n = re.search(r"algorithmic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
    return (float(m.group(1)) if m else None), (float(n.group(1)) if n else None)


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """Samples SM clock and clock-event reasons with NVML while running."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.idx, self.period = device_index, period_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.error = None

    def __enter__(self):
        if self.idx < 0:  # no sampling
            return self
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def run():
                while not self._stop.is_set():
                    try:
                        mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((mhz, rs))
                    except Exception as e:  # noqa: BLE001
                        self.error = str(e)
                        return
                    time.sleep(self.period)

            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
        except Exception as e:  # noqa: BLE001
            self.error = str(e)
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "note": self.error or "no samples"}
        mhz = sorted(s[0] for s in self.samples)
        bits = 0
        for _, r in self.samples:
            bits |= r
        reasons = [n for b, n in self.REASONS.items() if bits & b and b != 0x1]
        return {"sm_mhz": mhz[len(mhz) // 2], "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


# --------------------------------------------------------------- CPU legs

def cpu_sample_seqs():
    """Sequences of input set 0 the CPU legs start from: the whole mha batch;
    16 sequences of the gqa batch (~0.5 GB of KV; the whole batch holds ~7 GB)."""
    return None if WL.name == "mha" else 16


def cpu_call(O, q, pool, bt, ctx, nthreads):
    O.paged_attention(oracle_dtype(), q, WL.n_head * WL.head_dim, pool, bt, ctx, n_head=WL.n_head,
                      n_kv_head=WL.n_kv_head, head_dim=WL.head_dim, max_blocks_per_seq=bt.shape[1], layer_idx=0,
                      n_layer=1, nthreads=nthreads)


def call_bytes(ctx) -> int:
    from lis_b200.workloads import attention_bytes
    return attention_bytes(ctx, WL.n_head, WL.n_kv_head, WL.head_dim, 2, 2, 2)


def cpu_attention_rate(wl, budget_s: float, nthreads: int):
    """Times the oracle restatement of the reference CPU attention on a host
    copy of (part of) input set 0."""
    from oracle import oracle as O
    pool, bt, ctx, q = host_subset(wl, 0, cpu_sample_seqs())
    nbytes = call_bytes(ctx)
    reps, t0 = 0, time.perf_counter()
    while True:
        cpu_call(O, q, pool, bt, ctx, nthreads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return nbytes * reps / el / 1e9, reps, len(ctx), nbytes, el


def host_subset(wl, i, n_seq):
    from lis_b200.workloads import host_subset as hs
    return hs(wl, i, n_seq)


# ------------------------------------------------------------------ arms

def run_reference_arm(args, rank: int, world: int) -> None:
    """CPU reference arm: rank 0 only."""
    if rank != 0:
        return
    import torch
    from oracle import oracle as O
    b2 = import_package()
    O.load()
    nthreads = os.cpu_count() or 1
    # Inputs are generated exactly as for the GPU arm (host copy of input set 0).
    if torch.cuda.is_available():
        wl = b2_workload(b2, torch.device("cuda:0"), seed=0, n_sets=1, pool_blocks=WL.pool_blocks)
        pool, bt, ctx, q = host_subset(wl, 0, cpu_sample_seqs())
        n_batch = wl.batch
        del wl
        torch.cuda.empty_cache()
    else:
        pool, bt, ctx, q = host_workload(seed=0, n_seq=cpu_sample_seqs())
        n_batch = WL.batch
    nbytes_full = call_bytes(ctx)
    t0 = time.perf_counter()
    cpu_call(O, q, pool, bt, ctx, nthreads)
    t_full = time.perf_counter() - t0
    # Size each step so K+W steps stay within ~2 minutes.
    n_seq = len(ctx)
    budget = 120.0
    if (args.steps + args.warmup) * t_full > budget:
        n_seq = max(1, int(len(ctx) * budget / ((args.steps + args.warmup) * t_full)))
    row = WL.n_head * WL.head_dim
    ctx_s, bt_s, q_s = ctx[:n_seq], bt[:n_seq], q[: n_seq * row]
    nbytes = call_bytes(ctx_s)
    for _ in range(args.warmup):
        cpu_call(O, q_s, pool, bt_s, ctx_s, nthreads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_call(O, q_s, pool, bt_s, ctx_s, nthreads)
    el = time.perf_counter() - t0
    value = nbytes * args.steps / el / 1e9
    sample = (f"{n_seq} of the {n_batch} sequences of one batch per step ({nbytes / 1e6:.1f} MB of KV; the first "
              f"{len(ctx)} sequences hold {nbytes_full / 1e6:.1f} MB), oracle port of cpu_model.cpp:131-162 "
              f"through the block table")
    line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": WL.dtype, "data": "synthetic",
            "config": workload_config(1),
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": nthreads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def host_workload(seed: int, n_seq=None):
    """Host-only generation of one batch, or its first n_seq sequences (used
    when no GPU is present)."""
    from oracle import oracle as O
    rng = np.random.Generator(np.random.PCG64(seed))
    if WL.log_uniform:
        ctx = np.exp(rng.uniform(np.log(WL.ctx_lo), np.log(WL.ctx_hi), size=WL.batch)).astype(np.int32)
    else:
        ctx = rng.integers(WL.ctx_lo, WL.ctx_hi + 1, size=WL.batch).astype(np.int32)
    ctx = ctx[:n_seq] if n_seq else ctx
    nb = (ctx + 15) // 16
    bt = np.zeros((len(ctx), (WL.ctx_hi + 15) // 16), np.int32)
    o = 0
    for b in range(len(ctx)):
        bt[b, : nb[b]] = np.arange(o, o + nb[b])
        o += int(nb[b])
    dt = oracle_dtype()
    pool = O.round_to(dt, rng.standard_normal(o * 2 * 16 * WL.n_kv_head * WL.head_dim, dtype=np.float32))
    q = O.round_to(dt, rng.standard_normal(len(ctx) * WL.n_head * WL.head_dim, dtype=np.float32))
    return pool, bt, ctx, q


def b2_workload(b2, device, seed: int, n_sets: int, pool_blocks: int, batch: int | None = None):
    from lis_b200.workloads import make_attention_workload, make_layered_workload
    if WL.layout:
        return make_layered_workload(device, WL.layout, seed=seed, batch=batch or WL.batch, n_head=WL.n_head,
                                     head_dim=WL.head_dim, ctx_lo=WL.ctx_lo, ctx_hi=WL.ctx_hi, n_layer=WL.n_sets,
                                     dtype=torch_dtype())
    return make_attention_workload(device, seed=seed, n_sets=n_sets, batch=batch or WL.batch, n_head=WL.n_head,
                                   n_kv_head=WL.n_kv_head, head_dim=WL.head_dim, ctx_lo=WL.ctx_lo, ctx_hi=WL.ctx_hi,
                                   pool_blocks=pool_blocks, dtype=torch_dtype(), log_uniform=WL.log_uniform)


def reduce_over_ranks(dist, x: float, op: str, device) -> float:
    """x combined over every rank ("max" or "sum"); x itself without a process
    group.  The tensor lives on `device` (CUDA for NCCL, CPU for gloo).  Every
    rank must make the same calls in the same order."""
    if dist is None:
        return x
    import torch
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "sum": dist.ReduceOp.SUM}[op])
    return float(t.item())


def job_rate(dist, units: float, ms: float, device) -> tuple[float, float, float]:
    """Whole-job throughput of a weak- or strong-scaled run: (units of all
    ranks, the slowest rank's time in ms, units per second)."""
    total = reduce_over_ranks(dist, units, "sum", device)
    t_max = reduce_over_ranks(dist, ms, "max", device)
    return total, t_max, total / (t_max * 1e-3)


def run_ours(args, rank: int, world: int, dist) -> dict | None:
    import torch
    b2 = import_package()
    b2.load()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    wl = b2_workload(b2, dev, seed=1000 + rank, n_sets=args.sets or WL.n_sets,
                     pool_blocks=args.pool_blocks or WL.pool_blocks, batch=args.batch)
    # A non-default stream (graph capture needs one) that every torch op below uses too.
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    wl.workspace = b2.attention_workspace(wl.sets[0].args)
    ws = wl.workspace
    lib = b2.load()
    import ctypes
    ws_ptr, ws_n, sptr = ws.data_ptr(), ws.numel(), stream.cuda_stream
    arg_refs = [ctypes.byref(s.args) for s in wl.sets]
    nsets = len(wl.sets)

    def launch(i):
        rc = lib.b2_paged_attention(arg_refs[i % nsets], ws_ptr, ws_n, sptr)
        if rc != 0:
            raise RuntimeError(f"b2_paged_attention failed: {rc} {lib.b2_last_error_string().decode()}")

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x: float) -> float:
        return reduce_over_ranks(dist, x, "max", dev)

    def sum_over_ranks(x: float) -> float:
        return reduce_over_ranks(dist, x, "sum", dev)

    # --------------------------------------------------- device-resident timing
    # The launches are replayed from a CUDA graph holding one launch per input
    # set (the way a serving engine replays a captured decode step), so the
    # host's launch rate does not enter the kernel timing.  Every input is
    # written before the timed region, so the launches carry
    # B2_ATTN_INPUTS_READY (each may start streaming while the one before it
    # finishes); the same launches with flags 0 are timed too (value_flags0).
    def set_flags(f, cap=0):
        for s_ in wl.sets:
            s_.args.flags = f
            s_.args.max_ctas = cap

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                launch(i)
        return g

    def timed_replay(flags, steps, sampler=None, cap=0):
        # Every timed launch comes from a graph, so no host launch (and its
        # ~µs of Python overhead) sits in the timed region: up to 256 steps
        # one graph of exactly `steps` launches (the input sets in rotation,
        # as a decode step's graph holds one launch per layer); beyond that a
        # graph of 256 launches replayed, and one for the remainder.
        set_flags(flags, cap)
        for i in range(args.warmup):
            launch(i)
        torch.cuda.synchronize(dev)
        chunk = nsets * max(1, 256 // nsets)
        if steps <= chunk:
            full_reps, rem = 1, 0
            chunk = steps
        else:
            full_reps, rem = divmod(steps, chunk)
        graph = capture(chunk)
        graph_rem = capture(rem) if rem else None
        graph.replay()
        if graph_rem is not None:
            graph_rem.replay()
        barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with (sampler if sampler is not None else ClockSampler(-1)) as clk_:
            # a short device-side spin ahead of the start event, so the host's
            # graph launch (several µs) is not inside the timed region: the
            # region holds exactly the `steps` launches
            torch.cuda._sleep(SPIN_CYCLES)
            ev0.record(stream)
            for _ in range(full_reps):
                graph.replay()
            if graph_rem is not None:
                graph_rem.replay()
            ev1.record(stream)
            torch.cuda.synchronize(dev)
        barrier()
        del graph, graph_rem
        return ev0.elapsed_time(ev1), clk_

    strict_steps = min(args.steps, 2000)
    ms0, _ = timed_replay(0, strict_steps)
    value_flags0 = sum_over_ranks(float(sum(wl.sets[i % nsets].bytes for i in range(strict_steps)))) / (
        max_over_ranks(ms0) * 1e-3) / 1e9
    # Pipelined launches: every input written before the timed region
    # (B2_ATTN_INPUTS_READY) and max_ctas = one CTA per SM, so each launch
    # leaves every SM's second CTA slot to the launch after it -- consecutive
    # launches stream side by side instead of one waiting for the other's
    # slots (the value line).  value_flags0 above: each launch waits for the
    # previous one, full grid.
    # Which grid pipelines better depends on the shape (the one-CTA-per-SM grid
    # needs the kernel's shared-memory stash for a CTA's first piece), so both
    # are timed and the faster is the value; both figures go into the line.
    n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
    by_grid = {}
    for cap in (n_sm, 0):
        ms_c, clk_c = timed_replay(b2.ATTN_INPUTS_READY, args.steps, ClockSampler(dev.index), cap=cap)
        by_grid[cap] = (max_over_ranks(ms_c), ms_c, clk_c)
    best_cap = min(by_grid, key=lambda c: by_grid[c][0])
    _, ms, clk = by_grid[best_cap]
    set_flags(0)  # the e2e loop below rewrites inputs every step
    my_bytes = sum(wl.sets[i % nsets].bytes for i in range(args.steps))
    t_max = by_grid[best_cap][0]
    tot_bytes = sum_over_ranks(float(my_bytes))
    sum_bytes_steps = tot_bytes
    value = tot_bytes / (t_max * 1e-3) / 1e9
    errs = b2.device_errors()

    # ------------------------------------------------ end to end through the C-ABI
    # Per step, like Engine::decode_step (gpu-engine/src/engine.cu:343-368): upload
    # q, block tables and seq_lens from pinned host memory, launch, download the
    # output, synchronise -- one b2_paged_attention_host call (the inputs are
    # pinned, so a small kernel reads them over PCIe into the device buffer,
    # rewritten every step; the output buffer is pinned, so the attention
    # kernel stores into it over PCIe).  Each input set's q | block tables |
    # seq_lens sit back to back in one pinned host buffer and in one device
    # buffer.  The KV cache stays resident (it is the engine's state).
    layouts, host_in = [], []
    for s_ in wl.sets:
        qh = s_.d_q.cpu().contiguous().view(torch.uint8).reshape(-1)
        bth = torch.from_numpy(np.ascontiguousarray(s_.block_tables, np.int32)).view(torch.uint8).reshape(-1)
        slh = torch.from_numpy(np.ascontiguousarray(s_.seq_lens, np.int32)).view(torch.uint8).reshape(-1)
        buf = torch.cat([qh, bth, slh]).pin_memory()
        layouts.append((qh.numel(), bth.numel(), slh.numel()))
        host_in.append(buf)
    d_in = torch.empty(max(sum(l_) for l_ in layouts), dtype=torch.uint8, device=dev)
    d_out = torch.empty_like(wl.sets[0].d_out)
    hout = torch.empty_like(d_out, device="cpu").pin_memory()
    e2e_args, e2e_io = [], []
    for s_, (qb, btb, slb), hb in zip(wl.sets, layouts, host_in):
        a_ = type(s_.args).from_buffer_copy(s_.args)
        a_.q, a_.block_tables, a_.seq_lens = d_in.data_ptr(), d_in.data_ptr() + qb, d_in.data_ptr() + qb + btb
        a_.out, a_.flags = d_out.data_ptr(), 0
        e2e_args.append(a_)
        e2e_io.append(b2.AttnHostIO(hb.data_ptr(), hb.data_ptr() + qb, hb.data_ptr() + qb + btb, hout.data_ptr()))
    e2e_refs = [(ctypes.byref(a_), ctypes.byref(io_)) for a_, io_ in zip(e2e_args, e2e_io)]
    h2d = sum(layouts[0])
    d2h = hout.numel() * hout.element_size()

    def e2e_step(i):
        ar, ior = e2e_refs[i % nsets]
        rc = lib.b2_paged_attention_host(ar, ior, ws_ptr, ws_n, sptr)
        if rc != 0:
            raise RuntimeError(f"b2_paged_attention_host failed: {rc} {lib.b2_last_error_string().decode()}")

    e2e_steps = min(args.steps, 2000)
    for i in range(max(3, args.warmup)):
        e2e_step(i)
    barrier()
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev2.record(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    ev3.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = max_over_ranks(ev2.elapsed_time(ev3))
    e2e_bytes = sum_over_ranks(float(sum(wl.sets[i % nsets].bytes for i in range(e2e_steps))))
    e2e_value = e2e_bytes / (e2e_ms * 1e-3) / 1e9
    # the last host-side output against the device-resident launch of the same set
    last = wl.sets[(e2e_steps - 1) % nsets]
    torch.cuda.synchronize(dev)
    e2e_match = float((hout.float() - last.d_out.float().cpu()).abs().max())

    # --------------------------------------------------------------- CPU baseline
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        nthreads = os.cpu_count() or 1
        gbs, reps, nseq, nbytes, el = cpu_attention_rate(wl, args.cpu_seconds, nthreads)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": nthreads, "kind": "port",
               "sample": f"input set 0 ({nseq} sequences, {nbytes / 1e6:.1f} MB KV) x {reps} passes in {el:.1f} s; "
                         f"oracle restatement of cpu_model.cpp:131-162 through the block table"}

    if rank != 0:
        return
    peak, peak_kind = measured_peak()
    per_launch_bytes = my_bytes / args.steps
    per_launch_s = ms * 1e-3 / args.steps
    achieved = per_launch_bytes / per_launch_s / 1e9
    traffic, traffic_alg = profiled_traffic()
    tc_path = (WL.n_kv_head == 8 and WL.head_dim == 128 and
               not os.environ.get("B2_ATTENTION_TENSOR_CORES", "1").startswith("0"))
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(t_max / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": WL.dtype, "data": "synthetic",
        "config": workload_config(world, len(wl.sets)),
        "pct_of_peak": round(100.0 * value / (peak * world), 2),
        "flags": "B2_ATTN_INPUTS_READY (inputs are written before the timed region), "
                 + (f"max_ctas = {n_sm} (one CTA per SM: consecutive launches share every SM)" if best_cap else
                    "the planner's grid") + "; value_flags0: flags 0, full grid, each launch waits for the one before",
        "value_by_grid": {("one_cta_per_sm" if c else "planner_grid"): round(
            sum_bytes_steps / (v[0] * 1e-3) / 1e9, 2) for c, v in by_grid.items()},
        "timing": "CUDA events around a CUDA graph of the timed launches, a 0.05 ms device spin before the start "
                  "event so the host's graph launch falls outside the timed region",
        "value_flags0": round(value_flags0, 2),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": traffic, "traffic_note": "dram read+write bytes per launch of the attention kernel "
                                                         f"from the committed ncu summary (profiles/{WL.profile})"
                     if traffic else "no ncu summary committed yet",
                     "kernel": "paged_decode_tc_kernel (tcgen05)" if tc_path else "paged_decode_kernel",
                     "algorithmic_bytes_per_launch": int(per_launch_bytes),
                     "vs_nominal_8TBs": round(achieved / 8000.0, 4)},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps, "ms_per_step": round(e2e_ms / e2e_steps, 5),
                "path": "b2_paged_attention_host via ctypes, one call per step: pinned-host q|block tables|seq_lens "
                        "read over PCIe by a small kernel into device memory, attention launch (it stores the "
                        "output straight into the pinned host buffer), stream sync",
                "max_abs_vs_device_run": e2e_match},
        "clocks": clk.summary(),
        # one launch per call on the CUDA cores (in-kernel merge); the tensor-core kernel adds its merge kernel
        "gpu_launches": (2 if tc_path else 1) * args.steps,
        "device_errors": errs,
    }
    return line


ENGINE_NAMES = ("gpt2-xl", "gpt2-medium", "gpt2-xl-heads", "gpt2-small")


def engine_result(args, name: str, rank: int, world: int, dist, steps: int, warmup: int, allgather: int = 0,
                  per_rank_batch: int | None = None, linear: bool | None = None) -> dict | None:
    """GPT-2 decode tokens/s through b2_engine_decode_step (engine_bench.py) on
    every rank; the whole job's line fields on rank 0, None elsewhere."""
    import torch
    import_package()
    from lis_b200 import engine_bench as EB
    w = EB.ENGINE_WORKLOADS[name]
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    samplers: list[ClockSampler] = []

    def timed_region():  # clocks are sampled during the timed steps of each wave only
        samplers.append(ClockSampler(dev.index))
        return samplers[-1]

    linear = bool(getattr(args, "linear", 0)) if linear is None else linear
    r = EB.run(w, steps, warmup, rank, world, dist, dev, timed_region, per_rank_batch=per_rank_batch,
               allgather=allgather, linear=linear, gemm_mode=int(getattr(args, "gemm_mode", 0)))
    clk = samplers[0]
    for extra in samplers[1:]:
        clk.samples.extend(extra.samples)

    tokens, t_max, value = job_rate(dist, float(r["tokens"]), r["ms"], dev)
    nbytes = reduce_over_ranks(dist, r["bytes"], "sum", dev)
    if rank != 0:
        return None
    peak, peak_kind = measured_peak()
    achieved = nbytes / (t_max * 1e-3) / 1e9  # whole job, GB/s
    frac = achieved / (peak * world)
    steps_total = steps * r["waves"]
    head_sharded = w.head_sharded and world > 1
    # block-table update scatter, table gather, embedding, per layer LN/append/attention/LN/GELU, final LN,
    # argmax, error-word copy (+ per layer a barrier and an epoch bump per step when head-sharded with the
    # fused epilogue; an interleave kernel per layer with NCCL)
    ours_per_step = 2 + 1 + 5 * w.n_layer + 3
    if head_sharded:
        ours_per_step += w.n_layer if allgather else 1 + w.n_layer
    if head_sharded:
        par = (f"head-sharded x{world}: " + ("attention output all-gathered with ncclAllGather (captured in the "
                                             "step graph) and interleaved for the projection" if allgather else
                                             "attention output all-gathered over NVLink in the attention epilogue, "
                                             "one flag barrier per layer"))
    else:
        par = f"sequence-sharded x{world}, one engine and KV pool per GPU, no collective"
    return {
        "metric": "GPT-2 decode tok/s", "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": round(t_max / steps_total, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": {BF16_CODE: "bf16", 1: "f16", 0: "f32"}[w.dtype], "data": "synthetic",
        "config": {"workload": w.description, "name": w.name, "global_batch": w.global_batch,
                   "per_gpu_batch": r["per_rank"], "waves_per_gpu": r["waves"], "wave": r["wave"],
                   "l2": "inputs larger than L2: every step reads all weights (GB) and every cached KV row",
                   "parallelism": par},
        "roofline": {"bound": "hbm", "achieved": round(achieved / world, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(frac, 4), "peak_kind": peak_kind, "traffic": None,
                     "traffic_note": "per GPU; algorithmic bytes per step = all weights + every cached K/V row "
                                     "of every layer + the appended rows",
                     "roofline_tok_s": round(value / frac, 1)},
        "e2e": {"value": round(value, 1), "unit": "tok/s",
                # tokens, positions, seq_lens and table slots (4 int32 per sequence) + one 12-byte
                # (slot, index, block) update per newly allocated block: one per sequence every 16 steps
                "h2d_bytes_per_step": 16 * r["wave"] + (12 * r["wave"] + 15) // 16,
                "d2h_bytes_per_step": 4 * r["wave"] + 4,
                "path": "value is already end to end: b2_engine_decode_step (device-resident block tables updated "
                        "incrementally, one upload of the step inputs, graph replay, download of next tokens and "
                        "the device error word, stream sync) timed with CUDA events on the engine stream"},
        "clocks": clk.summary(),
        "gpu_launches": ours_per_step * steps_total,
    }


def tp_token_check(rank: int, world: int, dist, modes=(0, 1)) -> dict | None:
    """Greedy tokens of the head-sharded engine (every rank, both all-gather
    modes) against the one-GPU engine (rank 0) on the same synthetic GPT-2
    XL-shaped model and prompts.  f32, so a greedy choice cannot flip on
    rounding: the GEMMs of the two layouts reduce in different orders.  16
    prompts of 8 random tokens, 16 generated tokens each."""
    import torch
    import_package()
    from lis_b200 import engine as E
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    shape = E.ModelShape(n_layer=48, n_head=25, d_model=1600, vocab_size=50257, n_ctx=1024, layer_norm_epsilon=1e-5,
                         eos_token_id=-1)
    rng = np.random.Generator(np.random.PCG64(77))
    plen, n_new = 8, 16
    prompts = [rng.integers(0, shape.vocab_size, size=plen).tolist() for _ in range(16)]

    def greedy(tp_size: int, mode: int) -> list[list[int]]:
        eng = E.Engine()
        eng.init_synthetic(shape, E.Config(max_batch=len(prompts), max_seq_len=64, kv_block_budget=96, dtype=0,
                                           use_cuda_graphs=True, device=dev.index,
                                           tp_rank=rank if tp_size > 1 else 0, tp_size=tp_size, tp_allgather=mode),
                           seed=3, std=0.02)
        if tp_size > 1 and mode:
            box = [E.Engine.tp_nccl_id() if rank == 0 else None]
            dist.broadcast_object_list(box, src=0)
            eng.tp_connect_nccl(box[0])
        elif tp_size > 1:
            handles = [None] * world
            dist.all_gather_object(handles, eng.tp_handle())
            eng.tp_connect(handles)
        ids = [eng.add_sequence(p) for p in prompts]
        gen = [[] for _ in prompts]
        for step in range(plen + n_new - 1):  # equal prompt lengths: every sequence moves in lockstep
            out = eng.decode_step(ids)
            if step >= plen - 1:
                for g, t in zip(gen, out):
                    g.append(int(t))
        eng.close()
        return gen

    sharded = {m: greedy(world, m) for m in modes}
    if dist is not None:
        dist.barrier()
    if rank != 0:
        return None
    full = greedy(1, 0)
    res = {"dtype": "f32", "prompts": len(prompts), "prompt_len": plen, "new_tokens": n_new,
           "model": "GPT-2 XL shape (48 layers, 25 heads, d_model 1600), synthetic weights N(0,0.02)"}
    for m, gen in sharded.items():
        same = sum(a == b for ga, gb in zip(gen, full) for a, b in zip(ga, gb))
        key = "nccl" if m else "fused"
        res[f"tokens_match_{key}"] = same == len(prompts) * n_new
        res[f"tokens_equal_{key}"] = f"{same}/{len(prompts) * n_new}"
    return res


def gqa_record(args, rank: int, world: int, dist) -> dict | None:
    """configs[2] (grouped-query long-context decode on the tensor-core kernel)
    as a record of the default line: the gqa workload's own measurement, at
    most 40 timed launches (each ~1.2 ms over ~7 GB), no CPU leg."""
    import argparse as _ap
    global WL
    saved = WL
    WL = WORKLOADS["gqa"]
    sub = _ap.Namespace(**vars(args))
    sub.steps, sub.warmup, sub.no_cpu = min(args.steps, 40), 3, True
    sub.sets = sub.pool_blocks = sub.batch = None
    try:
        return run_ours(sub, rank, world, dist)
    finally:
        WL = saved


def engine_records(args, rank: int, world: int, dist) -> dict:
    """The GPT-2 XL decode records attached to the default bench line: the
    sequence-sharded step at N GPUs, and at N >= 2 the head-sharded step with
    its two all-gather implementations and the token check."""
    steps, warmup = min(args.steps, 20), 3
    out: dict = {}
    xl = engine_result(args, "gpt2-xl", rank, world, dist, steps, warmup)
    if rank == 0:
        out["gpt2_xl"] = xl
    if world >= 2:
        fused = engine_result(args, "gpt2-xl-heads", rank, world, dist, steps, warmup, allgather=0)
        nccl = engine_result(args, "gpt2-xl-heads", rank, world, dist, steps, warmup, allgather=1)
        check = tp_token_check(rank, world, dist)
        if rank == 0:
            out["gpt2_xl_heads"] = {"fused_epilogue": fused, "nccl_allgather": nccl, "token_check": check,
                                    "fused_vs_nccl": round(fused["value"] / nccl["value"], 4)}
    return out


def gpt2_small_cpu(model_dir: str, prompts, n_new: int, nthreads: int, sample_new: int) -> dict:
    """The reference's CPUModel::greedy_generate (cpu_model.cpp:198-216, built
    from the reference's sources into oracle/_ref) on the host cores: the whole
    job on min(prompts, cores) threads (one CPUModel per thread, one prompt
    each), and a 1-thread sample of the shortest prompt with sample_new new
    tokens, scaled to the job by its forward steps."""
    from oracle import oracle as O
    gen, secs = O.ref_greedy_generate(model_dir, prompts, n_new, n_threads=nthreads)
    short = min(prompts, key=len)
    _, secs1 = O.ref_greedy_generate(model_dir, [short], sample_new, n_threads=1)
    steps1 = len(short) + sample_new - 1
    job_steps = sum(len(p) + n_new - 1 for p in prompts)
    est1 = secs1 / steps1 * job_steps
    return {"tokens": gen, "value": round(len(prompts) * n_new / secs, 3), "secs": secs,
            "one_thread_tok_s": round(len(prompts) * n_new / est1, 3),
            "one_thread_sample": f"1 prompt of {len(short)} tokens + {sample_new} new on 1 thread in {secs1:.2f} s "
                                 f"({steps1 / secs1:.2f} forward steps/s), scaled to the job's {job_steps} steps"}


def cpu_model_name() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_gpt2_small(args, rank: int, world: int, cpu: bool = True) -> dict | None:
    """GPT-2 small fp32 greedy decode (8 prompts of U[16,128] random tokens,
    64 new tokens each, weights N(0,0.02) seed 0 in the reference exporter's
    format): one step is the whole job through the engine's public calls --
    add_sequence, one b2_engine_prefill (first token), 63 decode_steps --
    timed with CUDA events on the engine stream.  The tokens are checked
    against the reference CPUModel's (committed fixture), and the reference's
    own CPU path is timed on the host cores as the baseline.  Rank 0 only."""
    if rank != 0:
        return None
    import torch
    import_package()
    from lis_b200 import engine as E
    from lis_b200 import model_files as MF
    fx = json.loads((ROOT / "tests" / "golden" / "gpt2_small_greedy.json").read_text())
    prompts, n_new = fx["prompts"], fx["n_new"]
    mdir = ROOT / "_models" / f"gpt2_small_seed{fx['seed']}"
    if not (mdir / "weights.bin").exists():
        MF.write_model_dir(mdir, MF.GPT2_SMALL, seed=fx["seed"], std=fx["std"])
    torch.cuda.set_device(0)
    eng = E.Engine()
    total = sum(len(p) for p in prompts)
    if not eng.init(str(mdir), E.Config(max_batch=len(prompts), max_seq_len=1024, kv_block_budget=1024, dtype=0,
                                         use_cuda_graphs=True, device=0, max_prefill_tokens=max(2048, total))):
        raise RuntimeError(eng.last_error())
    stream = torch.cuda.ExternalStream(eng.stream_handle(), device=torch.device("cuda:0"))

    def job():
        ids = [eng.add_sequence(p) for p in prompts]
        gen = [[t] for t in eng.prefill(ids)]
        for _ in range(n_new - 1):
            for g, t in zip(gen, eng.decode_step(ids)):
                g.append(t)
        for i in ids:
            eng.free_sequence(i)
        return gen

    steps, warmup = min(args.steps, 10), max(3, min(args.warmup, 5))
    for _ in range(warmup):
        gen = job()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        ev0.record(stream)
        for _ in range(steps):
            gen = job()
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / steps
    eng.close()
    match = sum(g == want[:n_new] for g, want in zip(gen, fx["generated"]))
    rec = {"metric": "GPT-2 small fp32 greedy tok/s", "value": round(len(prompts) * n_new / (ms * 1e-3), 1),
           "unit": "tok/s", "n_gpus": 1, "steps": steps, "warmup": warmup, "ms_per_step": round(ms, 3),
           "dtype": "f32", "data": "synthetic",
           "config": {"workload": "GPT-2 small (12 layers, 12 heads, d_model 768, vocab 50257), fp32, weights "
                                  "N(0,0.02) seed 0, LN gamma 1 beta 0; 8 prompts of U[16,128] random token ids, "
                                  "64 greedy tokens each; one step = add_sequence x8, b2_engine_prefill, 63 "
                                  "b2_engine_decode_step", "prompt_tokens": total},
           "tokens_match_reference": f"{match}/{len(prompts)} prompts identical to CPUModel::greedy_generate",
           "clocks": clk.summary(), "cpu_baseline": None}
    if cpu:
        from oracle import oracle as O
        if O.ref_available():
            nth = min(len(prompts), os.cpu_count() or 1)
            c = gpt2_small_cpu(str(mdir), prompts, n_new, nth, sample_new=8)
            rec["cpu_baseline"] = {
                "value": c["value"], "unit": "tok/s", "cores": nth, "kind": "reference",
                "cpu_model": cpu_model_name(), "host_cores": os.cpu_count(),
                "sample": f"the whole job (8 prompts x 64 tokens) by the reference CPUModel::greedy_generate, one "
                          f"CPUModel per thread, {nth} threads, {c['secs']:.1f} s; tokens identical to the GPU run: "
                          f"{c['tokens'] == gen}",
                "one_thread": {"value": c["one_thread_tok_s"], "unit": "tok/s", "sample": c["one_thread_sample"]}}
        else:
            rec["cpu_baseline_note"] = "oracle/_ref/libref_cpu.so (the reference CPU path) is not built here"
    return rec


def run_gpt2_small_reference(args, rank: int) -> None:
    """--impl reference --workload gpt2-small: the reference's own CPU forward
    path, CPUModel::greedy_generate (built from its sources into oracle/_ref),
    on the host cores -- the same 8 prompts x 64 tokens job, metric and unit as
    our arm.  Each step is the whole job on min(8, cores) threads.  Rank 0."""
    if rank != 0:
        return
    import_package()
    from lis_b200 import model_files as MF
    from oracle import oracle as O
    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref_cpu.so (the reference CPUModel "
                          "compiled from its sources) is not built"}), flush=True)
        return
    fx = json.loads((ROOT / "tests" / "golden" / "gpt2_small_greedy.json").read_text())
    prompts, n_new = fx["prompts"], fx["n_new"]
    mdir = ROOT / "_models" / f"gpt2_small_seed{fx['seed']}"
    if not (mdir / "weights.bin").exists():
        MF.write_model_dir(mdir, MF.GPT2_SMALL, seed=fx["seed"], std=fx["std"])
    nth = min(len(prompts), os.cpu_count() or 1)
    # each step is the whole job; bound the run: at most a few steps of it
    steps, warmup = min(args.steps, 3), min(args.warmup, 1)
    for _ in range(warmup):
        O.ref_greedy_generate(str(mdir), prompts, n_new, n_threads=nth)
    secs = 0.0
    for _ in range(steps):
        _, t = O.ref_greedy_generate(str(mdir), prompts, n_new, n_threads=nth)
        secs += t
    value = round(len(prompts) * n_new * steps / secs, 3)
    sample = (f"the whole job per step (8 prompts x 64 greedy tokens), CPUModel::greedy_generate with one CPUModel "
              f"per thread on {nth} threads ({cpu_model_name()}); {steps} timed of the requested {args.steps} "
              f"steps, {warmup} warm-up")
    print(json.dumps({"metric": "GPT-2 small fp32 greedy tok/s", "value": value, "unit": "tok/s", "impl": "reference",
                      "n_gpus": 1, "steps": steps, "warmup": warmup, "ms_per_step": round(secs / steps * 1e3, 3),
                      "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                      "data": "synthetic", "config": {"workload": "GPT-2 small fp32 greedy, 8 prompts x 64 tokens"},
                      "cpu_baseline": {"value": value, "unit": "tok/s", "cores": nth, "kind": "reference",
                                       "sample": sample},
                      "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


def run_engine(args, rank: int, world: int, dist) -> None:
    """One engine workload as the bench line (--workload gpt2-xl | gpt2-medium | gpt2-xl-heads)."""
    line = engine_result(args, args.workload, rank, world, dist, args.steps, args.warmup,
                         allgather=args.allgather, per_rank_batch=args.batch)
    if line is not None:
        line["cpu_baseline"] = None
        print(json.dumps(line), flush=True)


BF16_CODE = 2


HARNESS = ROOT / "oracle" / "_ref" / "ref_scheduler_harness"
REF_BENCH = ROOT / "oracle" / "_ref" / "ref_bench_gpu_scheduler"


def model_dir(shape_name: str, seed: int = 0, std: float = 0.02) -> Path:
    """A synthetic GPT-2 in the reference exporter's format under _models/ (written once)."""
    import_package()
    from lis_b200 import model_files as MF
    d = ROOT / "_models" / f"{shape_name}_seed{seed}"
    MF.write_model_dir(d, {"gpt2_small": MF.GPT2_SMALL, "gpt2_medium": MF.GPT2_MEDIUM}[shape_name], seed=seed, std=std)
    return d


def harness(mdir: Path, generator: str, env: dict | None = None, **opts) -> dict:
    """One run of the reference ContinuousBatchScheduler harness; its summary line."""
    import subprocess
    cmd = [str(HARNESS), str(mdir), generator] + [f"{k}={v}" for k, v in opts.items()]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=1800, env=dict(os.environ, **(env or {})))
    if r.returncode != 0:
        raise RuntimeError(f"scheduler harness failed ({r.returncode}): {r.stderr[-2000:]}")
    return [json.loads(ln) for ln in r.stdout.splitlines() if ln.startswith("{") and '"summary"' in ln][0]


def run_serve(args, rank: int, world: int) -> None:
    """configs[3] through the reference's own scheduler loop: the reference's
    ContinuousBatchScheduler (cpp-engine/src/scheduler.cpp, compiled unchanged)
    drives the engine on rank 0's GPU, with this library's
    BatchedPrefillGenerator (one b2_engine_prefill per admission) and, on the
    first requests of the same trace, the reference's GpuEngineGenerator
    (prompts walked token by token at batch 1, gpu_engine_generator.cpp:28-42).
    GPT-2 medium shape fp16, weights N(0, 0.02); Poisson arrivals at 50
    requests/s, prompts U[32, 512] token ids, outputs U[16, 512], max batch 128."""
    if rank != 0:
        return
    if not HARNESS.exists():
        print(json.dumps({"metric": "GPT-2 medium continuous-batching output tok/s", "unavailable":
                          "oracle/_ref/ref_scheduler_harness is not built (it links the reference's scheduler "
                          "sources)"}), flush=True)
        return
    mdir = model_dir("gpt2_medium")
    trace = dict(vocab=50257, seed=3, rate=50, prompt_lo=32, prompt_hi=512, out_lo=16, out_hi=512, max_batch=128,
                 max_seq_len=1024, kv_block_budget=9000, max_prefill_tokens=16384)
    with ClockSampler(0) as clk:
        full = harness(mdir, "batched", requests=args.requests, **trace)
        small_b = harness(mdir, "batched", requests=args.requests_compare, **trace)
        small_r = harness(mdir, "reference", requests=args.requests_compare, **trace)
    line = {
        "metric": "GPT-2 medium continuous-batching output tok/s", "value": round(full["output_tok_s"], 1),
        "unit": "tok/s", "n_gpus": 1, "steps": full["requests"], "warmup": 0,
        "ms_per_step": round(full["makespan_s"] * 1e3 / max(1, full["output_tokens"]), 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "GPT-2 medium shape (24 layers, 16 heads, d_model 1024), fp16, weights N(0,0.02); "
                               "Poisson 50 req/s, prompts U[32,512] random token ids, outputs U[16,512], max batch "
                               "128, block 16", "requests": full["requests"],
                   "loop": "the reference's ContinuousBatchScheduler (scheduler.cpp, unchanged) in "
                           "oracle/_ref/ref_scheduler_harness", "generator": "BatchedPrefillGenerator"},
        "ttft_p50_ms": full["ttft_p50_ms"], "ttft_p99_ms": full["ttft_p99_ms"], "makespan_s": full["makespan_s"],
        "prefill_comparison": {"requests": args.requests_compare, "batched (BatchedPrefillGenerator)": small_b,
                               "token by token (the reference's GpuEngineGenerator, unchanged)": small_r},
        "roofline": None, "roofline_note": "serving trace: arrival-bound and host-driven, no single-kernel roofline",
        "cpu_baseline": None,
        "e2e": {"value": round(full["output_tok_s"], 1), "unit": "tok/s", "h2d_bytes_per_step": None,
                "d2h_bytes_per_step": None, "path": "already end to end: requests submitted to the reference "
                "scheduler, tokens counted in its callback"},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_serve_ref(args, rank: int) -> None:
    """The reference's own scheduler benchmark, cpp-engine/bench/bench_gpu_scheduler.cpp compiled
    unchanged against this engine (oracle/_ref/ref_bench_gpu_scheduler): GPT-2 small shape fp16
    (the reference engine's dtype), 500 requests, outputs U[16,512], max batch 8, Poisson arrivals at
    85% of the measured continuous capacity; continuous vs static batching.  The reference publishes
    this benchmark's result (1317.9 / 1142.1 tok/s on an RTX 3060)."""
    if rank != 0:
        return
    import subprocess
    if not REF_BENCH.exists():
        print(json.dumps({"metric": "reference scheduler bench continuous tok/s", "unavailable":
                          "oracle/_ref/ref_bench_gpu_scheduler is not built"}), flush=True)
        return
    mdir = model_dir("gpt2_small")
    with ClockSampler(0) as clk:
        r = subprocess.run([str(REF_BENCH), str(mdir)], capture_output=True, text=True, timeout=3600)
    if r.returncode != 0:
        raise RuntimeError(f"ref_bench_gpu_scheduler failed: {r.stderr[-2000:]}")
    vals = {}
    for ln in r.stdout.splitlines():
        for key in ("continuous tok/s", "static tok/s", "ratio"):
            if ln.startswith(key + ":"):
                vals[key] = float(ln.split(":")[1].strip().rstrip("x"))
    cont = vals["continuous tok/s"]
    line = {
        "metric": "reference scheduler bench continuous tok/s", "value": cont, "unit": "tok/s", "n_gpus": 1,
        "steps": 500, "warmup": 0, "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(cont / 1317.9, 3), "dtype": "f16", "data": "synthetic",
        "config": {"workload": "cpp-engine/bench/bench_gpu_scheduler.cpp unchanged: GPT-2 small shape fp16 "
                               "(weights N(0,0.02)), 500 requests, outputs U[16,512], max batch 8, Poisson at 85% "
                               "of continuous capacity", "static_tok_s": vals.get("static tok/s"),
                   "continuous_over_static": vals.get("ratio"),
                   "published": "1317.9 / 1142.1 tok/s continuous / static on an RTX 3060 "
                                "(gpu-engine/VERIFICATION.md:157-158)"},
        "log_tail": r.stdout.splitlines()[-12:], "clocks": clk.summary(), "cpu_baseline": None, "roofline": None,
        "e2e": {"value": cont, "unit": "tok/s", "h2d_bytes_per_step": None, "d2h_bytes_per_step": None},
    }
    print(json.dumps(line), flush=True)


def run_lm_head(args, rank: int) -> None:
    """The decode step's tied lm_head + greedy argmax at the GPT-2 XL shape
    (d_model 1600, vocab 50257 padded to 50264 rows, bf16, weights N(0, 0.02),
    x N(0, 1)): b2_lm_head_argmax (one tensor-core launch, no logits) against
    the engine's unfused pair (cuBLAS GEMM into bf16 logits + b2_argmax_rows),
    at batch 1 .. 512.  Four weight copies rotate (161 MB each) so every launch
    streams its weights from HBM; a CUDA graph of 40 launches per timing, best
    of 3.  The tokens of the two paths are compared on the last launch."""
    import torch
    if rank != 0:
        return
    b2 = import_package()
    b2.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    V, Vp, D = 50257, 50264, 1600
    g = torch.Generator(device=dev).manual_seed(5)
    ws_ = [(torch.randn(Vp, D, generator=g, device=dev) * 0.02).to(torch.bfloat16) for _ in range(4)]
    rows = []
    for B in (1, 32, 128, 256, 512):
        x = torch.randn(B, D, generator=g, device=dev).to(torch.bfloat16)
        tok = torch.empty(B, dtype=torch.int32, device=dev)
        ref = torch.empty(B, dtype=torch.int32, device=dev)
        logits = torch.empty(B, Vp, device=dev, dtype=torch.bfloat16)
        wsp = b2.lm_head_argmax_workspace(B, dev)

        def fused(i):
            b2.lm_head_argmax(tok, x, ws_[i % 4], vocab=V, workspace=wsp)

        def unfused(i):
            torch.matmul(x, ws_[i % 4].T, out=logits)
            b2.argmax(ref, logits, vocab=V)

        def timeit(f):
            for i in range(8):
                f(i)
            torch.cuda.synchronize(dev)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                for i in range(40):
                    f(i)
            gr.replay()
            torch.cuda.synchronize(dev)
            best = 1e9
            for _ in range(3):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda._sleep(SPIN_CYCLES)
                e0.record(stream)
                gr.replay()
                e1.record(stream)
                torch.cuda.synchronize(dev)
                best = min(best, e0.elapsed_time(e1) * 1e3 / 40)
            return best

        tf, tu = timeit(fused), timeit(unfused)
        rows.append({"batch": B, "fused_us": round(tf, 2), "cublas_argmax_us": round(tu, 2),
                     "fused_weight_gbs": round(Vp * D * 2 / tf / 1e3, 1),
                     "tokens_identical": bool(torch.equal(tok, ref))})
    print(json.dumps({"metric": "GPT-2 XL lm_head + argmax, us per call", "unit": "us", "higher_is_better": False,
                      "dtype": "bf16", "data": "synthetic", "rows": rows, "device_errors": b2.device_errors(),
                      "config": {"workload": "tied lm_head + greedy argmax, d_model 1600, vocab 50257, bf16",
                                 "l2": "4 weight copies of 161 MB rotated"}}), flush=True)


def run_prefill(args, rank: int, world: int) -> None:
    """Prompt tokens/s of b2_engine_prefill (prefill_bench.py), rank 0."""
    if rank != 0:
        return
    import torch
    import_package()
    from lis_b200 import prefill_bench as PB
    torch.cuda.set_device(0)
    n_prompts, prompt_len = args.batch or 8, 512
    with ClockSampler(0) as clk:
        r = PB.run(n_prompts, prompt_len, steps=args.steps or 5, warmup=args.warmup or 3)
    tc, rows = r["tensor_cores"], r["decode_rows"]
    line = {
        "metric": "GPT-2 medium prefill prompt tok/s", "value": tc["prompt_tok_s"], "unit": "tok/s", "n_gpus": 1,
        "steps": r["steps"], "warmup": r["warmup"], "ms_per_step": tc["ms_per_call"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"b2_engine_prefill of {n_prompts} prompts x {prompt_len} uniform random tokens, "
                               "GPT-2 medium shape (24 layers, 16 heads, d_model 1024), fp16, weights N(0,0.02)",
                   "attention": "b2_prefill_attention (tcgen05, 128-row query tiles)"},
        "decode_rows": rows,
        "speedup_vs_decode_rows": round(tc["prompt_tok_s"] / rows["prompt_tok_s"], 2),
        "roofline": None, "roofline_note": "whole-model prefill call: GEMM-dominated; the attention kernel's "
                                           "tensor-pipe use is in profiles/prefill_attention_tc.md",
        "cpu_baseline": None,
        "e2e": {"value": tc["prompt_tok_s"], "unit": "tok/s", "h2d_bytes_per_step": None, "d2h_bytes_per_step": None,
                "path": "already end to end: each step is one blocking b2_engine_prefill call"},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default 5000; 20 for engine workloads)")
    ap.add_argument("--warmup", type=int, default=None, help="warm-up steps (default 50; 3 for engine workloads)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample duration")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    ap.add_argument("--no-engine", action="store_true",
                    help="default workload: skip the GPT-2 records attached to the attention line")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + list(ENGINE_NAMES) + ["serve-medium", "serve-ref", "prefill-medium", "lm-head"],
                    default="mha",
                    help="mha: the headline microbench (+ GPT-2 XL / small decode records); gqa: grouped-query long "
                         "contexts (tensor-core kernel); gpt2-xl / gpt2-medium / gpt2-xl-heads: GPT-2 decode "
                         "tokens/s through the engine; gpt2-small: the fp32 greedy job against the reference CPU")
    ap.add_argument("--sets", type=int, default=None, help="rotating input sets (profiling uses fewer)")
    ap.add_argument("--pool-blocks", type=int, default=None, help="KV pool size in blocks (profiling uses fewer)")
    ap.add_argument("--batch", type=int, default=None, help="sequences per GPU (profiling uses fewer)")
    ap.add_argument("--allgather", type=int, choices=[0, 1], default=0,
                    help="gpt2-xl-heads: 0 all-gather fused into the attention epilogue, 1 ncclAllGather")
    ap.add_argument("--linear", type=int, choices=[0, 1], default=0,
                    help="engine workloads: decode GEMMs on b2_linear (tcgen05) instead of cuBLAS")
    ap.add_argument("--gemm-mode", type=int, choices=[0, 1, 2, 3], default=0,
                    help="engine workloads: 1 cuBLASLt with timed algorithm choice, 3 also FC bias+GELU fused")
    ap.add_argument("--requests", type=int, default=200, help="serve-medium: requests in the trace")
    ap.add_argument("--requests-compare", type=int, default=24,
                    help="serve-medium: requests replayed with both prefill modes")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    engine = args.workload in ENGINE_NAMES
    if args.workload in ("serve-medium", "serve-ref"):
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the serving trace has no CPU arm"}), flush=True)
            return
        if args.workload == "serve-medium":
            run_serve(args, rank, world)
        else:
            run_serve_ref(args, rank)
        return
    if args.workload == "lm-head":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the lm_head comparison has no CPU arm"}), flush=True)
            return
        run_lm_head(args, rank)
        return
    if args.workload == "prefill-medium":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference has no batched prefill"}), flush=True)
            return
        run_prefill(args, rank, world)
        return
    if args.steps is None:
        args.steps = 20 if engine else 5000
    if args.warmup is None:
        args.warmup = 3 if engine else 50
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    global WL
    if not engine:
        WL = WORKLOADS[args.workload]

    if args.impl == "reference":
        if args.workload == "gpt2-small":
            run_gpt2_small_reference(args, rank)
            return
        if engine:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference CPU arm is timed for the "
                                  "attention workloads and gpt2-small; the GPT-2 XL / medium shapes have no CPU "
                                  "arm"}), flush=True)
            return
        run_reference_arm(args, rank, world)
        return
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        dist = tdist
    try:
        if args.workload == "gpt2-small":
            rec = run_gpt2_small(args, rank, world, cpu=not args.no_cpu)
            if rec is not None:
                rec.update({"higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                            "e2e": {"value": rec["value"], "unit": "tok/s", "h2d_bytes_per_step": None,
                                    "d2h_bytes_per_step": None, "path": "already end to end through "
                                    "b2_engine_add_sequence / b2_engine_prefill / b2_engine_decode_step"}})
                print(json.dumps(rec), flush=True)
        elif engine:
            run_engine(args, rank, world, dist)
        else:
            line = run_ours(args, rank, world, dist)
            import gc

            import torch
            gc.collect()
            torch.cuda.empty_cache()
            if WL.name == "mha" and not args.no_engine:
                extra = {}
                if world == 1:
                    extra["gqa"] = gqa_record(args, rank, world, dist)
                    gc.collect()
                    torch.cuda.empty_cache()
                extra.update(engine_records(args, rank, world, dist))
                if world == 1:
                    extra["gpt2_small"] = run_gpt2_small(args, rank, world, cpu=not args.no_cpu)
                if rank == 0:
                    line.update(extra)
            if rank == 0:
                print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
