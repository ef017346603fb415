"""The reference's own scheduler loop on this library's engine (GPU).

oracle/_ref/ref_scheduler_harness links the reference's ContinuousBatchScheduler,
its slot allocator and its GpuEngineGenerator -- cpp-engine/src/scheduler.cpp,
kv_cache.cpp and gpu_engine_generator.cpp, compiled unchanged from the
reference's sources, the generator's "engine/engine_api.h" resolving to
include/compat/engine/engine_api.h -- against libb2engine.so.  Requests with
token-count-controlled prompts are submitted through
ContinuousBatchScheduler::submit; the tokens its callback streams must equal
the greedy tokens the engine gives each prompt on its own (the Python
binding, batch 1).  The engine runs f32 (B2_ENGINE_DTYPE=f32), where the f32
engine already reproduces the reference CPUModel token for token, so a
mismatch can only come from the scheduler path.  Also checked: the same with
static batching, and with this library's BatchedPrefillGenerator
(include/b2_batched_generator.hpp) in place of the reference's generator.
"""
from __future__ import annotations

import json
import os
import subprocess

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

HARNESS = ROOT / "oracle" / "_ref" / "ref_scheduler_harness"
SHAPE = dict(n_layer=4, n_head=4, d_model=256, vocab_size=1024, n_ctx=1024)


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory, b2):
    from lis_b200 import model_files as MF
    return MF.write_model_dir(tmp_path_factory.mktemp("sched_model"), MF.GPT2Shape(**SHAPE), seed=11, std=0.02)


def _run(model_dir, generator, **opts):
    args = [str(HARNESS), str(model_dir), generator, "per_request=1", f"vocab={SHAPE['vocab_size']}"]
    args += [f"{k}={v}" for k, v in opts.items()]
    env = dict(os.environ, B2_ENGINE_DTYPE="f32")
    r = subprocess.run(args, capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = [json.loads(ln) for ln in r.stdout.splitlines() if ln.startswith("{")]
    reqs = [d for d in lines if "req" in d]
    summary = [d for d in lines if d.get("summary")][0]
    return reqs, summary


def _greedy(model_dir, prompt, n_new):
    from lis_b200 import engine as E
    eng = E.Engine()
    assert eng.init(str(model_dir), E.Config(max_batch=1, max_seq_len=1024, kv_block_budget=256, dtype=0, device=0))
    sid = eng.add_sequence(prompt)
    out = []
    for i in range(len(prompt) + n_new - 1):
        t = eng.decode_step([sid])[0]
        if i >= len(prompt) - 1:
            out.append(t)
    eng.close()
    return out


@pytest.mark.skipif(not HARNESS.exists(), reason="oracle/_ref/ref_scheduler_harness is built only where the "
                                                 "reference sources are (oracle/Makefile)")
@pytest.mark.parametrize("generator,static", [("reference", 0), ("reference", 1), ("batched", 0)])
def test_reference_scheduler_streams_the_engines_greedy_tokens(model_dir, generator, static):
    reqs, summary = _run(model_dir, generator, requests=10, max_batch=4, seed=5, prompt_lo=2, prompt_hi=40,
                         out_lo=3, out_hi=20, static=static)
    assert summary["requests"] == 10 and len(reqs) == 10
    for d in reqs:
        want = _greedy(model_dir, d["prompt"], len(d["tokens"]))
        assert d["tokens"] == want, f"request {d['req']} ({generator}, static={static})"
        assert d["finish"] == 2  # length: the test model's eos id is never generated
