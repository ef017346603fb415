"""Head-sharded engine on 2 GPUs (GPU; skipped with fewer than 2).

GPT-2 small fp32 split over two ranks (6 heads each): every layer's attention
writes its heads' output rows into both ranks' gathered buffers over NVLink and
the ranks meet at the flag barrier before the output projection.  Both ranks
must reproduce, token for token, the greedy tokens of the reference's
CPUModel::greedy_generate (tests/golden/gpt2_small_greedy.json) -- the same bar
the single-GPU engine meets.
"""
from __future__ import annotations

import multiprocessing as mp
import queue

import pytest

pytestmark = pytest.mark.gpu


def _two_gpus() -> bool:
    import torch
    return torch.cuda.is_available() and torch.cuda.device_count() >= 2


@pytest.mark.skipif(not _two_gpus(), reason="needs 2 GPUs")
def test_head_sharded_gpt2_small_matches_reference_tokens(b2, golden, tmp_path_factory):
    import tp_worker
    from lis_b200 import model_files as MF
    fx = golden("gpt2_small_greedy.json")
    d = MF.write_model_dir(tmp_path_factory.mktemp("tp_small"), MF.GPT2_SMALL, seed=fx["seed"], std=fx["std"])
    prompts, n_new = fx["prompts"][:4], 24
    ctx = mp.get_context("spawn")
    to_parent = ctx.Queue()
    to_child = [ctx.Queue() for _ in range(2)]
    procs = [ctx.Process(target=tp_worker.run, args=(r, 2, str(d), prompts, n_new, 0, to_parent, to_child[r]))
             for r in range(2)]
    for p in procs:
        p.start()
    try:
        handles, results = {}, {}
        while len(results) < 2:
            kind, rank, payload = to_parent.get(timeout=600)
            if kind == "error":
                pytest.fail(f"rank {rank} failed:\n{payload}")
            if kind == "handle":
                handles[rank] = payload
                if len(handles) == 2:
                    for q in to_child:
                        q.put([handles[0], handles[1]])
            else:
                results[rank] = payload
    except queue.Empty:
        pytest.fail("head-sharded ranks did not finish in time")
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank in range(2):
        gen, errs = results[rank]
        assert errs == 0, f"rank {rank} device errors {errs}"
        for i, (g, want) in enumerate(zip(gen, fx["generated"])):
            assert g == want[:n_new], f"rank {rank}, prompt {i} diverged"
