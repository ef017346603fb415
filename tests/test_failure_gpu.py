"""Failure detection on the GPU without a GPU fault.

Nothing here makes a kernel fail.  A bounded wait is made to run out by
waiting on a flag that nothing sets (the cross-GPU barrier with a 50 ms limit),
and the engine's error path is driven by setting a bit in the device error
word from a one-thread kernel (b2_raise_device_error).  The two-GPU case stops
one head-sharded rank between steps -- it connects, then never runs a step --
and the other rank's step must come back with B2_ERR_KERNEL once its barrier's
bounded wait gives up, instead of returning tokens.  Plain peer stores only (no
NVLink multicast, no NCCL).
"""
from __future__ import annotations

import ctypes
import multiprocessing as mp
import queue
import time

import pytest

pytestmark = pytest.mark.gpu

DEVERR_TIMEOUT = 4
ERR_KERNEL = -10


def test_barrier_wait_runs_out_and_reports_timeout(b2, cuda):
    import torch
    lib = b2.load()
    b2.device_errors()  # start from a clear word
    local = torch.zeros(4, dtype=torch.int32, device=cuda)
    nobody = torch.zeros(4, dtype=torch.int32, device=cuda)  # the "peer": no one ever writes our slot
    peers = torch.tensor([local.data_ptr(), nobody.data_ptr()], dtype=torch.int64, device=cuda)
    epoch = torch.ones(1, dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    rc = lib.b2_tp_barrier_timed(local.data_ptr(), peers.data_ptr(), 0, 2, epoch.data_ptr(), 0, 50_000_000, stream)
    assert rc == 0, lib.b2_last_error_string().decode()
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert waited < 5.0, f"the 50 ms wait took {waited:.2f} s"
    assert b2.device_errors() & DEVERR_TIMEOUT
    # our own slot was published, to ourselves and to the silent peer
    assert local[0].item() == 1 and nobody[0].item() == 1
    # the same barrier with the peer's flag present completes without an error
    local[1] = 1
    rc = lib.b2_tp_barrier_timed(local.data_ptr(), peers.data_ptr(), 0, 2, epoch.data_ptr(), 0, 50_000_000, stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert b2.device_errors() == 0


def _small_engine(b2, seed=5):
    from lis_b200 import engine as E
    shape = E.ModelShape(n_layer=2, n_head=2, d_model=128, vocab_size=512, n_ctx=128, layer_norm_epsilon=1e-5,
                         eos_token_id=-1)
    eng = E.Engine()
    eng.init_synthetic(shape, E.Config(max_batch=4, max_seq_len=128, kv_block_budget=64, dtype=b2.F16,
                                       use_cuda_graphs=True, device=0), seed=seed, std=0.02)
    ids = [eng.add_sequence_cached(20 + 7 * i, 3 + i) for i in range(3)]
    return eng, ids


def test_engine_step_fails_on_device_error_and_does_not_advance(b2, cuda):
    import torch
    from lis_b200 import B2Error
    lib = b2.load()
    b2.device_errors()
    a, ids_a = _small_engine(b2)
    b, ids_b = _small_engine(b2)
    first = a.decode_step(ids_a)
    assert b.decode_step(ids_b) == first
    second = b.decode_step(ids_b)
    # a bit set on engine a's stream before its step, as a kernel that gave up would set it
    assert lib.b2_raise_device_error(DEVERR_TIMEOUT, ctypes.c_void_p(a.stream_handle())) == 0
    with pytest.raises(B2Error) as ei:
        a.decode_step(ids_a)
    assert ei.value.code == ERR_KERNEL
    assert "bounded wait" in str(ei.value)
    torch.cuda.synchronize()
    assert b2.device_errors() == 0  # the engine cleared the word
    # no sequence advanced: the retried step gives what the clean engine's second step gave
    assert a.decode_step(ids_a) == second
    a.close()
    b.close()


def _two_gpus() -> bool:
    import torch
    return torch.cuda.is_available() and torch.cuda.device_count() >= 2


@pytest.mark.skipif(not _two_gpus(), reason="needs 2 GPUs")
def test_head_sharded_step_fails_when_a_rank_stops(b2, tmp_path_factory):
    import tp_worker
    from lis_b200 import model_files as MF
    shape = MF.GPT2Shape(n_layer=4, n_head=4, d_model=256, vocab_size=1024, n_ctx=256)
    d = MF.write_model_dir(tmp_path_factory.mktemp("tp_absent"), shape, seed=3, std=0.02)
    prompts = [[5, 6, 7], [8, 9]]
    ctx = mp.get_context("spawn")
    to_parent = ctx.Queue()
    to_child = [ctx.Queue() for _ in range(2)]
    procs = [ctx.Process(target=tp_worker.run, args=(r, 2, str(d), prompts, 1, 0, to_parent, to_child[r], 1))
             for r in range(2)]
    for p in procs:
        p.start()
    try:
        handles, result = {}, None
        while result is None:
            kind, rank, payload = to_parent.get(timeout=600)
            if kind == "error":
                pytest.fail(f"rank {rank} failed:\n{payload}")
            if kind == "handle":
                handles[rank] = payload
                if len(handles) == 2:
                    for q in to_child:
                        q.put([handles[0], handles[1]])
            elif kind == "failed_step":
                result = payload
        to_child[1].put("done")  # the stopped rank may close now
    except queue.Empty:
        pytest.fail("ranks did not report in time")
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    code, seconds, errs = result
    assert code == ERR_KERNEL, f"step returned {code} instead of B2_ERR_KERNEL"
    # one 2 s limit for the first layer's barrier; later layers do not wait again
    assert seconds < 20.0, f"the failed step took {seconds:.1f} s"
    assert errs == 0  # the engine cleared the word when it reported
