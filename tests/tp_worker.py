"""Worker process of the head-sharded engine tests (one process per GPU).

Each worker builds its rank's engine, publishes its IPC handles through
`to_parent`, receives every rank's handles from `from_parent`, connects, runs
the greedy decode of `prompts` and returns the tokens.  Kept in its own module
so `multiprocessing` (spawn) can import it without the test module.
"""
from __future__ import annotations

import sys
import traceback
from pathlib import Path


def run(rank: int, world: int, model_dir: str, prompts, n_new: int, dtype: int, to_parent, from_parent,
        absent_rank: int = -1) -> None:
    """absent_rank >= 0: that rank connects and registers its sequences, then
    never calls decode_step (it stops between steps, nothing of its own in
    flight) and closes only when the parent says so; the other ranks try one
    step, which must fail with B2_ERR_KERNEL once the barrier's bounded wait
    runs out, and report (code, seconds)."""
    try:
        root = Path(__file__).resolve().parents[1]
        sys.path.insert(0, str(root / "tests"))
        sys.path.insert(0, str(root))
        from conftest import import_package
        import_package()
        import torch
        torch.cuda.set_device(rank)
        from lis_b200 import engine as E
        eng = E.Engine()
        ok = eng.init(model_dir, E.Config(max_batch=len(prompts), max_seq_len=256, kv_block_budget=256, dtype=dtype,
                                          device=rank, tp_rank=rank, tp_size=world))
        if not ok:
            raise RuntimeError(eng.last_error())
        to_parent.put(("handle", rank, eng.tp_handle()))
        handles = from_parent.get(timeout=300)
        eng.tp_connect(handles)
        ids = [eng.add_sequence(p) for p in prompts]
        if absent_rank >= 0:
            import time
            import lis_b200
            if rank == absent_rank:
                to_parent.put(("absent", rank, None))
                from_parent.get(timeout=300)  # the others are done
                eng.close()
                return
            t0 = time.perf_counter()
            try:
                eng.decode_step(ids)
                code = 0
            except lis_b200.B2Error as e:
                code = e.code
            to_parent.put(("failed_step", rank, (code, time.perf_counter() - t0, lis_b200.device_errors())))
            eng.close()
            return
        consumed = [0] * len(prompts)
        gen = [[] for _ in prompts]
        while any(len(g) < n_new for g in gen):
            active = [i for i in range(len(prompts)) if len(gen[i]) < n_new]
            out = eng.decode_step([ids[i] for i in active])
            for i, tok in zip(active, out):
                consumed[i] += 1
                if consumed[i] >= len(prompts[i]):
                    gen[i].append(tok)
        import lis_b200
        errs = lis_b200.device_errors()
        eng.close()
        to_parent.put(("tokens", rank, (gen, errs)))
    except Exception:  # noqa: BLE001 -- reported to the parent
        to_parent.put(("error", rank, traceback.format_exc()))
