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


def run(rank: int, world: int, model_dir: str, prompts, n_new: int, dtype: int, to_parent, from_parent) -> None:
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
