"""The N > 1 host paths of bench.py on the CPU: two ranks over gloo.

Covers what every multi-GPU bench line relies on besides the kernels: how an
engine workload's global batch is spread over the ranks (sequence-sharded:
disjoint shares that add up to the batch, one seed per rank; head-sharded: the
whole batch on every rank, one seed, each token counted once), the cross-rank
reductions (slowest rank's time, units of all ranks) and the job rate made
from them, the reference arm under torchrun (rank 0 alone works and prints
one line; the other rank exits 0 without output), and a rank that leaves
between steps: the next reduction on the rank that stays ends in an error
within the group's short timeout instead of waiting.  CPU only."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

import pytest

from conftest import ROOT, import_package


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _load_bench():
    import importlib.util
    if "bench_under_test" in sys.modules:
        return sys.modules["bench_under_test"]
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["bench_under_test"] = mod
    spec.loader.exec_module(mod)
    return mod


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    """One gloo rank: its shard plans, the reductions, the job rate."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        bench = _load_bench()
        import_package()
        from lis_b200 import engine_bench as EB
        cpu = torch.device("cpu")
        plans = {name: EB.shard_plan(w, rank, world).__dict__ for name, w in EB.ENGINE_WORKLOADS.items()
                 if w.global_batch % world == 0}
        every = [None] * world
        dist.all_gather_object(every, plans)
        ms = 10.0 + 5.0 * rank          # this rank's timed region
        units = 1000.0 * (rank + 1)     # what it processed
        got = {
            "max": bench.reduce_over_ranks(dist, ms, "max", cpu),
            "sum": bench.reduce_over_ranks(dist, units, "sum", cpu),
            "job": bench.job_rate(dist, units, ms, cpu),
            "plans": every,
        }
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(got, f)
    finally:
        dist.destroy_process_group()


def _rank_leaves_early(rank: int, world: int, port: int, out_dir: str) -> None:
    """Rank 1 leaves between steps (exits before the step's reduction); rank 0's
    reduction must end with an error within the group's short timeout."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import time

    import torch.distributed as dist
    sys.path.insert(0, str(ROOT))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    bench = _load_bench()
    bench.reduce_over_ranks(dist, 1.0, "sum", "cpu")  # step 1: both ranks
    if rank == 1:
        os._exit(0)  # gone before step 2, with nothing in flight
    t0 = time.perf_counter()
    try:
        bench.reduce_over_ranks(dist, 1.0, "sum", "cpu")
        outcome = "returned"
    except Exception as e:  # noqa: BLE001 -- any error is the detection
        outcome = type(e).__name__
    with open(os.path.join(out_dir, "rank0.json"), "w") as f:
        json.dump({"outcome": outcome, "waited_s": time.perf_counter() - t0}, f)
    os._exit(0)  # the group cannot be torn down cleanly without its peer


def test_a_rank_that_leaves_is_detected_by_the_next_reduction(tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.start_processes(_rank_leaves_early, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
        assert p.exitcode == 0
    r = json.loads((tmp_path / "rank0.json").read_text())
    assert r["outcome"] != "returned"
    assert r["waited_s"] < 60


def test_two_gloo_ranks_shard_and_reduce(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    res = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(world)]
    for r in res:
        assert r["max"] == 15.0
        assert r["sum"] == 3000.0
        total, t_max, rate = r["job"]
        assert (total, t_max) == (3000.0, 15.0) and rate == pytest.approx(3000.0 / 15e-3)
        assert r["plans"] == res[0]["plans"]  # every rank sees the same gathered plans
    import_package()
    from lis_b200 import engine_bench as EB
    steps = 7
    for name, w in EB.ENGINE_WORKLOADS.items():
        plans = [p[name] for p in res[0]["plans"]]
        tokens = sum(p["per_rank"] * steps / p["token_div"] for p in plans)
        assert tokens == w.global_batch * steps, name  # each token of the job counted once
        for p in plans:
            assert p["wave"] <= w.wave_cap and p["waves"] * p["wave"] >= p["per_rank"]
            assert (p["waves"] - 1) * p["wave"] < p["per_rank"]
        if w.head_sharded:
            assert all(p["sharded"] and p["per_rank"] == w.global_batch for p in plans)
            assert len({p["seed"] for p in plans}) == 1  # the same sequences on every rank
        else:
            assert sum(p["per_rank"] for p in plans) == w.global_batch
            assert len({p["seed"] for p in plans}) == world  # each rank its own sequences


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_plans_cover_the_job(world):
    import_package()
    from lis_b200 import engine_bench as EB
    for name, w in EB.ENGINE_WORKLOADS.items():
        if w.head_sharded and world == 1:
            with pytest.raises(ValueError):
                EB.shard_plan(w, 0, world)
            continue
        plans = [EB.shard_plan(w, r, world) for r in range(world)]
        assert sum(p.tokens(5) for p in plans) == w.global_batch * 5, name
    xl = EB.ENGINE_WORKLOADS["gpt2-xl"]
    assert (EB.shard_plan(xl, 0, 1).waves, EB.shard_plan(xl, 0, 1).wave) == (2, 512)  # one GPU: 2 waves of 512
    assert (EB.shard_plan(xl, 3, 8).per_rank, EB.shard_plan(xl, 3, 8).waves) == (128, 1)
    assert EB.shard_plan(xl, 0, 8, per_rank_batch=64).per_rank == 64
    with pytest.raises(ValueError):
        EB.shard_plan(xl, 0, 3)  # 1024 does not split over 3 ranks


def test_reduce_without_process_group_is_identity():
    bench = _load_bench()
    assert bench.reduce_over_ranks(None, 2.5, "max", "cpu") == 2.5
    assert bench.job_rate(None, 100.0, 20.0, "cpu") == (100.0, 20.0, 100.0 / 20e-3)


def test_reference_arm_under_torchrun_two_ranks():
    """Rank 0 alone runs the CPU reference arm and prints one line; rank 1
    exits 0 without work or output."""
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "3", "--warmup", "3"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["cpu_baseline"]["value"] == d["value"]
