"""Host side of the decode engine (CPU only: nothing here touches a GPU).

* libb2engine.so exports every function include/b2_engine.h declares;
* its BlockPool behaves like the reference's BlockPool
  (gpu-engine/src/kv_cache_pool.cpp:6-28, tests gpu-engine/tests/test_kv_cache.cpp:8-63),
  checked op for op against the reference's own class when it is built;
* engine creation refuses missing / inconsistent weight files and bad
  configs before it touches a device.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import ROOT
from test_abi import declared_functions


@pytest.fixture(scope="module")
def E(b2):
    from lis_b200 import engine
    engine.load()
    return engine


def test_engine_library_exports_every_declared_symbol(E):
    lib = E.load()
    names = declared_functions("b2_engine.h")
    assert set(names) == set(E.ENGINE_SYMBOLS), "binding list out of date with include/b2_engine.h"
    for n in names:
        assert hasattr(lib, n), f"{n} not exported"


def test_block_pool_reference_cases(E):
    """gpu-engine/tests/test_kv_cache.cpp:8-63 against the engine's pool."""
    p = E.BlockPool(4)
    assert p.num_free() == 4
    b0 = p.allocate()
    assert b0 == 0 and p.num_free() == 3
    p.free(b0)
    assert p.num_free() == 4
    with pytest.raises(RuntimeError):
        p.free(b0)
    with pytest.raises(IndexError):
        p.free(5)
    with pytest.raises(IndexError):
        p.free(-1)
    ids = [p.allocate() for _ in range(4)]
    assert sorted(ids) == [0, 1, 2, 3] and p.allocate() == -1
    p.free(ids[1])
    assert p.allocate() == ids[1]
    assert E.BlockPool(0).allocate() == -1


def test_block_pool_matches_reference_op_for_op(E, oracle):
    if not oracle.ref_available():
        pytest.skip("reference CPU library not built (no reference checkout)")
    R = oracle.load_ref()
    rng = np.random.default_rng(7)
    n = 37
    ours, ref = E.BlockPool(n), R.ref_pool_create(n)
    try:
        held: list[int] = []
        for step in range(4000):
            r = rng.random()
            if r < 0.5:
                a, b = ours.allocate(), R.ref_pool_allocate(ref)
                assert a == b, f"allocate diverged at op {step}"
                if a >= 0:
                    held.append(a)
            else:
                if held and rng.random() < 0.8:
                    bid = held.pop(int(rng.integers(len(held))))
                else:  # a bad id: out of range or not allocated
                    bid = int(rng.integers(-3, n + 3))
                    if bid in held:
                        continue
                rc = R.ref_pool_free(ref, bid)
                if rc == 0:
                    ours.free(bid)
                elif rc == 1:
                    with pytest.raises(IndexError):
                        ours.free(bid)
                else:
                    with pytest.raises(RuntimeError):
                        ours.free(bid)
            assert ours.num_free() == R.ref_pool_num_free(ref)
    finally:
        R.ref_pool_destroy(ref)


def test_engine_create_refuses_missing_and_bad_files(E, tmp_path):
    eng = E.Engine()
    assert eng.init(tmp_path / "nowhere", E.Config()) is False
    assert "config.json" in eng.last_error()
    from lis_b200 import model_files as MF
    d = MF.write_model_dir(tmp_path / "m", MF.GPT2Shape(n_layer=1, n_head=2, d_model=128, vocab_size=64, n_ctx=32),
                           seed=3, std=0.1)
    # max_seq_len beyond n_ctx: refused before any device work.
    assert eng.init(d, E.Config(max_seq_len=64)) is False
    assert "max_seq_len" in eng.last_error()
    # head_dim outside the kernels' set.
    cfg = json.loads((d / "config.json").read_text())
    bad = tmp_path / "bad"
    bad.mkdir()
    cfg.update(n_head=4, head_dim=32)
    (bad / "config.json").write_text(json.dumps(cfg))
    assert eng.init(bad, E.Config(max_seq_len=32)) is False
    assert "head_dim" in eng.last_error()
    # head-sharded configs outside 1..8 ranks, or a rank outside the group
    for tp_size, tp_rank in ((9, 0), (2, 2), (2, -1)):
        assert eng.init(d, E.Config(max_seq_len=32, tp_size=tp_size, tp_rank=tp_rank)) is False
        assert "tp_size" in eng.last_error()


CXX_CALLER = r"""
#include <cstdio>
#include "b2_engine_api.hpp"
// A caller written against the reference's Engine declarations.
int main(int argc, char** argv) {
    EngineConfig cfg;
    cfg.max_batch = 8;
    Engine eng;
    if (eng.init(argv[1], cfg)) return 1;          // the directory does not exist
    std::printf("%s\n", Engine::last_error().c_str());
    try { int id = 0, out = 0; eng.decode_step(&id, 1, &out); return 2; }
    catch (const std::runtime_error&) {}
    b2_block_pool* p = b2_block_pool_create(2);
    const int a = b2_block_pool_allocate(p), b = b2_block_pool_allocate(p), c = b2_block_pool_allocate(p);
    const int r = b2_block_pool_free(p, 7);
    b2_block_pool_destroy(p);
    return (a == 0 && b == 1 && c == -1 && r == 1) ? 0 : 3;
}
"""


def test_cpp_engine_class_compiles_and_links(E, tmp_path):
    """include/b2_engine_api.hpp gives a reference-style caller what it binds."""
    import shutil
    import subprocess
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    src = tmp_path / "caller.cpp"
    src.write_text(CXX_CALLER)
    exe = tmp_path / "caller"
    lib = E.lib_path().parent
    subprocess.run([gxx, "-std=c++17", "-I", str(ROOT / "include"), str(src), "-o", str(exe), "-L", str(lib),
                    "-lb2engine", f"-Wl,-rpath,{lib}"], check=True)
    res = subprocess.run([str(exe), str(tmp_path / "missing")], capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "config.json" in res.stdout


def test_engine_header_documents_reference_calls():
    text = (ROOT / "include" / "b2_engine.h").read_text()
    for ref in ("engine_api.h", "engine.cu:296-307", "engine.cu:309-377", "kv_cache_pool.cpp"):
        assert ref in text
