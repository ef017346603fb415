"""Pins the oracle to the reference's own CPU forward path (CPU only).

The greedy decode composed from the oracle primitives over a paged KV cache
(oracle/gpt2.py) must reproduce, token for token, what the reference's
CPUModel::greedy_generate (gpu-engine/src/reference/cpu_model.cpp:198-216)
produced on the same synthetic weights: the committed fixtures were made by
the reference compiled from its own sources (tests/golden/make_golden.py).
When the reference library is present (oracle/_ref), a fresh model and prompt
are also compared live.  The reference's BlockPool is exercised as its own
tests do (gpu-engine/tests/test_kv_cache.cpp:8-63).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import gpt2, oracle as O


def _model(b2, tmp_root, name, shape, seed, std):
    from lis_b200 import model_files as MF
    d = tmp_root / name
    MF.write_model_dir(d, MF.GPT2Shape(**shape), seed=seed, std=std)
    return MF.load_model_dir(d), d


def test_oracle_reproduces_reference_greedy_tokens(b2, golden, tmp_path_factory):
    fx = golden("gpt2_tiny_greedy.json")
    root = tmp_path_factory.mktemp("models")
    for case in fx["cases"]:
        (cfg, tensors), _ = _model(b2, root, case["name"], case["shape"], case["seed"], case["std"])
        for prompt, expected in zip(case["prompts"], case["generated"]):
            got = gpt2.greedy_generate(cfg, tensors, prompt, case["n_new"], nthreads=2)
            assert got == expected, f"{case['name']} prompt len {len(prompt)}"


def test_oracle_matches_gpt2_small_fixture_prefix(b2, golden, tmp_path_factory):
    """GPT-2 small fp32 (the greedy-identity workload): the shortest prompt, first 6 tokens."""
    fx = golden("gpt2_small_greedy.json")
    from lis_b200 import model_files as MF
    d = MF.write_model_dir(tmp_path_factory.mktemp("small"), MF.GPT2_SMALL, seed=fx["seed"], std=fx["std"])
    cfg, tensors = MF.load_model_dir(d)
    i = int(np.argmin([len(p) for p in fx["prompts"]]))
    got = gpt2.greedy_generate(cfg, tensors, fx["prompts"][i], 6, nthreads=8)
    assert got == fx["generated"][i][:6]


@pytest.mark.skipif(not O.ref_available(), reason="reference CPU library not built (no reference checkout)")
def test_oracle_matches_reference_live(b2, tmp_path_factory):
    root = tmp_path_factory.mktemp("live")
    (cfg, tensors), d = _model(b2, root, "live", dict(n_layer=2, n_head=2, d_model=64, vocab_size=257, n_ctx=80),
                               seed=11, std=0.3)
    prompts = [[3, 1, 4, 1, 5, 9, 2, 6], list(range(40, 61))]
    ref, _ = O.ref_greedy_generate(str(d), prompts, 25, n_threads=2)
    for p, r in zip(prompts, ref):
        assert gpt2.greedy_generate(cfg, tensors, p, 25, nthreads=2) == r


@pytest.mark.skipif(not O.ref_available(), reason="reference CPU library not built (no reference checkout)")
def test_reference_block_pool_behaviour():
    """gpu-engine/tests/test_kv_cache.cpp:8-63 run against the reference's own BlockPool."""
    R = O.load_ref()
    p = R.ref_pool_create(4)
    try:
        assert R.ref_pool_num_free(p) == 4
        b0 = R.ref_pool_allocate(p)
        assert b0 >= 0 and R.ref_pool_num_free(p) == 3
        assert R.ref_pool_free(p, b0) == 0 and R.ref_pool_num_free(p) == 4
        assert R.ref_pool_free(p, b0) == 2      # double free -> std::logic_error
        assert R.ref_pool_free(p, 5) == 1       # out of range -> std::out_of_range
        assert R.ref_pool_free(p, -1) == 1
        ids = [R.ref_pool_allocate(p) for _ in range(4)]
        assert sorted(ids) == [0, 1, 2, 3] and R.ref_pool_allocate(p) == -1
        R.ref_pool_free(p, ids[1])
        assert R.ref_pool_allocate(p) == ids[1]  # LIFO reuse
    finally:
        R.ref_pool_destroy(p)
