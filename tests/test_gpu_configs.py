"""The engine at the benchmark configurations' full size, against the oracle.

tests/golden/oracle_configs.npz (tests/golden/make_oracle_fixtures.py) holds
the CPU oracle's outputs -- the oracle is pinned to the reference's own
outputs by tests/test_ref_fixtures.py -- on:
* 1.7B (28 layers, V = 151936): the benchmark's 2811-id prompt, then 3
  rounds of 16 tokens at T = 0.7, top_k = 20, top_p = 0.8 with the
  benchmark's 40-id appends between them; attention runs over 2811-2939
  positions with every split of the decode loop in use;
* 4B (36 layers, 32 query heads over 8 KV heads, G = 4): 8 greedy tokens at
  contexts 512 and 3840.
Every decode call is one multi-step loop launch (the benchmarked mode).
Criteria as everywhere (tests/parity.py): logits within 1e-3 of full scale,
greedy tokens identical up to a gap-rule divergence, sampled tokens identical up
to a divergence where each side's token is the checker's draw from its own
logits.
"""

import os

import numpy as np
import pytest

from parity import FULL_SCALE, draw_ok, greedy_agree, top_row, row_err, sampled_agree
from rpgbarenginecuda_b200 import Model, SampleOptions, Session, counter_uniform, launch_count, synthetic

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

FIX = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "oracle_configs.npz")
SAMPLE = (0.7, 20, 0.8)
SAMPLE_SEED = 1234


@pytest.fixture(scope="module")
def fix():
    if not os.path.exists(FIX):
        pytest.skip("tests/golden/oracle_configs.npz not generated")
    return np.load(FIX)


def model_for(fix, name, model_cache):
    if f"{name}/digest" not in fix:
        pytest.skip(f"no {name} fixture")
    path = synthetic.cached_model(name, seed=0, cache_dir=model_cache)
    assert synthetic.file_digest(path) == str(fix[f"{name}/digest"]), "the synthetic model writer changed"
    return Model(path, 0, 4096)


def test_17b_benchmark_turn(fix, model_cache, oracle):
    k = "qwen3-1.7b"
    m = model_for(fix, k, model_cache)
    s = Session(m, 4096)
    V = m.vocab
    rand_idx = fix[f"{k}/rand_idx"]
    lg = s.prefill(fix[f"{k}/prompt"])
    assert row_err(fix, f"{k}/prefill", 0, lg, rand_idx) <= FULL_SCALE
    for r in range(3):
        kr = f"{k}/r{r}"
        start = int(fix[f"{kr}/start"])
        assert len(s) == start
        before = launch_count()
        ids, steps = s.generate(SampleOptions(*SAMPLE), SAMPLE_SEED, 16, step_logits=True)
        assert launch_count() - before <= 4
        ref_ids = fix[f"{kr}/ids"]
        u = lambda i: counter_uniform(SAMPLE_SEED, start + i)  # noqa: E731
        ok, n = sampled_agree(ids, ref_ids, lambda i, tok: draw_ok(oracle, steps[i], SAMPLE, u(i), tok),
                              lambda i, tok: draw_ok(oracle, top_row(fix, f"{kr}/steps", i, V), SAMPLE, u(i), tok))
        assert ok, (r, n, list(ids), list(ref_ids))
        for i in range(min(n + 1, len(ids))):
            assert row_err(fix, f"{kr}/steps", i, steps[i], rand_idx) <= FULL_SCALE, (r, i)
        if n < len(ref_ids):
            break
        if r < 2:
            lg = s.prefill(fix[f"{kr}/append"])
            assert row_err(fix, f"{kr}/append_logits", 0, lg, rand_idx) <= FULL_SCALE
    s.close()
    m.close()


@pytest.mark.parametrize("ctx", [512, 3840])
def test_4b_greedy_at_context(fix, model_cache, ctx):
    k = "qwen3-4b"
    m = model_for(fix, k, model_cache)
    s = Session(m, 4096)
    kc = f"{k}/ctx{ctx}"
    if f"{kc}/prompt" not in fix:
        pytest.skip(f"no {kc} fixture")
    rand_idx = fix[f"{k}/rand_idx"]
    lg = s.prefill(fix[f"{kc}/prompt"])
    assert row_err(fix, f"{kc}/prefill", 0, lg, rand_idx) <= FULL_SCALE
    ids, steps = s.generate(SampleOptions(0.0, 0, 1.0), 0, 8, step_logits=True)
    ok, n = greedy_agree(ids, fix[f"{kc}/ids"], steps)
    assert ok, (n, list(ids), list(fix[f"{kc}/ids"]))
    for i in range(n):
        assert row_err(fix, f"{kc}/steps", i, steps[i], rand_idx) <= FULL_SCALE, i
    s.close()
    m.close()
