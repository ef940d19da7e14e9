"""The engine on the GPU against the reference's own outputs.

Same runs and criteria as tests/test_ref_fixtures.py (which pins the CPU
oracle to the same fixtures), now through the engine: the reference's engine
and sampler outputs in tests/golden/ref_engine.npz / ref_sampler.npz (its
CUDA sources compiled for the host and run by
tests/golden/make_ref_fixtures.py) against prefill logits, per-step logits
and tokens of the engine's decode loop -- every generate call here is one
multi-step loop launch, the benchmarked mode, with each step's logits row
kept on the device -- and against the engine's sampler.
"""

import os
from dataclasses import replace

import numpy as np
import pytest

from parity import (draw_ok, FULL_SCALE, REF_CASES, case_logits, greedy_agree, top_row, near_boundary, row_err,
                    sampled_agree)
from rpgbarenginecuda_b200 import Model, SampleOptions, Session, counter_uniform, launch_count, sample, synthetic

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOY = {"tiny": 1, "tiny-g4": 2, "small": 3}
TOY_STD = 0.06
SAMPLE = (0.7, 20, 0.8)
SAMPLE_SEED = 1234


@pytest.fixture(scope="module")
def eng():
    return np.load(os.path.join(GOLD, "ref_engine.npz"))


@pytest.fixture(scope="module")
def smp():
    return np.load(os.path.join(GOLD, "ref_sampler.npz"))


def toy_path(name, fix, model_cache):
    path = synthetic.cached_model(replace(synthetic.PRESETS[name], weight_std=TOY_STD), seed=TOY[name],
                                  cache_dir=model_cache)
    assert synthetic.file_digest(path) == str(fix[f"{name}/digest"]), "the synthetic model writer changed"
    return path


def generate_one_launch(s, opts, seed, n):
    """generate with step logits; asserts the steps ran in one loop launch."""
    before = launch_count()
    ids, steps = s.generate(SampleOptions(*opts), seed, n, step_logits=True)
    assert launch_count() - before <= 4, "the decode steps did not run in one loop launch"
    return ids, steps


@pytest.mark.parametrize("name", list(TOY))
def test_engine_greedy_vs_reference(eng, model_cache, name):
    m = Model(toy_path(name, eng, model_cache), 0, 1024)
    s = Session(m, 512)
    k = f"{name}/greedy"
    rand_idx = eng[f"{name}/rand_idx"]
    lg = s.prefill(eng[f"{k}/prompt"])
    assert row_err(eng, f"{k}/prefill", 0, lg, rand_idx) <= FULL_SCALE
    ids, steps = generate_one_launch(s, (0.0, 0, 1.0), 0, 32)
    ref_ids = eng[f"{k}/ids"]
    ok, n = greedy_agree(ids, ref_ids, steps)
    assert ok, (n, ids, ref_ids)
    assert len(set(ids[:n].tolist())) >= min(8, n)
    for i in range(n):
        assert row_err(eng, f"{k}/steps", i, steps[i], rand_idx) <= FULL_SCALE, i
    assert len(s) == 21 + len(ids)
    s.close()
    m.close()


@pytest.mark.parametrize("name", list(TOY))
def test_engine_sampled_turns_vs_reference(eng, model_cache, oracle, name):
    """Prompt, then rounds of (16 tokens at T=0.7 top_k=20 top_p=0.8, append 9 ids)."""
    m = Model(toy_path(name, eng, model_cache), 0, 1024)
    s = Session(m, 512)
    k = f"{name}/turns"
    V = m.vocab
    rand_idx = eng[f"{name}/rand_idx"]
    lg = s.prefill(eng[f"{k}/prompt"])
    assert row_err(eng, f"{k}/prefill0", 0, lg, rand_idx) <= FULL_SCALE
    for r in range(3):
        kr = f"{k}/r{r}"
        start = int(eng[f"{kr}/start"])
        assert len(s) == start
        ids, steps = generate_one_launch(s, SAMPLE, SAMPLE_SEED, 16)
        ref_ids = eng[f"{kr}/ids"]
        u = lambda i: counter_uniform(SAMPLE_SEED, start + i)  # noqa: E731
        ok, n = sampled_agree(ids, ref_ids, lambda i, tok: draw_ok(oracle, steps[i], SAMPLE, u(i), tok),
                              lambda i, tok: draw_ok(oracle, top_row(eng, f"{kr}/steps", i, V), SAMPLE, u(i), tok))
        assert ok, (r, n, ids, ref_ids)
        for i in range(min(n + 1, len(ids))):
            assert row_err(eng, f"{kr}/steps", i, steps[i], rand_idx) <= FULL_SCALE, (r, i)
        if n < len(ref_ids):
            break  # later steps have different histories
        if r < 2:
            lg = s.prefill(eng[f"{kr}/append"])
            assert row_err(eng, f"{kr}/append_logits", 0, lg, rand_idx) <= FULL_SCALE
    s.close()
    m.close()


def test_engine_06b_config_vs_reference(eng, model_cache):
    """The 0.6B configuration: 21-id prompt, 32 greedy steps in one loop launch, V = 151936."""
    path = synthetic.cached_model("qwen3-0.6b", seed=0, cache_dir=model_cache)
    assert synthetic.file_digest(path) == str(eng["qwen3-0.6b/digest"])
    m = Model(path, 0, 4096)
    s = Session(m, 4096)
    k = "qwen3-0.6b/greedy"
    rand_idx = eng["qwen3-0.6b/rand_idx"]
    lg = s.prefill(eng[f"{k}/prompt"])
    assert row_err(eng, f"{k}/prefill", 0, lg, rand_idx) <= FULL_SCALE
    ids, steps = generate_one_launch(s, (0.0, 0, 1.0), 0, 32)
    ok, n = greedy_agree(ids, eng[f"{k}/ids"], steps)
    assert ok, (n, ids, eng[f"{k}/ids"])
    for i in range(n):
        assert row_err(eng, f"{k}/steps", i, steps[i], rand_idx) <= FULL_SCALE, i
    s.close()
    m.close()


@pytest.mark.parametrize("vocab", [4096, 151936])
def test_engine_sampler_vs_reference(oracle, smp, vocab):
    """tools/sample_check.cu's 12 cases and the 36-case sweep, 16 draws each, both
    engine paths (fast top-k and the general block), against the reference's tokens."""
    cases = [(float(t), int(k), float(p), int(seed), bool(tie)) for t, k, p, seed, tie in smp["cases"]]
    toks = smp[f"tokens_{vocab}"]
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    pr = torch.empty(vocab, dtype=torch.float32, device="cuda")
    for ci, case in enumerate(cases):
        t, k, p, seed, tie = case
        lg = case_logits(case, vocab)
        ld = torch.from_numpy(lg).cuda()
        probs = oracle.filter_to_probs(lg, t, k, p)
        if vocab == 4096 and ci < len(REF_CASES) and t > 0.0:
            sample(ld.data_ptr(), vocab, SampleOptions(t, k, p), seed, 0, tok.data_ptr(), pr.data_ptr())
            torch.cuda.synchronize()
            ours_p = pr.cpu().numpy()
            ref_p = smp[f"probs_{ci}"]
            assert np.abs(ours_p - ref_p).max() <= 1e-5 * np.abs(ref_p).max(), case
            assert np.array_equal(ours_p > 0, ref_p > 0), case
        for c in range(16):
            for want_probs in (False, True):
                sample(ld.data_ptr(), vocab, SampleOptions(t, k, p), seed, c, tok.data_ptr(),
                       pr.data_ptr() if want_probs else None)
                got = int(tok.item())
                if got != int(toks[ci, c]):
                    assert near_boundary(probs, counter_uniform(seed, c)), (case, c, got, int(toks[ci, c]))
