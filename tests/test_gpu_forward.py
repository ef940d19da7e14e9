"""End-to-end token-loop parity against the CPU oracle on toy Qwen3 models.

The oracle itself is pinned to the reference's own outputs
(tests/test_ref_fixtures.py); tests/test_gpu_ref_fixtures.py compares the
engine with those outputs directly.  Criteria (tests/parity.py, the
reference's tests/cmp_gen.py and tests/cmp_sample.py):
* prefill / per-step logits within 1e-3 of full scale;
* greedy tokens identical; a divergence only where the two tokens' logits
  differ by <= 1e-2 of the logit span, and the comparison stops there;
* sampled tokens identical; at a divergence each side's token must be the
  checker's draw from that side's own logits with the same u;
* cache.len == prompt + generated (src/qwen3_gpu.cu:585-593), the stop token
  is forwarded.
Every generate call with step logits runs its steps in one decode-loop launch
(the benchmarked mode); each step's logits row is kept on the device.
"""

import numpy as np
import pytest

from oracle.oracle import OracleModel, OracleSession
from parity import FULL_SCALE, draw_ok, full_scale_err, greedy_agree, sampled_agree
from rpgbarenginecuda_b200 import Model, SampleOptions, Session, counter_uniform, launch_count, synthetic

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", params=["tiny", "tiny_g4", "small"])
def pair(request, tiny_model, tiny_g4_model, small_model):
    path = {"tiny": tiny_model, "tiny_g4": tiny_g4_model, "small": small_model}[request.param]
    m = Model(path, 0, 1024)
    om = OracleModel(path, 1024)
    yield m, om
    m.close()
    om.close()


def check_sampled(oracle, ids, steps, rids, rsteps, opts, seed, start):
    """Sampled tokens against the oracle's; returns how many agree."""
    u = lambda i: counter_uniform(seed, start + i)  # noqa: E731
    ok, n = sampled_agree(ids, rids, lambda i, tok: draw_ok(oracle, steps[i], opts, u(i), tok),
                          lambda i, tok: draw_ok(oracle, rsteps[i], opts, u(i), tok))
    assert ok, (n, list(ids), list(rids))
    for i in range(min(n + 1, len(ids))):
        assert full_scale_err(steps[i], rsteps[i]) <= FULL_SCALE, i
    return n


def test_prefill_logits_and_greedy_32(pair):
    m, om = pair
    toks = synthetic.seeded_tokens(21, 0, m.vocab)
    s, os_ = Session(m, 512), OracleSession(om, 512)
    lg = s.prefill(toks)
    ref = os_.prefill(toks)
    assert full_scale_err(lg, ref) <= FULL_SCALE
    before = launch_count()
    ids, steps = s.generate(SampleOptions(0.0, 0, 1.0), 0, 32, step_logits=True)
    assert launch_count() - before <= 4  # one loop launch for the 32 steps
    rids, rsteps = os_.generate(0.0, 0, 1.0, 0, 32, step_logits=True)
    ok, at = greedy_agree(ids, rids, steps)
    assert ok, (at, ids, rids)
    assert at >= 16 and len(set(ids[:at].tolist())) >= 8, (at, ids)
    for i in range(at):
        assert full_scale_err(steps[i], rsteps[i]) <= FULL_SCALE, i
    assert len(s) == 21 + len(ids)
    s.close()
    os_.close()


def test_multi_round_sampled(pair, oracle):
    """A turn's shape: prefill, then rounds of (sampled decode, append tokens)."""
    m, om = pair
    s, os_ = Session(m, 512), OracleSession(om, 512)
    opts = (0.7, 20, 0.8)
    prompt = synthetic.seeded_tokens(40, 1, m.vocab)
    s.prefill(prompt, want_logits=False)
    os_.prefill(prompt)
    for r in range(3):
        start = len(s)
        ids, steps = s.generate(SampleOptions(*opts), 1234, 16, step_logits=True)
        rids, rsteps = os_.generate(*opts, 1234, 16, step_logits=True)
        n = check_sampled(oracle, ids, steps, rids, rsteps, opts, 1234, start)
        if n < len(rids):
            return  # later steps have different histories
        app = synthetic.seeded_tokens(8, 10 + r, m.vocab)
        lg = s.prefill(app)
        rlg = os_.prefill(app)
        assert full_scale_err(lg, rlg) <= FULL_SCALE
        assert len(s) == len(os_)


def test_bench_mode_64_sampled_steps_one_launch(small_model, oracle):
    """The benchmarked decode mode: 64 steps at T=0.7, top_k=20, top_p=0.8 in one
    loop launch (cross-step weight prefetch, attention chunks held back across
    steps, the in-kernel candidate sampler) after a 300-token prompt."""
    m = Model(small_model, 0, 1024)
    om = OracleModel(small_model, 1024)
    s, os_ = Session(m, 1024), OracleSession(om, 1024)
    prompt = synthetic.seeded_tokens(300, 21, m.vocab)
    s.prefill(prompt, want_logits=False)
    os_.prefill(prompt)
    opts = (0.7, 20, 0.8)
    before = launch_count()
    ids, steps = s.generate(SampleOptions(*opts), 4321, 64, step_logits=True)
    assert launch_count() - before <= 4
    rids, rsteps = os_.generate(*opts, 4321, 64, step_logits=True)
    n = check_sampled(oracle, ids, steps, rids, rsteps, opts, 4321, 300)
    assert n >= 32, (n, list(ids), list(rids))  # a boundary hit this early would be a one-in-millions draw
    s.close()
    m.close()
    os_.close()
    om.close()


def test_stop_token_is_forwarded(pair):
    m, _ = pair
    s = Session(m, 512)
    toks = synthetic.seeded_tokens(21, 0, m.vocab)
    s.prefill(toks)
    free = s.generate(SampleOptions(0.7, 20, 0.8), 77, 12)
    stop_at = int(free[5])
    first = next(i for i, t in enumerate(free) if t == stop_at)
    s.set_len(0)
    s.prefill(toks)
    ids = s.generate(SampleOptions(0.7, 20, 0.8), 77, 12, stop=[stop_at])
    assert list(ids) == list(free[: first + 1])
    assert len(s) == 21 + first + 1


def test_continue_after_generate(pair):
    """generate twice without a prefill in between == one long generate."""
    m, _ = pair
    toks = synthetic.seeded_tokens(30, 4, m.vocab)
    a = Session(m, 512)
    a.prefill(toks)
    one = a.generate(SampleOptions(0.0, 0, 1.0), 0, 20)
    b = Session(m, 512)
    b.prefill(toks)
    two = np.concatenate([b.generate(SampleOptions(0.0, 0, 1.0), 0, 10),
                          b.generate(SampleOptions(0.0, 0, 1.0), 0, 10)])
    assert list(one) == list(two)


@pytest.mark.parametrize("splits", ["1", "2", "3"])
@pytest.mark.parametrize("which", ["tiny", "tiny_g4"])
def test_decode_attention_multi_stage(tiny_model, tiny_g4_model, monkeypatch, splits, which):
    """Decode attention with many chunks per block (and split merges across
    blocks) against the oracle at a context of ~430 positions, for 2 and 4 q
    heads per KV head."""
    monkeypatch.setenv("RPGB_ATTN_SPLITS", splits)
    path = tiny_model if which == "tiny" else tiny_g4_model
    m = Model(path, 0, 512)
    om = OracleModel(path, 512)
    toks = synthetic.seeded_tokens(420, 3, m.vocab)
    s, os_ = Session(m, 512), OracleSession(om, 512)
    s.prefill(toks)
    os_.prefill(toks)
    ids, steps = s.generate(SampleOptions(0.0, 0, 1.0), 0, 12, step_logits=True)
    rids, rsteps = os_.generate(0.0, 0, 1.0, 0, 12, step_logits=True)
    ok, at = greedy_agree(ids, rids, steps)
    assert ok, (splits, at)
    for i in range(at):
        assert full_scale_err(steps[i], rsteps[i]) <= FULL_SCALE, (splits, i)
    s.close()
    m.close()
    om.close()


@pytest.mark.parametrize("opts", [(1.0, 0, 0.95), (0.7, 100, 0.9), (1.3, 1, 1.0)])
def test_sampled_general_paths(pair, oracle, opts):
    """Sampling options the candidate fast path does not take (top_k off, above
    64, or 1 = off with plain temperature): the decode loop's general sampler,
    one launch for all steps, against the oracle."""
    m, om = pair
    s, os_ = Session(m, 512), OracleSession(om, 512)
    prompt = synthetic.seeded_tokens(33, 7, m.vocab)
    s.prefill(prompt, want_logits=False)
    os_.prefill(prompt)
    ids, steps = s.generate(SampleOptions(*opts), 99, 16, step_logits=True)
    rids, rsteps = os_.generate(*opts, 99, 16, step_logits=True)
    check_sampled(oracle, ids, steps, rids, rsteps, opts, 99, 33)
    s.close()
    os_.close()


def test_many_stop_ids(pair):
    """More stop ids than the device-side list holds: the host checks them and
    the session length and continuation still follow the reference loop."""
    m, _ = pair
    s = Session(m, 512)
    toks = synthetic.seeded_tokens(21, 0, m.vocab)
    s.prefill(toks)
    free = s.generate(SampleOptions(0.7, 20, 0.8), 77, 12)
    stop_at = int(free[6])
    first = next(i for i, t in enumerate(free) if t == stop_at)
    stops = [stop_at] + [int(v) for v in synthetic.seeded_tokens(24, 9, m.vocab) if int(v) not in set(free.tolist())][:20]
    assert len(stops) > 16
    s.set_len(0)
    s.prefill(toks)
    ids = s.generate(SampleOptions(0.7, 20, 0.8), 77, 12, stop=stops)
    assert list(ids) == list(free[: first + 1])
    assert len(s) == 21 + first + 1
    s.close()


def test_multi_launch_path(pair, monkeypatch):
    """The per-step graph path (kept for group sizes the decode loop kernel is
    not built for), forced on a supported model: greedy tokens and step logits
    against the oracle."""
    monkeypatch.setenv("RPGB_DECODE_GRAPH", "1")
    m, om = pair
    toks = synthetic.seeded_tokens(21, 0, m.vocab)
    s, os_ = Session(m, 512), OracleSession(om, 512)
    s.prefill(toks)
    os_.prefill(toks)
    ids, steps = s.generate(SampleOptions(0.0, 0, 1.0), 0, 16, step_logits=True)
    rids, rsteps = os_.generate(0.0, 0, 1.0, 0, 16, step_logits=True)
    ok, at = greedy_agree(ids, rids, steps)
    assert ok, (at, ids, rids)
    for i in range(at):
        assert full_scale_err(steps[i], rsteps[i]) <= FULL_SCALE
    s.close()
    os_.close()
