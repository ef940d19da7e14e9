"""Q5_K and Q8_0 on the GPU: dequant (bit-exact), matvec / GEMM and whole
models against the CPU oracle.

The reference's host dequantiser covers these types (src/quant.cc:29-45,
132-141, 281-313); its GPU loader rejects them (src/gpu_model.cu:26-38).
Here they run on the same kernels as Q4_K / Q6_K: one byte per weight in
the block group, the integer tensor-core units (u8 x s8 for Q5_K, s8 x s8
for Q8_0), the tcgen05 GEMM's dequant split from 16 tokens.  The oracle's
dequant of both types is pinned to src/quant.cc (tests/test_oracle_pins.py);
criteria as everywhere (tests/parity.py).
"""

from dataclasses import replace

import numpy as np
import pytest

from oracle.oracle import OracleModel, OracleSession
from parity import FULL_SCALE, draw_ok, full_scale_err, greedy_agree, sampled_agree
from rpgbarenginecuda_b200 import GGML_Q5_K, GGML_Q8_0, Matrix, Model, SampleOptions, Session, counter_uniform, \
    launch_count, synthetic

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

QT = {GGML_Q5_K: "q5_k", GGML_Q8_0: "q8_0"}


def make_matrix(qtype, rows, cols, seed):
    return synthetic.quantize(synthetic.normal(seed, rows * cols, 0.0, 0.02), QT[qtype])


@pytest.mark.parametrize("qtype", [GGML_Q5_K, GGML_Q8_0])
@pytest.mark.parametrize("rows,cols", [(8, 256), (64, 2048), (33, 6144)])
def test_dequant_bitexact(oracle, qtype, rows, cols):
    b = make_matrix(qtype, rows, cols, rows + cols)
    m = Matrix(qtype, rows, cols, b)
    out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    m.dequant(0, rows, out.data_ptr())
    torch.cuda.synchronize()
    ref = oracle.dequant(qtype, b, rows * cols)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    m.close()


@pytest.mark.parametrize("qtype", [GGML_Q5_K, GGML_Q8_0])
@pytest.mark.parametrize("rows,cols", [(2048, 2048), (2048, 6144), (9728, 2560)])
@pytest.mark.parametrize("n_tok", [1, 2, 5, 15, 64, 200])
def test_matvec_vs_oracle(oracle, qtype, rows, cols, n_tok):
    b = make_matrix(qtype, rows, cols, 17)
    x = synthetic.normal(99, n_tok * cols, 0.0, 1.0).reshape(n_tok, cols)
    m = Matrix(qtype, rows, cols, b)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty((n_tok, rows), dtype=torch.float32, device="cuda")
    m.matvec(xd.data_ptr(), n_tok, out.data_ptr())
    torch.cuda.synchronize()
    ref = oracle.matvec(qtype, b, rows, cols, x)
    err = np.abs(out.cpu().numpy() - ref).max() / np.abs(ref).max()
    tol = 5e-5 if n_tok >= 16 and rows % 128 == 0 else 2e-5
    assert err < tol, err
    m.close()


@pytest.fixture(scope="module", params=["q5_k_m", "q8_0"])
def mixed_pair(request, model_cache):
    path = synthetic.cached_model(replace(synthetic.PRESETS["tiny"], weight_std=0.06, mix=request.param), seed=5,
                                  cache_dir=model_cache)
    m = Model(path, 0, 1024)
    om = OracleModel(path, 1024)
    yield m, om
    m.close()
    om.close()


def test_model_greedy_and_sampled(mixed_pair, oracle):
    """A two-layer model in the Q5_K_M or Q8_0 mix: prefill logits, 24 greedy
    steps and 16 sampled steps (T = 0.7, top_k 20, top_p 0.8), each generate
    call one decode-loop launch, against the oracle."""
    m, om = mixed_pair
    toks = synthetic.seeded_tokens(21, 0, m.vocab)
    s, os_ = Session(m, 512), OracleSession(om, 512)
    assert full_scale_err(s.prefill(toks), os_.prefill(toks)) <= FULL_SCALE
    before = launch_count()
    ids, steps = s.generate(SampleOptions(0.0, 0, 1.0), 0, 24, step_logits=True)
    assert launch_count() - before <= 4
    rids, rsteps = os_.generate(0.0, 0, 1.0, 0, 24, step_logits=True)
    ok, at = greedy_agree(ids, rids, steps)
    assert ok and at >= 8, (at, list(ids), list(rids))
    for i in range(at):
        assert full_scale_err(steps[i], rsteps[i]) <= FULL_SCALE, i
    if at < len(rids):
        return
    start = len(s)
    opts = (0.7, 20, 0.8)
    ids, steps = s.generate(SampleOptions(*opts), 7, 16, step_logits=True)
    rids, rsteps = os_.generate(*opts, 7, 16, step_logits=True)
    u = lambda i: counter_uniform(7, start + i)  # noqa: E731
    ok, n = sampled_agree(ids, rids, lambda i, t: draw_ok(oracle, steps[i], opts, u(i), t),
                          lambda i, t: draw_ok(oracle, rsteps[i], opts, u(i), t))
    assert ok, (n, list(ids), list(rids))
    for i in range(min(n + 1, len(ids))):
        assert full_scale_err(steps[i], rsteps[i]) <= FULL_SCALE, i
    s.close()
    os_.close()
