"""Tensor parallelism on the GPU: the split model against the one-GPU engine
and against the CPU oracle.

Parity rule for the split (the 8B tensor-parallel plan): logits within 1e-3
of full scale of the one-GPU run and the same tokens, a divergence tolerated
only at a top-2 tie of the reference's logits (the forward tests' rule).
Every split run is also held to the oracle directly (tests/parity.py's
criteria: logits within 1e-3 of full scale, greedy tokens identical up to a
gap-rule divergence, sampled tokens identical up to a divergence where each
side's token is the checker's draw from its own logits).
* TP = 1 through an NCCL group of one rank: the same shard code path
  (partials, sum, residual add, gathered logits, sampler on the gathered row,
  the decode loop's candidate exchange) on one GPU, so the driver's one-GPU
  run covers it.
* TP = 2, 4 and 8 where the box has the GPUs: one process per GPU
  (tests/tp_worker.py), NVLS off, each process under a time limit; the
  "wide" model (the 8B model's widths, two layers) splits like the 8B plan
  over up to eight ranks.
"""

import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from parity import draw_ok, greedy_agree, near_boundary, sampled_agree
from rpgbarenginecuda_b200 import Model, TpGroup, counter_uniform, synthetic

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from tp_worker import run  # noqa: E402

FULL_SCALE = 1e-3


def full_scale_err(ours, ref):
    return float(np.abs(ours.astype(np.float64) - ref).max() / np.abs(ref).max())


def check_loop_sampled(got, oracle):
    """The decode loop's sampled tokens (no step logits) against the same
    round through the step graph: identical, or a first divergence where the
    draw lies within 1e-4 of a boundary of the graph run's distribution (the
    two paths' logits differ at the 1e-6 level)."""
    loop, graph, steps = got["sampled_loop"], got["sampled"], got["sampled_steps"]
    start = int(got["sampled_start"])
    assert len(loop) == len(graph)
    for i in range(len(loop)):
        if loop[i] != graph[i]:
            probs = oracle.filter_to_probs(np.ascontiguousarray(steps[i], np.float32), 0.7, 20, 0.8)
            assert near_boundary(probs, counter_uniform(1234, start + i), 1e-4), (i, list(loop), list(graph))
            return


def check_same(got, ref):
    assert full_scale_err(got["prefill"], ref["prefill"]) <= FULL_SCALE
    assert full_scale_err(got["short_prefill"], ref["short_prefill"]) <= FULL_SCALE
    for key in ("greedy", "sampled"):
        ids, rids, rsteps = got[key], ref[key], ref[key + "_steps"]
        n = min(len(ids), len(rids))
        for i in range(n):
            if ids[i] != rids[i]:
                top2 = np.sort(rsteps[i])[-2:]
                gap = (top2[1] - top2[0]) / (rsteps[i].max() - rsteps[i].min())
                assert gap <= 1e-2, (key, i, ids, rids)
                return
            assert full_scale_err(got[key + "_steps"][i], rsteps[i]) <= FULL_SCALE, (key, i)
        assert len(ids) == len(rids), key
    assert int(got["len"]) == int(ref["len"])
    # the one-launch loop: same greedy tokens as the reference's loop (ties as above)
    loop, rloop = got["greedy_loop"], ref["greedy_loop"]
    for i in range(min(len(loop), len(rloop))):
        if loop[i] != rloop[i]:
            row = ref["greedy_steps"][i]
            top2 = np.sort(row)[-2:]
            assert (top2[1] - top2[0]) / (row.max() - row.min()) <= 1e-2, ("loop", i, loop, rloop)
            return
    assert len(loop) == len(rloop)
    assert np.array_equal(got["greedy_loop2"], ref["greedy_loop2"])
    assert int(got["len_loop"]) == int(ref["len_loop"])


_ORACLE = {}


def oracle_run(path, max_seq=512):
    """The calls of tests/tp_worker.py's run(), made on the CPU oracle (cached per model)."""
    if path not in _ORACLE:
        from oracle.oracle import OracleModel, OracleSession

        om = OracleModel(path, 1024)
        s = OracleSession(om, max_seq)
        out = {"prefill": s.prefill(synthetic.seeded_tokens(21, 0, om.vocab))}
        out["greedy"], out["greedy_steps"] = s.generate(0.0, 0, 1.0, 0, 32, step_logits=True)
        s.prefill(synthetic.seeded_tokens(40, 1, om.vocab))
        out["sampled_start"] = len(s)
        out["sampled"], out["sampled_steps"] = s.generate(0.7, 20, 0.8, 1234, 24, step_logits=True)
        out["short_prefill"] = s.prefill(synthetic.seeded_tokens(5, 2, om.vocab))
        s.close()
        om.close()
        _ORACLE[path] = out
    return _ORACLE[path]


def check_oracle(got, ref, oracle):
    """A run of tests/tp_worker.py's calls against the oracle's; comparisons
    stop at a tolerated divergence (the histories differ after it)."""
    assert full_scale_err(got["prefill"], ref["prefill"]) <= FULL_SCALE
    ok, n = greedy_agree(got["greedy"], ref["greedy"], got["greedy_steps"])
    assert ok, ("greedy", n, list(got["greedy"]), list(ref["greedy"]))
    for i in range(n):
        assert full_scale_err(got["greedy_steps"][i], ref["greedy_steps"][i]) <= FULL_SCALE, ("greedy", i)
    if n < len(ref["greedy"]):
        return
    opts, start = (0.7, 20, 0.8), int(ref["sampled_start"])
    u = lambda i: counter_uniform(1234, start + i)  # noqa: E731
    ok, n = sampled_agree(got["sampled"], ref["sampled"],
                          lambda i, t: draw_ok(oracle, got["sampled_steps"][i], opts, u(i), t),
                          lambda i, t: draw_ok(oracle, ref["sampled_steps"][i], opts, u(i), t))
    assert ok, ("sampled", n, list(got["sampled"]), list(ref["sampled"]))
    for i in range(min(n + 1, len(got["sampled"]))):
        assert full_scale_err(got["sampled_steps"][i], ref["sampled_steps"][i]) <= FULL_SCALE, ("sampled", i)
    if n == len(ref["sampled"]):
        assert full_scale_err(got["short_prefill"], ref["short_prefill"]) <= FULL_SCALE


@pytest.fixture(scope="module", params=["tiny", "tiny_g4", "small", "wide"])
def model_path(request, tiny_model, tiny_g4_model, small_model, wide_model):
    return {"tiny": tiny_model, "tiny_g4": tiny_g4_model, "small": small_model, "wide": wide_model}[request.param]


def test_tp1_group_matches_one_gpu(model_path, oracle):
    m = Model(model_path, 0, 1024)
    ref = run(m)
    m.close()
    g = TpGroup(TpGroup.unique_id(), 0, 1, 0)
    mt = Model(model_path, 0, 1024, tp=g)
    got = run(mt, attach=True)
    mt.close()
    g.close()
    check_same(got, ref)
    # the prefill is the same kernels in both; only the residual add is a separate launch
    assert full_scale_err(got["prefill"], ref["prefill"]) <= 1e-6
    check_oracle(ref, oracle_run(model_path), oracle)
    check_oracle(got, oracle_run(model_path), oracle)
    check_loop_sampled(ref, oracle)
    check_loop_sampled(got, oracle)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("size", [2, 4, 8])
def test_tp_ranks_match_one_gpu(model_path, size, tmp_path, oracle):
    if torch.cuda.device_count() < size:
        pytest.skip(f"needs {size} GPUs")
    base = os.path.basename(model_path)
    if ("tiny" in base and size > 2) or ("small" in base and size > 4):
        pytest.skip("the model does not split over that many ranks (whole super-blocks per rank)")
    port, out = _free_port(), str(tmp_path / "tp.npz")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "tp_worker.py"), "--model", model_path,
                               "--rank", str(r), "--size", str(size), "--port", str(port), "--out", out],
                              env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT) for r in range(size)]
    logs = []
    for p in procs:
        try:
            o, _ = p.communicate(timeout=300)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        logs.append(o.decode(errors="replace")[-2000:])
    assert all(p.returncode == 0 for p in procs), logs
    got = dict(np.load(out))
    check_oracle(got, oracle_run(model_path), oracle)
    check_loop_sampled(got, oracle)
    m = Model(model_path, 0, 1024)
    ref = run(m)
    m.close()
    check_same(got, ref)
