"""Writes tests/golden/oracle_configs.npz: the CPU oracle's outputs on the
benchmark configurations, for GPU tests at full size.

The oracle (oracle/rpg_oracle.c) is pinned to the reference's own outputs by
tests/test_ref_fixtures.py; the reference itself, run on the host through the
SIMT emulation layer, would take hours for a 2811-token prefill, so these
larger runs come from the oracle:

* 1.7B (28 layers, hidden 2048, V = 151936), the benchmark turn with shorter
  rounds: the 2811-id prompt of the benchmark (seed 1000) with its prefill
  logits, then 3 rounds of 16 tokens sampled at T = 0.7, top_k = 20,
  top_p = 0.8 (seed 1234) with every step's logits, separated by the
  benchmark's 40-id appends (seeds 2000, 2001) and their prefill logits;
* 4B (36 layers, hidden 2560, 32 query heads over 8 KV heads: G = 4): a
  3840-id prompt (seed 7) and 8 greedy tokens with step logits, attention
  over a context of 3840 positions; and a 512-id prompt (seed 8) with 8
  greedy tokens.

Rows are stored as in tests/parity.py (full scale, top entries, fixed random
entries); the sampled steps also keep the oracle's filtered distribution
(kept entries).  Rerun after changing the oracle or the inputs:
    make -C oracle && python tests/golden/make_oracle_fixtures.py [1.7b] [4b]
"""

import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

from oracle.oracle import Oracle, OracleModel, OracleSession  # noqa: E402
from parity import row_indices, store_kept, store_rows  # noqa: E402
from rpgbarenginecuda_b200 import synthetic  # noqa: E402

OUT = os.path.join(HERE, "oracle_configs.npz")
SAMPLE = (0.7, 20, 0.8)
SAMPLE_SEED = 1234


def run_17b(out):
    o = Oracle()
    path = synthetic.cached_model("qwen3-1.7b", seed=0)
    V = 151936
    rand_idx = row_indices(V, 480, 17)
    k = "qwen3-1.7b"
    out[f"{k}/digest"] = np.array(synthetic.file_digest(path))
    out[f"{k}/rand_idx"] = rand_idx
    om = OracleModel(path, 4096)
    s = OracleSession(om, 4096)
    prompt = synthetic.seeded_tokens(2811, 1000, V)
    t0 = time.time()
    lg = s.prefill(prompt)
    print(f"1.7b prefill {time.time() - t0:.0f} s", flush=True)
    out[f"{k}/prompt"] = prompt
    store_rows(out, f"{k}/prefill", [lg], rand_idx)
    for r in range(3):
        start = len(s)
        ids, steps = s.generate(*SAMPLE, SAMPLE_SEED, 16, step_logits=True)
        out[f"{k}/r{r}/start"] = np.int64(start)
        out[f"{k}/r{r}/ids"] = ids
        store_rows(out, f"{k}/r{r}/steps", steps, rand_idx)
        store_kept(out, f"{k}/r{r}", [o.filter_to_probs(row, *SAMPLE) for row in steps])
        if r < 2:
            app = synthetic.seeded_tokens(40, 2000 + r, V)
            lg = s.prefill(app)
            out[f"{k}/r{r}/append"] = app
            store_rows(out, f"{k}/r{r}/append_logits", [lg], rand_idx)
        print(f"1.7b round {r} {time.time() - t0:.0f} s", flush=True)
    s.close()
    om.close()


def run_4b(out):
    path = synthetic.cached_model("qwen3-4b", seed=0)
    V = 151936
    rand_idx = row_indices(V, 480, 4)
    k = "qwen3-4b"
    out[f"{k}/digest"] = np.array(synthetic.file_digest(path))
    out[f"{k}/rand_idx"] = rand_idx
    om = OracleModel(path, 4096)
    for ctx, seed in ((512, 8), (3840, 7)):
        t0 = time.time()
        s = OracleSession(om, 4096)
        prompt = synthetic.seeded_tokens(ctx, seed, V)
        lg = s.prefill(prompt)
        ids, steps = s.generate(0.0, 0, 1.0, 0, 8, step_logits=True)
        out[f"{k}/ctx{ctx}/prompt"] = prompt
        store_rows(out, f"{k}/ctx{ctx}/prefill", [lg], rand_idx)
        out[f"{k}/ctx{ctx}/ids"] = ids
        store_rows(out, f"{k}/ctx{ctx}/steps", steps, rand_idx)
        s.close()
        print(f"4b ctx {ctx} {time.time() - t0:.0f} s", flush=True)
    om.close()


def main():
    which = sys.argv[1:] or ["1.7b", "4b"]
    out = dict(np.load(OUT)) if os.path.exists(OUT) else {}
    if "1.7b" in which:
        out = {k: v for k, v in out.items() if not k.startswith("qwen3-1.7b/")}
        run_17b(out)
        np.savez_compressed(OUT, **out)
    if "4b" in which:
        out = {k: v for k, v in out.items() if not k.startswith("qwen3-4b/")}
        run_4b(out)
        np.savez_compressed(OUT, **out)


if __name__ == "__main__":
    main()
