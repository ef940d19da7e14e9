"""Writes tests/golden/ref_engine.npz and tests/golden/ref_sampler.npz: outputs
of the reference's own engine and sampler on fixed synthetic inputs.

The reference is compiled from its sources (CUDA files included) for the host
CPU by oracle/Makefile into oracle/_ref/libref_emu.so (the SIMT emulation
layer of oracle/emu); no GPU is used.  Inputs:

* engine runs on synthetic GGUFs written by rpgbarenginecuda_b200.synthetic
  (their digests are stored, so a test notices a changed writer):
  - the toy models tiny (G = 2), tiny-g4 (G = 4) and small (16 heads) with
    weights N(0, 0.06), whose greedy output does not settle on one token:
      greedy: 21-id prompt (seed 0), prefill logits, the residual stream after
              every layer (GpuForwardOptions::capture_hidden), 32 greedy
              tokens with every step's logits;
      turns:  40-id prompt (seed 1), then 3 rounds of 16 tokens sampled at
              T = 0.7, top_k = 20, top_p = 0.8 (seed 1234), 9 appended ids
              (seeds 10, 11) between rounds, with step logits, each step's
              filtered distribution (its kept entries) and the appended
              prefills' logits;
  - the 0.6B configuration (28 layers, hidden 1024, weights N(0, 0.02)):
    21-id prompt (seed 0) and 32 greedy tokens;
* the sampler on the logits of tools/sample_check.cu (its 12-case matrix) and
  on N(0, 3^2) logits (the 36-case operator sweep) at V = 4096 and 151936,
  counters 0..15 (tokens; the filtered distribution at V = 4096).

Logits rows are stored as in tests/parity.py (full scale, top entries, fixed
random entries).  Rerun after changing the inputs (about 7 minutes on 8
cores):
    make -C oracle && python tests/golden/make_ref_fixtures.py
"""

import os
import sys
import time
from dataclasses import replace

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

from oracle.oracle import RefEmu  # noqa: E402
from parity import REF_CASES, SWEEP_CASES, case_logits, row_indices, store_kept, store_rows  # noqa: E402
from rpgbarenginecuda_b200 import synthetic  # noqa: E402

TOY = [("tiny", 1), ("tiny-g4", 2), ("small", 3)]
TOY_STD = 0.06
SAMPLE = (0.7, 20, 0.8)
SAMPLE_SEED = 1234


def toy_shape(name):
    return replace(synthetic.PRESETS[name], weight_std=TOY_STD)


def engine_runs(ref, out):
    for name, seed in TOY:
        sh = toy_shape(name)
        path = synthetic.cached_model(sh, seed=seed)
        V = sh.vocab
        rand_idx = row_indices(V, 224, seed)
        key = f"{name}"
        out[f"{key}/digest"] = np.array(synthetic.file_digest(path))
        out[f"{key}/rand_idx"] = rand_idx
        # greedy
        s = ref.session(path, 1024, 512)
        toks = synthetic.seeded_tokens(21, 0, V)
        lg, hid = s.prefill(toks, V, n_layers=sh.n_layers, hidden=sh.hidden)
        ids, steps = s.generate(0.0, 0, 1.0, 0, 32, V, step_logits=True)
        out[f"{key}/greedy/prompt"] = toks
        if name == "tiny-g4":
            out[f"{key}/greedy/hidden"] = hid
        store_rows(out, f"{key}/greedy/prefill", [lg], rand_idx)
        out[f"{key}/greedy/ids"] = ids
        store_rows(out, f"{key}/greedy/steps", steps, rand_idx)
        assert len(s) == 21 + len(ids)
        s.close()
        # turns: prompt, then rounds of sampled decode with appended ids between them
        s = ref.session(path, 1024, 512)
        prompt = synthetic.seeded_tokens(40, 1, V)
        lg = s.prefill(prompt, V)
        out[f"{key}/turns/prompt"] = prompt
        store_rows(out, f"{key}/turns/prefill0", [lg], rand_idx)
        for r in range(3):
            start = len(s)
            ids, steps = s.generate(*SAMPLE, SAMPLE_SEED, 16, V, step_logits=True)
            out[f"{key}/turns/r{r}/start"] = np.int64(start)
            out[f"{key}/turns/r{r}/ids"] = ids
            store_rows(out, f"{key}/turns/r{r}/steps", steps, rand_idx)
            store_kept(out, f"{key}/turns/r{r}",
                       [ref.sample(steps[i], *SAMPLE, SAMPLE_SEED, start + i, want_probs=True)[1]
                        for i in range(len(ids))])
            if r < 2:
                app = synthetic.seeded_tokens(9, 10 + r, V)
                lg = s.prefill(app, V)
                out[f"{key}/turns/r{r}/append"] = app
                store_rows(out, f"{key}/turns/r{r}/append_logits", [lg], rand_idx)
        s.close()
        print(f"{name}: done", flush=True)

    # the 0.6B configuration
    path = synthetic.cached_model("qwen3-0.6b", seed=0)
    V = 151936
    rand_idx = row_indices(V, 480, 0)
    out["qwen3-0.6b/digest"] = np.array(synthetic.file_digest(path))
    out["qwen3-0.6b/rand_idx"] = rand_idx
    s = ref.session(path, 4096, 4096)
    toks = synthetic.seeded_tokens(21, 0, V)
    lg = s.prefill(toks, V)
    ids, steps = s.generate(0.0, 0, 1.0, 0, 32, V, step_logits=True)
    out["qwen3-0.6b/greedy/prompt"] = toks
    store_rows(out, "qwen3-0.6b/greedy/prefill", [lg], rand_idx)
    out["qwen3-0.6b/greedy/ids"] = ids
    store_rows(out, "qwen3-0.6b/greedy/steps", steps, rand_idx)
    s.close()
    print("qwen3-0.6b: done", flush=True)


def sampler_runs(ref, out):
    cases = REF_CASES + SWEEP_CASES
    out["cases"] = np.array([[t, k, p, seed, int(tie)] for t, k, p, seed, tie in cases], np.float64)
    for V in (4096, 151936):
        toks = np.zeros((len(cases), 16), np.int32)
        for ci, case in enumerate(cases):
            t, k, p, seed, tie = case
            lg = case_logits(case, V)
            for c in range(16):
                toks[ci, c], probs = ref.sample(lg, t, k, p, seed, c, want_probs=(c == 0 and V == 4096))
                if probs is not None and ci < len(REF_CASES):
                    out[f"probs_{ci}"] = probs
        out[f"tokens_{V}"] = toks
        print(f"sampler V={V}: done", flush=True)


def main():
    ref = RefEmu()
    t0 = time.time()
    out = {}
    sampler_runs(ref, out)
    np.savez_compressed(os.path.join(HERE, "ref_sampler.npz"), **out)
    out = {}
    engine_runs(ref, out)
    np.savez_compressed(os.path.join(HERE, "ref_engine.npz"), **out)
    print(f"fixtures written in {time.time() - t0:.0f} s")


if __name__ == "__main__":
    main()
