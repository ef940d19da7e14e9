"""Parity criteria and inputs shared by the tests and the golden-fixture
scripts (not a test module).

Criteria are the reference's own:
* logits: max|d| <= 1e-3 * max|ref| (tests/cmp_gen.py:63-82, full_scale_err);
* greedy tokens: identical; a divergence is acceptable only where the two
  tokens' logits differ by <= 1e-2 of the logit span (tests/cmp_gen.py:186-211),
  and the comparison of later steps stops there (their histories differ);
* sampled tokens on the same logits: identical; a divergence only where u
  lies within 1e-6 of a cumulative-probability boundary (tests/cmp_sample.py
  criterion 3);
* sampled tokens after the model: the two sides' logits differ by float
  rounding, so a draw near a cumulative boundary can select different tokens
  (the reference's own tools/gen_sample_check.cu:6-9 declines token identity
  there for this reason).  Tokens must agree up to the first divergence; there
  each side's token must be the draw the checker's sampler (pinned to the
  reference's sampler on identical logits) makes from that side's own logits
  with the same u, and the logits themselves are held to the 1e-3 full-scale
  bound -- so a divergence is explained exactly by the logit difference.  The
  comparison stops there (later steps have different histories);
* filtered distributions: within 1e-5 of full scale and the same kept set
  (tests/cmp_sample.py criterion 2).
"""

import numpy as np

FULL_SCALE = 1e-3
GAP = 1e-2
MASK = (1 << 64) - 1

# (temperature, top_k, top_p, seed, tie) -- the reference's sample_check case
# matrix (tools/sample_check.cu:71-84)
REF_CASES = [
    (0.0, 0, 1.0, 11, False), (0.0, 8, 0.9, 12, False), (1.0, 0, 1.0, 13, False), (0.7, 40, 1.0, 14, False),
    (1.3, 0, 0.9, 15, False), (0.5, 20, 0.95, 16, False), (1.0, 2, 1.0, 17, False), (1.0, 0, 0.05, 18, False),
    (0.001, 0, 1.0, 19, False), (5.0, 0, 1.0, 20, False), (1.0, 8, 1.0, 21, True), (0.0, 0, 1.0, 22, True),
]
# the operator sweep of the sampler: T in {0, 0.7, 1.0} x top_k in {0, 2, 20, 40}
# x top_p in {1.0, 0.8, 0.95}
SWEEP_CASES = [(t, k, p, 100 + i, False) for i, (t, k, p) in enumerate(
    (t, k, p) for t in (0.0, 0.7, 1.0) for k in (0, 2, 20, 40) for p in (1.0, 0.8, 0.95))]


def ref_case_logits(seed, tie, n):
    """The logits of tools/sample_check.cu:94-105: SplitMix64 -> [-8, 8), 1/8 grid for ties."""
    idx = np.arange(n, dtype=np.uint64)
    x = (np.uint64(seed) * np.uint64(1000003) + idx).astype(np.uint64)
    x = x + np.uint64(0x9E3779B97F4A7C15)
    x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    x = x ^ (x >> np.uint64(31))
    u = (x >> np.uint64(40)).astype(np.float32) * np.float32(1.0 / 16777216.0)
    v = (u - np.float32(0.5)) * np.float32(16.0)
    if tie:
        v = np.round(v * np.float32(8.0)) / np.float32(8.0)
    return v.astype(np.float32)


def sweep_logits(seed, n):
    """Sampler sweep input: N(0, 3^2)."""
    return (np.random.default_rng(seed).standard_normal(n) * 3.0).astype(np.float32)


def case_logits(case, n):
    t, k, p, seed, tie = case
    return ref_case_logits(seed, tie, n) if case in REF_CASES else sweep_logits(seed, n)


def near_boundary(probs, u, tol=1e-6):
    cum = np.cumsum(probs.astype(np.float64))
    return bool(np.min(np.abs(cum - u)) < tol)


def full_scale_err(ours, ref):
    return float(np.abs(np.asarray(ours, np.float64) - ref).max() / np.abs(ref).max())


def greedy_agree(ours, ref, ours_steps):
    """(ok, n): ours == ref for the first n tokens; a first divergence at n is ok
    only when the two tokens' logits (ours) differ by <= GAP of the span."""
    for i, (a, b) in enumerate(zip(ours, ref)):
        if a != b:
            row = np.asarray(ours_steps[i], np.float64)
            span = row.max() - row.min()
            return abs(row[int(a)] - row[int(b)]) <= GAP * span, i
    return len(ours) == len(ref), min(len(ours), len(ref))


def draw_ok(oracle, row, opts, u, tok):
    """tok is the token the checker's sampler draws from logits row with u
    (or u lies within 1e-6 of a boundary of that distribution)."""
    t, k, p = opts
    row = np.ascontiguousarray(row, dtype=np.float32)
    if oracle.sample_token(row, t, k, p, u) == int(tok):
        return True
    return near_boundary(oracle.filter_to_probs(row, t, k, p), u)


def sampled_agree(ours, ref, ours_ok, ref_ok):
    """(ok, n): ours == ref for the first n tokens; at a first divergence n,
    ours_ok(n, token) and ref_ok(n, token) must both hold (each side drew its
    token correctly from its own logits)."""
    for i, (a, b) in enumerate(zip(ours, ref)):
        if a != b:
            return bool(ours_ok(i, a) and ref_ok(i, b)), i
    return len(ours) == len(ref), min(len(ours), len(ref))


# ---------------------------------------------------------------- stored rows
#
# A logits row is stored as its full-scale value, its 32 largest entries and
# fixed random indices; the full-scale check runs on those entries.

def row_indices(vocab, n_random, seed):
    return np.sort(np.random.default_rng(seed).choice(vocab, size=n_random, replace=False)).astype(np.int32)


def pack_row(row, rand_idx, top=32):
    row = np.asarray(row, np.float32)
    top_idx = np.argsort(-row, kind="stable")[:top].astype(np.int32)
    return {"scale": np.float32(np.abs(row).max()), "top_idx": top_idx, "top_val": row[top_idx],
            "rand_val": row[rand_idx]}


def packed_err(ours_row, scale, top_idx, top_val, rand_idx, rand_val):
    """max|ours - ref| over the stored entries / the reference's full scale."""
    o = np.asarray(ours_row, np.float64)
    d = max(np.abs(o[top_idx] - top_val).max(), np.abs(o[rand_idx] - rand_val).max())
    return float(d / scale)


def store_rows(out, key, rows, rand_idx):
    packs = [pack_row(r, rand_idx) for r in rows]
    out[f"{key}/scale"] = np.array([p["scale"] for p in packs], np.float32)
    out[f"{key}/top_idx"] = np.stack([p["top_idx"] for p in packs])
    out[f"{key}/top_val"] = np.stack([p["top_val"] for p in packs])
    out[f"{key}/rand_val"] = np.stack([p["rand_val"] for p in packs])


def row_err(fix, key, i, ours_row, rand_idx):
    return packed_err(ours_row, float(fix[f"{key}/scale"][i]), fix[f"{key}/top_idx"][i], fix[f"{key}/top_val"][i],
                      rand_idx, fix[f"{key}/rand_val"][i])


def top_row(fix, key, i, vocab):
    """Stored row i with only its top entries (the rest -inf): enough to
    recompute a top_k <= 32 filtered distribution exactly."""
    row = np.full(vocab, -np.inf, dtype=np.float32)
    row[fix[f"{key}/top_idx"][i]] = fix[f"{key}/top_val"][i]
    return row


def kept_probs(fix, key, i, vocab):
    """The stored filtered distribution (kept entries) of sampled step i, as a dense row."""
    off = fix[f"{key}/kept_off"]
    p = np.zeros(vocab, np.float64)
    p[fix[f"{key}/kept_idx"][off[i]:off[i + 1]]] = fix[f"{key}/kept_p"][off[i]:off[i + 1]]
    return p


def store_kept(out, key, probs_rows):
    ks = []
    for p in probs_rows:
        idx = np.nonzero(p)[0].astype(np.int32)
        ks.append((idx, np.asarray(p)[idx].astype(np.float32)))
    out[f"{key}/kept_off"] = np.cumsum([0] + [len(x[0]) for x in ks]).astype(np.int32)
    out[f"{key}/kept_idx"] = np.concatenate([x[0] for x in ks])
    out[f"{key}/kept_p"] = np.concatenate([x[1] for x in ks])
