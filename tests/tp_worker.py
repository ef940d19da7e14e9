"""One rank of the tensor-parallel GPU test (tests/test_gpu_tp.py).

Joins a gloo group on 127.0.0.1 to pass rank 0's NCCL id, loads its shard of
the model on GPU `rank`, runs the same calls as the one-GPU reference run of
the test (prefill with logits, 32 greedy steps with per-step logits, a
sampled append-and-decode round) and, on rank 0, saves what it got.
"""

import argparse
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

from rpgbarenginecuda_b200 import Model, SampleOptions, Session, TpGroup, synthetic  # noqa: E402


def run(m, max_seq=512, attach=False):
    """The calls both the tensor-parallel ranks and the one-GPU reference make.

    The greedy run with per-step logits goes through the step graph (NCCL
    between launches when split); the second session's greedy runs are the
    one-launch decode loop (partials exchanged between the GPUs once
    attached), and its second generate call starts from the logits gathered
    after the first."""
    s = Session(m, max_seq)
    toks = synthetic.seeded_tokens(21, 0, m.vocab)
    out = {"prefill": s.prefill(toks)}
    ids, steps = s.generate(SampleOptions(0.0, 0, 1.0), 0, 32, step_logits=True)
    out["greedy"], out["greedy_steps"] = np.asarray(ids), np.asarray(steps)
    app = synthetic.seeded_tokens(40, 1, m.vocab)
    s.prefill(app, want_logits=False)
    out["sampled_start"] = np.asarray(len(s))
    sids, ssteps = s.generate(SampleOptions(0.7, 20, 0.8), 1234, 24, step_logits=True)
    out["sampled"], out["sampled_steps"] = np.asarray(sids), np.asarray(ssteps)
    # a short prompt (fewer than 16 tokens) takes the per-token matvec prefill
    out["short_prefill"] = s.prefill(synthetic.seeded_tokens(5, 2, m.vocab))
    out["len"] = np.asarray(len(s))
    s.close()
    s2 = Session(m, max_seq)
    if attach:
        s2.attach_tp()
    s2.prefill(toks, want_logits=False)
    out["greedy_loop"] = np.asarray(s2.generate(SampleOptions(0.0, 0, 1.0), 0, 32))
    out["greedy_loop2"] = np.asarray(s2.generate(SampleOptions(0.0, 0, 1.0), 0, 16))
    out["len_loop"] = np.asarray(len(s2))
    s2.close()
    # the sampled tokens again, from the same history, in the one-launch loop
    # (the fast sampler; split: candidates exchanged between the GPUs)
    s3 = Session(m, max_seq)
    if attach:
        s3.attach_tp()
    s3.prefill(np.concatenate([toks, out["greedy"], app]).astype(np.int32), want_logits=False)
    out["sampled_loop"] = np.asarray(s3.generate(SampleOptions(0.7, 20, 0.8), 1234, 24))
    s3.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True)
    ap.add_argument("--rank", type=int, required=True)
    ap.add_argument("--size", type=int, required=True)
    ap.add_argument("--port", type=int, required=True)
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{a.port}", rank=a.rank, world_size=a.size,
                            timeout=datetime.timedelta(seconds=120))
    g = TpGroup.from_process_group(device=a.rank)
    m = Model(a.model, a.rank, 1024, tp=g)
    out = run(m, attach=True)
    m.close()
    g.close()
    if a.rank == 0:
        np.savez(a.out, **out)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
