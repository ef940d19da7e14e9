"""Tensor-parallel host logic, on the CPU.

* The shard plan (rpgb_tp_shard_plan): the split planned for the 8B
  configuration at TP = 1, 2, 4, 8 and the models that do not split.
* The split itself on quantised bytes, with the oracle as the checker: row
  slices of q / k / v / gate / up / lm_head are whole GGUF rows, and column
  slices of attn_output / ffn_down are whole 256-column super-blocks of every
  row, so the concatenated row outputs and the summed column partials equal
  the unsplit matvec.
* The group id exchange over torch.distributed (gloo, world size 2).
"""

import os

import numpy as np
import pytest

from rpgbarenginecuda_b200 import EngineError, GGML_Q4_K, GGML_Q6_K, TpGroup, shard_plan, synthetic

SHAPE_8B = dict(n_heads=32, n_kv_heads=8, head_dim=128, ffn=12288, vocab=151936)


@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_shard_plan_8b(size):
    rows = 0
    for rank in range(size):
        p = shard_plan(SHAPE_8B, rank, size)
        assert p["heads"] == 32 // size and p["kv_heads"] == 8 // size
        assert p["ffn"] == 12288 // size and p["ffn"] % 256 == 0
        assert p["heads"] * 128 % 256 == 0
        assert p["vocab0"] == rows and p["vocab_rows"] % 16 == 0
        rows += p["vocab_rows"]
    assert rows == 151936


@pytest.mark.parametrize("shape,size,what", [
    (dict(n_heads=16, n_kv_heads=8, head_dim=128, ffn=6144, vocab=151936), 16, "KV heads"),
    (dict(n_heads=4, n_kv_heads=4, head_dim=128, ffn=1024, vocab=4096), 4, "super-blocks of attn_output"),
    (dict(n_heads=16, n_kv_heads=8, head_dim=128, ffn=3072, vocab=8192), 8, "ffn"),
    (dict(n_heads=8, n_kv_heads=2, head_dim=128, ffn=1024, vocab=4104), 2, "vocabulary"),
    (SHAPE_8B, 2, "rank"),
])
def test_shard_plan_rejects(shape, size, what):
    rank = size if what == "rank" else 0
    with pytest.raises(EngineError, match=what):
        shard_plan(shape, rank, size)


# Which configurations split over 2 / 4 / 8 GPUs: FFN columns per rank must
# be whole 256-column super-blocks (0.6B ffn 3072 / 8 = 384 and 4B ffn
# 9728 / 4 = 2432 are not).
SUPPORT = {"qwen3-0.6b": (2, 4), "qwen3-1.7b": (2, 4, 8), "qwen3-4b": (2,), "qwen3-8b": (2, 4, 8)}


@pytest.mark.parametrize("name", sorted(SUPPORT))
@pytest.mark.parametrize("size", [2, 4, 8])
def test_shard_plan_support_matrix(name, size):
    sh = synthetic.PRESETS[name]
    shape = dict(n_heads=sh.n_heads, n_kv_heads=sh.n_kv_heads, head_dim=sh.head_dim, ffn=sh.ffn, vocab=sh.vocab)
    if size in SUPPORT[name]:
        plans = [shard_plan(shape, r, size) for r in range(size)]
        assert sum(p["ffn"] for p in plans) == sh.ffn and sum(p["heads"] for p in plans) == sh.n_heads
    else:
        with pytest.raises(EngineError):
            shard_plan(shape, 0, size)


def _q(rows, cols, qt, seed):
    w = synthetic.normal(seed, rows * cols, 0.0, 0.02)
    return synthetic.quantize(w, qt).reshape(rows, -1)


@pytest.mark.parametrize("qt,qtype,blk", [("q4_k", GGML_Q4_K, 144), ("q6_k", GGML_Q6_K, 210)])
def test_split_matvec_equals_whole(oracle, qt, qtype, blk):
    rows, cols, size = 64, 1024, 2
    b = _q(rows, cols, qt, 5)
    x = synthetic.normal(6, cols, 0.0, 1.0).reshape(1, cols)
    whole = oracle.matvec(qtype, b.reshape(-1), rows, cols, x)[0]
    # rows: rank r holds rows [r R/size, (r+1) R/size)
    parts = [oracle.matvec(qtype, b[r * rows // size:(r + 1) * rows // size].reshape(-1), rows // size, cols, x)[0]
             for r in range(size)]
    assert np.array_equal(np.concatenate(parts), whole)
    # columns: rank r holds super-blocks [r nb/size, (r+1) nb/size) of every row
    nb = cols // 256
    k = nb // size
    acc = np.zeros(rows)
    for r in range(size):
        sl = np.ascontiguousarray(b[:, r * k * blk:(r + 1) * k * blk]).reshape(-1)
        acc += oracle.matvec(qtype, sl, rows, cols // size, x[:, r * k * 256:(r + 1) * k * 256])[0]
    assert np.abs(acc - whole).max() <= 1e-5 * np.abs(whole).max()


def _exchange_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        uid = TpGroup.exchange_id(rank)
        q.put((rank, uid))
    finally:
        dist.destroy_process_group()


def test_group_id_exchange_gloo():
    """Rank 0's id reaches every rank unchanged (the step before ncclCommInitRank)."""
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert len(got[0]) == 128 and got[0] == got[1]
