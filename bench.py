#!/usr/bin/env python3
"""Benchmark of the token loop on the 1.7B chat-turn workload (the reference's headline configuration).

One step = one chat turn of the Qwen3-1.7B-shaped Q4_K_M synthetic model:
a 2811-token seeded prompt prefill, then three rounds of (append 40 seeded
tokens, 64-token decode) with T=0.7, top_k=20, top_p=0.8 and a fixed seed.

* value    decode tok/s, device time from CUDA events on the session stream;
           weights (1.1 GB per token, > L2) and KV resident in HBM.
* e2e      the same decode tok/s measured on the host around the C-ABI calls
           (rpgb_prefill / rpgb_generate with host buffers: the H2D of the
           token ids and the D2H of the generated ids are inside).
* roofline the decode loop kernel (one cooperative launch per generate call
           runs every decode step): algorithmic bytes per decoded token = the
           quantised weights of every matrix + lm_head + norms, plus the fp16
           K/V rows the step's attention reads (2 * layers * kv_dim * 2 bytes
           per cached position), divided by the decode device time from CUDA
           events on the session stream.
* roofline_matvec  the standalone decode matvec: every matrix of the model
           plus lm_head, one launch each, back to back in a CUDA graph, CUDA
           events on the launching stream, algorithmic bytes =
           M*K/256*{144,210} + x + y.
* cpu_baseline  the CPU restatement of the reference loop (oracle/, the
           reference's own CPU engine is not vendored), bounded sample.

Multi-GPU (torchrun): one independent session per GPU (the path shards by
session, no collective on the data path); value = all ranks' decode tokens /
max over ranks of the decode time.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT_LEN = 2811
ROUNDS = 3
APPEND = 40
DECODE = 64
SAMPLE = (0.7, 20, 0.8)
SEED = 1234
MODEL = "qwen3-1.7b"
METRIC = "batch-1 decode tok/s + prefill tok/s (Qwen3-1.7B Q4_K_M); matvec % HBM peak"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default=MODEL)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-roofline", action="store_true")
    ap.add_argument("--matvec-shapes", action="store_true",
                    help="launch the decode matvec once per distinct matrix shape of the model and exit "
                         "(the command profiled by ncu for profiles/)")
    ap.add_argument("--tcgemm-shape", action="store_true",
                    help="run the tcgen05 prefill GEMM twice on a Q4_K 6144x2048 matrix x 1024 tokens and exit "
                         "(the command profiled by ncu for profiles/)")
    ap.add_argument("--decode-trace", type=int, default=0,
                    help="print the decode loop's per-phase critical times at this context")
    ap.add_argument("--decode-loop-ctx", type=int, default=0,
                    help="prefill this many tokens, then two generate calls (2 and 4 decode steps) and exit "
                         "(the second decode-loop launch is the one profiled for profiles/)")
    ap.add_argument("--suite", action="store_true",
                    help="the other single-GPU configurations: 0.6B (21-id prompt + 32 greedy steps) and 4B "
                         "(prefill at n = 1, 4, 16, 128, 2048; 256 greedy steps from contexts 512 and 3840); "
                         "one JSON line each")
    ap.add_argument("--tp", action="store_true",
                    help="tensor-parallel measurement of the 8B configuration: run under torchrun with N ranks "
                         "(N = 1: the whole model on one GPU); 1024-token prefill + 128 greedy steps per turn")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi clock/throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = tempfile.mktemp(suffix=".csv")

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        try:
            rows = [ln.split(",") for ln in open(self.path).read().strip().splitlines()]
        except Exception:
            return None
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_baseline(path, n_prompt=64, n_decode=8, ctx=None):
    """The oracle (CPU restatement of the reference loop) on all host cores, bounded
    sample.  With ctx, the prompt is prefilled at positions ctx - n_prompt ..
    ctx - 1, so the decode steps attend over ctx positions as the benchmark's
    do (the KV rows below the prompt are zero-filled: the work per step is
    that of a full context, the values are not)."""
    from oracle.oracle import OracleModel, OracleSession
    from rpgbarenginecuda_b200 import synthetic

    cores = os.cpu_count()
    om = OracleModel(path, 4096)
    s = OracleSession(om, 4096, cores)
    prompt = synthetic.seeded_tokens(n_prompt, 0, om.vocab)
    if ctx is not None:
        s.set_len(ctx - n_prompt)
    t0 = time.perf_counter()
    s.prefill(prompt)
    t1 = time.perf_counter()
    s.generate(*SAMPLE, SEED, n_decode)
    t2 = time.perf_counter()
    s.close()
    om.close()
    where = f" at context {ctx}" if ctx is not None else ""
    return {"decode_tok_s": n_decode / (t2 - t1), "prefill_tok_s": n_prompt / (t1 - t0), "cores": cores,
            "sample": f"{n_prompt}-token prefill + {n_decode}-token decode (T=0.7,k=20,p=0.8){where} of the "
                      f"{MODEL} turn (the builder's C port of the reference loop, oracle/rpg_oracle.c)",
            "seconds": t2 - t0}


def reference_arm(args):
    world, rank, _ = dist()
    if rank != 0:
        return 0
    from rpgbarenginecuda_b200 import synthetic

    path = synthetic.cached_model(args.model, seed=0)
    vals, pre = [], []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(path, 8, 4, ctx=PROMPT_LEN + APPEND)
        if i >= args.warmup:
            vals.append(r["decode_tok_s"])
            pre.append(r["prefill_tok_s"])
    v = statistics.mean(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 * 4 / v, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "prefill_tok_s": round(statistics.mean(pre), 4),
        "config": {"workload": f"{MODEL} turn sample: 4-token decode at context {PROMPT_LEN + APPEND} per step "
                               "(after an 8-token prefill), T=0.7 top_k=20 top_p=0.8", "model": args.model},
        "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"4-token decode at context {PROMPT_LEN + APPEND} per step, by the builder's C "
                                   "port of the reference loop (oracle/rpg_oracle.c; the reference's CPU engine "
                                   "tools/cpu_ref_gen links sources that are not vendored)"},
        "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def matvec_roofline(path, device, peak):
    """Decode matvec roofline: every matrix of the model launched back to back
    (one decode's weight stream, 1.1 GB > L2), one pass captured in a CUDA
    graph so that the host's per-call cost stays out of the device timeline,
    three replays timed with CUDA events; algorithmic bytes =
    M*K/256*{144,210} + 4(M+K) per launch.  The lm_head shape (151936 x 2048
    Q6_K, 255 MB) is also timed alone, 20 launches back to back."""
    import numpy as np
    import torch
    from gguf import GGUFReader

    from rpgbarenginecuda_b200 import Matrix

    rd = GGUFReader(path)
    mats = []
    for t in rd.tensors:
        if len(t.shape) != 2 or int(t.tensor_type) not in (12, 14):
            continue
        cols, rows = int(t.shape[0]), int(t.shape[1])
        mats.append((t.name, int(t.tensor_type), rows, cols, np.asarray(t.data).view(np.uint8).reshape(-1)))
    handles = [(Matrix(q, r, c, b, device), q, r, c, name) for (name, q, r, c, b) in mats]
    del mats, rd
    kmax = max(c for _, _, _, c, _ in handles)
    rmax = max(r for _, _, r, _, _ in handles)
    x = torch.randn(kmax, device=f"cuda:{device}")
    y = torch.empty(rmax, device=f"cuda:{device}")
    stream = torch.cuda.current_stream(device)
    sp = stream.cuda_stream
    nbytes = lambda q, r, c: r * c // 256 * (144 if q == 12 else 210) + 4 * (r + c)
    for m, _, _, _, _ in handles:  # warm-up pass
        m.matvec(x.data_ptr(), 1, y.data_ptr(), sp)
    torch.cuda.synchronize(device)
    graph, cap = torch.cuda.CUDAGraph(), torch.cuda.Stream(device)
    with torch.cuda.graph(graph, stream=cap, capture_error_mode="thread_local"):
        cs = torch.cuda.current_stream(device).cuda_stream
        for m, _, _, _, _ in handles:
            m.matvec(x.data_ptr(), 1, y.data_ptr(), cs)
    graph.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    passes = 3
    e0.record(stream)
    for _ in range(passes):
        graph.replay()
    e1.record(stream)
    e1.synchronize()
    del graph
    ms = e0.elapsed_time(e1)
    total_bytes = passes * sum(nbytes(q, r, c) for _, q, r, c, _ in handles)
    launches = passes * len(handles)
    achieved = total_bytes / (ms * 1e-3) / 1e9
    big = max(handles, key=lambda h: h[2] * h[3])
    m, q, r, c, _ = big
    e0.record(stream)
    for _ in range(20):
        m.matvec(x.data_ptr(), 1, y.data_ptr(), sp)
    e1.record(stream)
    e1.synchronize()
    big_ms = e0.elapsed_time(e1) / 20
    big_gbs = nbytes(q, r, c) / (big_ms * 1e-3) / 1e9
    for h in handles:
        h[0].close()
    traffic = None
    tf = os.path.join(ROOT, "profiles", "matvec_traffic.json")
    if os.path.exists(tf):  # dram bytes per launch of each shape, from the committed ncu capture
        with open(tf) as f:
            per = json.load(f).get("dram_bytes_per_launch", {})
        keys = [f"{'q4k' if q == 12 else 'q6k'}_{r}x{c}" for _, q, r, c, _ in handles]
        if keys and all(k in per for k in keys):
            traffic = round(sum(per[k] for k in keys) / len(keys))
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": traffic,
            "kernel": "MatvecKernel (decode Q4_K/Q6_K dequant-matvec, n=1): all matrices of the model, back to back in a CUDA graph",
            "bytes_per_launch": round(total_bytes / launches), "avg_launch_us": round(1000 * ms / launches, 2),
            "lm_head": {"shape": f"{'q4k' if q == 12 else 'q6k'}_{r}x{c}", "bytes": nbytes(q, r, c),
                        "avg_launch_us": round(1000 * big_ms, 2), "gbs": round(big_gbs, 1),
                        "frac": round(big_gbs / peak, 4)}}


SWEEP_SHAPES = [(2048, 2048), (6144, 2048), (2048, 6144), (151936, 2048), (9728, 2560)]
SWEEP_N = [1, 2, 4, 8, 64]


def matvec_sweep(device, peak, l2_bytes=126 << 20):
    """The Q4_K / Q6_K operator sweep: every (type, M x K) of SWEEP_SHAPES at
    n = 1, 2, 4, 8, 64 activation columns.  Each shape is uploaded in enough
    copies that one pass over them exceeds L2 twice (weights stream from HBM
    as in decode), one pass of launches over the copies is captured in a CUDA
    graph and replayed, CUDA events time the replays; achieved = algorithmic bytes (quantised weights + 4n(M+K)) per
    launch / average launch time."""
    import numpy as np
    import torch

    from rpgbarenginecuda_b200 import Matrix, synthetic

    out = {}
    stream = torch.cuda.current_stream(device)
    sp = stream.cuda_stream
    for qtype, qname, blk in ((12, "q4k", 144), (14, "q6k", 210)):
        for rows, cols in SWEEP_SHAPES:
            wbytes = rows * cols // 256 * blk
            copies = max(1, min(128, -(-2 * l2_bytes // wbytes)))
            b = synthetic.quantize(synthetic.normal(7 + rows + cols, rows * cols, 0.0, 0.02),
                                   {"q4k": "q4_k", "q6k": "q6_k"}[qname])
            mats = [Matrix(qtype, rows, cols, b, device) for _ in range(copies)]
            del b
            x = torch.randn(max(SWEEP_N), cols, device=f"cuda:{device}")
            y = torch.empty(max(SWEEP_N), rows, device=f"cuda:{device}")
            for n in SWEEP_N:
                for m in mats:  # warm-up pass (sizes the tensor-core scratch)
                    m.matvec(x.data_ptr(), n, y.data_ptr(), sp)
                torch.cuda.synchronize(device)
                # one pass over the copies as a CUDA graph: the launches run
                # back to back without the host's per-call cost in between
                graph, cap = torch.cuda.CUDAGraph(), torch.cuda.Stream(device)
                with torch.cuda.graph(graph, stream=cap, capture_error_mode="thread_local"):
                    cs = torch.cuda.current_stream(device).cuda_stream
                    for m in mats:
                        m.matvec(x.data_ptr(), n, y.data_ptr(), cs)
                graph.replay()
                reps = max(3, 192 // copies)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(reps):
                    graph.replay()
                e1.record(stream)
                e1.synchronize()
                del graph
                us = 1000.0 * e0.elapsed_time(e1) / (reps * copies)
                alg = wbytes + 4 * n * (rows + cols)
                gbs = alg / (us * 1e-6) / 1e9
                out[f"{qname}_{rows}x{cols}_n{n}"] = {"us": round(us, 2), "gbs": round(gbs, 1),
                                                      "frac": round(gbs / peak, 4)}
            for m in mats:
                m.close()
            del x, y
            torch.cuda.empty_cache()
    n1 = [v["frac"] for k, v in out.items() if k.endswith("_n1")]
    return {"kernel": "rpgb_matrix_matvec: Q4_K/Q6_K operator sweep (weights > L2, launches back to back in a CUDA graph)",
            "bound": "hbm", "peak": peak, "unit": "GB/s", "frac_n1_mean": round(sum(n1) / len(n1), 4),
            "shapes": out}


def matvec_shapes(args):
    """One decode-matvec launch per distinct (type, rows, cols) of the model, after one warm-up launch each."""
    import numpy as np
    import torch
    from gguf import GGUFReader

    from rpgbarenginecuda_b200 import Matrix, synthetic

    path = synthetic.cached_model(args.model, seed=0)
    rd = GGUFReader(path)
    seen = {}
    for t in rd.tensors:
        if len(t.shape) != 2 or int(t.tensor_type) not in (12, 14):
            continue
        key = (int(t.tensor_type), int(t.shape[1]), int(t.shape[0]))
        if key not in seen:
            seen[key] = np.asarray(t.data).view(np.uint8).reshape(-1).copy()
    x = torch.randn(max(k[2] for k in seen), device="cuda")
    y = torch.empty(max(k[1] for k in seen), device="cuda")
    sp = torch.cuda.current_stream().cuda_stream
    for (q, r, c), b in sorted(seen.items()):
        m = Matrix(q, r, c, b, 0)
        m.matvec(x.data_ptr(), 1, y.data_ptr(), sp)  # warm-up
        m.matvec(x.data_ptr(), 1, y.data_ptr(), sp)
        torch.cuda.synchronize()
        print(f"{'q4k' if q == 12 else 'q6k'}_{r}x{c}", flush=True)
        m.close()


def tcgemm_shape(args):
    """Two launches of the tensor-core prefill GEMM (operator entry, 1024 tokens)."""
    import torch

    from rpgbarenginecuda_b200 import GGML_Q4_K, Matrix, synthetic

    rows, cols, n = 6144, 2048, 1024
    b = synthetic.quantize(synthetic.normal(1, rows * cols, 0.0, 0.02), "q4_k")
    m = Matrix(GGML_Q4_K, rows, cols, b)
    x = torch.from_numpy(synthetic.normal(2, n * cols, 0.0, 1.0).reshape(n, cols)).cuda()
    out = torch.empty((n, rows), dtype=torch.float32, device="cuda")
    for _ in range(2):
        m.matvec(x.data_ptr(), n, out.data_ptr())
    torch.cuda.synchronize()
    print("tcgemm q4k_6144x2048 n=1024 max|out| %.4f" % float(out.abs().max()), flush=True)
    m.close()


def decode_loop_ctx(args):
    """Prefill args.decode_loop_ctx tokens, then generate 2 and 4 tokens (two decode-loop launches)."""
    from rpgbarenginecuda_b200 import Model, SampleOptions, Session, synthetic

    m = Model(synthetic.cached_model(args.model, seed=0), 0, 4096)
    s = Session(m, 4096)
    s.prefill(synthetic.seeded_tokens(args.decode_loop_ctx, 0, m.vocab), want_logits=False)
    opts = SampleOptions(*SAMPLE)
    s.generate(opts, 1, 2)
    ids = s.generate(opts, 1, 4)
    print("decode loop at context %d: %s" % (args.decode_loop_ctx, list(map(int, ids))), flush=True)
    s.close()
    m.close()


def decode_trace(args):
    """Per-phase critical times of the decode loop kernel at one context.

    Prefills args.decode_trace seeded tokens, runs a 16-token sampled generate
    (one loop launch, untimed warm-up) and then a traced one, and prints, per
    phase kind, the mean over layers and steps of the phase's critical time:
    the latest block's end of the phase minus the latest block's end of the
    phase before it (the step's first phase: minus the previous step's
    sampler).  Times come from the kernel's own device timeline (SM cycle
    counter anchored to %globaltimer)."""
    import numpy as np

    from rpgbarenginecuda_b200 import Model, SampleOptions, Session, synthetic

    m = Model(synthetic.cached_model(args.model, seed=0), 0, 4096)
    s = Session(m, 4096)
    ctx, n_steps = args.decode_trace, 16
    toks = synthetic.seeded_tokens(ctx, 0, m.vocab)
    s.prefill(toks, want_logits=False)
    opts = SampleOptions(*SAMPLE)
    s.generate(opts, SEED, n_steps)
    s.set_len(ctx - 1)
    s.prefill(toks[-1:], want_logits=False)  # the next position's logits again
    s.trace_enable(1 << 20)
    s.generate(opts, SEED, n_steps)
    rec = s.trace_take(1 << 20)
    s.trace_enable(0)
    L = m.shape["n_layers"]
    per = 5 * L + 2
    main = rec[(rec["launch"] != 0xFFFFFFFF) & ((rec["block"] >> 24) == 0)]
    ends = {}
    for r in main:
        k = int(r["launch"])
        ends[k] = max(ends.get(k, 0), int(r["t_end"]))
    names = ["qkv", "attention", "o", "gate/up", "down"]
    acc = {n: [] for n in names + ["lm_head", "sampler", "step"]}
    keys = sorted(ends)
    for i in range(1, len(keys)):
        k, kp = keys[i], keys[i - 1]
        if k != kp + 1:
            continue
        ph = k % per
        dt = (ends[k] - ends[kp]) / 1000.0
        acc[names[ph % 5] if ph < 5 * L else ("lm_head" if ph == 5 * L else "sampler")].append(dt)
    steps = sorted({k // per for k in keys})
    for st in steps[1:]:
        a, b = (st - 1) * per + per - 1, st * per + per - 1
        if a in ends and b in ends:
            acc["step"].append((ends[b] - ends[a]) / 1000.0)
    print(f"decode loop trace: {args.model}, context {ctx}, {n_steps} sampled steps (T=0.7, top_k=20, top_p=0.8)")
    print("| phase | mean us | min us | max us | per token us |")
    print("|---|---|---|---|---|")
    for n in names + ["lm_head", "sampler", "step"]:
        v = np.array(acc[n]) if acc[n] else np.zeros(1)
        mult = L if n in names else 1
        print(f"| {n} | {v.mean():.2f} | {v.min():.2f} | {v.max():.2f} | {v.mean() * mult:.1f} |")
    # inside a block: mean times from the end of the block's previous phase
    # to its marks (matvec phases: 1 digits of warp 0 stored, 2 every unit
    # done, 4 epilogue stores issued; attention: 1 first chunk's data there,
    # 2 first chunk computed, 3 its slot refilled, 4 warp 0's chunks done)
    # and to the end of the phase
    kinds = {}
    for r in rec[rec["launch"] != 0xFFFFFFFF]:
        ph = int(r["launch"]) % per
        n = names[ph % 5] if ph < 5 * L else ("lm_head" if ph == 5 * L else "sampler")
        k = int(r["block"]) >> 24
        if int(r["t_end"]) and int(r["t_start"]):
            kinds.setdefault(n, {}).setdefault(k, []).append((int(r["t_end"]) - int(r["t_start"])) / 1000.0)
    print("| phase | to mark 1 | mark 2 | mark 3 | mark 4 | end (us, per block) |")
    print("|---|---|---|---|---|---|")
    for n in names + ["lm_head", "sampler"]:
        d = kinds.get(n, {})
        cells = [f"{np.mean(d[k]):.2f}" if d.get(k) else "-" for k in (1, 2, 3, 4, 0)]
        print(f"| {n} | " + " | ".join(cells) + " |")
    s.close()
    m.close()


def ours(args):
    import numpy as np
    import torch

    from rpgbarenginecuda_b200 import Model, SampleOptions, Session, launch_count, synthetic

    world, rank, local = dist()
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as tdist

        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device(f"cuda:{local}"))
        pg = tdist

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    path = synthetic.cached_model(args.model, seed=0)
    model = Model(path, device=local, max_pos=4096)
    sess = Session(model, 4096)
    V = model.vocab
    stream = torch.cuda.ExternalStream(sess.stream_ptr, device=local)
    prompt = synthetic.seeded_tokens(PROMPT_LEN, 1000 + rank, V)
    appends = [synthetic.seeded_tokens(APPEND, 2000 + 10 * rank + r, V) for r in range(ROUNDS)]
    opts = SampleOptions(*SAMPLE)

    shape = synthetic.PRESETS[args.model]
    w_tok, kv_pos = shape.weight_bytes_per_token(), shape.kv_bytes_per_position()

    def turn_bytes():
        """Algorithmic HBM bytes of one turn's decode steps (weights + K/V rows read)."""
        tot, length = 0, PROMPT_LEN
        for _ in range(ROUNDS):
            length += APPEND
            for i in range(DECODE):  # the step forwarding the token at position length + i reads length + i + 1 rows
                tot += w_tok + kv_pos * (length + i + 1)
            length += DECODE
        return tot

    def turn(timing):
        sess.set_len(0)
        ev = []
        h0 = time.perf_counter()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        sess.prefill(prompt, want_logits=False)
        e1.record(stream)
        ev.append(("prefill", e0, e1, PROMPT_LEN))
        host_prefill = time.perf_counter() - h0
        host_decode, n_dec = 0.0, 0
        for r in range(ROUNDS):
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            sess.prefill(appends[r], want_logits=False)
            a1.record(stream)
            ev.append(("append", a0, a1, APPEND))
            d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            h1 = time.perf_counter()
            d0.record(stream)
            ids = sess.generate(opts, SEED, DECODE)
            d1.record(stream)
            host_decode += time.perf_counter() - h1
            n_dec += len(ids)
            ev.append(("decode", d0, d1, len(ids)))
        torch.cuda.synchronize()
        for kind, a, b, n in ev:
            timing[kind][0] += a.elapsed_time(b)
            timing[kind][1] += n
        timing["host_decode"][0] += host_decode * 1e3
        timing["host_decode"][1] += n_dec
        timing["host_prefill"][0] += host_prefill * 1e3
        timing["host_prefill"][1] += PROMPT_LEN

    for _ in range(args.warmup):
        turn({k: [0.0, 0] for k in ("prefill", "append", "decode", "host_decode", "host_prefill")})
    barrier()
    timing = {k: [0.0, 0] for k in ("prefill", "append", "decode", "host_decode", "host_prefill")}
    l0 = launch_count()
    with Clocks(local) as clk:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        w0 = time.perf_counter()
        for _ in range(args.steps):
            turn(timing)
        t1.record()
        barrier()
        wall = time.perf_counter() - w0
    launches = launch_count() - l0
    total_ms = t0.elapsed_time(t1)
    dec_ms, dec_tok = timing["decode"]
    # max over ranks of the decode time, sum of tokens
    agg = np.array([dec_ms, dec_tok, timing["prefill"][0], timing["host_decode"][0], total_ms], dtype=np.float64)
    if pg is not None:
        t = torch.tensor(agg, device=f"cuda:{local}")
        mx = t.clone()
        pg.all_reduce(mx, op=pg.ReduceOp.MAX)
        sm = t.clone()
        pg.all_reduce(sm, op=pg.ReduceOp.SUM)
        dec_ms_max, pre_ms_max, host_dec_max, total_max = float(mx[0]), float(mx[2]), float(mx[3]), float(mx[4])
        dec_tok_all = float(sm[1])
    else:
        dec_ms_max, pre_ms_max, host_dec_max, total_max = dec_ms, timing["prefill"][0], timing["host_decode"][0], total_ms
        dec_tok_all = dec_tok
    value = dec_tok_all / (dec_ms_max * 1e-3)
    prefill_tok_s = world * PROMPT_LEN * args.steps / (pre_ms_max * 1e-3)
    e2e = dec_tok_all / (host_dec_max * 1e-3)
    clocks = clk.summary()
    stats = sess.stats()

    # the decode loop kernel's roofline: algorithmic bytes / decode device time
    hbm_peak, hbm_kind = peaks()
    loop_bytes = turn_bytes() * args.steps
    achieved = loop_bytes / (dec_ms * 1e-3) / 1e9
    loop_roof = {"kernel": "DecodeLoopKernel", "bound": "hbm", "achieved": round(achieved, 1),
                 "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                 "traffic": None, "peak_kind": hbm_kind,
                 "bytes_per_token": {"weights": w_tok,
                                     "kv_mean": round(loop_bytes / args.steps / (ROUNDS * DECODE) - w_tok)}}
    tf = os.path.join(ROOT, "profiles", "decode_loop_traffic.json")
    if os.path.exists(tf):  # dram bytes per decoded token from the committed ncu capture
        with open(tf) as f:
            loop_roof["traffic"] = json.load(f).get("dram_bytes_per_token")

    roof = sweep = None
    if rank == 0 and not args.no_roofline:
        sess.close()
        model.close()
        torch.cuda.empty_cache()
        hbm, kind = peaks()
        roof = matvec_roofline(path, local, hbm)
        sweep = matvec_sweep(local, hbm)
        roof["peak_kind"] = kind
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        c = cpu_baseline(path, 16, 8, ctx=PROMPT_LEN + APPEND)
        cpu = {"value": round(c["decode_tok_s"], 4), "unit": "tok/s", "cores": c["cores"], "kind": "port",
               "sample": c["sample"], "prefill_tok_s": round(c["prefill_tok_s"], 3)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_max / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights quantised to Q4_K/Q6_K, seeded token ids)",
            "prefill_tok_s": round(prefill_tok_s, 1),
            # the 40-token appends at context ~2900 (prefill calls of their own)
            "append_ms": round(timing["append"][0] / max(1, args.steps * ROUNDS), 3),
            "config": {"workload": f"{args.model} turn: {PROMPT_LEN}-token prefill + {ROUNDS} x ({APPEND} appended "
                                   f"+ {DECODE} decoded) tokens, T=0.7 top_k=20 top_p=0.8",
                       "model": args.model, "global_batch": world, "seq_len": PROMPT_LEN + ROUNDS * (APPEND + DECODE),
                       "parallelism": f"sessions x{world}",
                       "l2": "inputs larger than L2 (1.1 GB of weights streamed per token)"},
            "e2e": {"value": round(e2e, 2), "unit": "tok/s",
                    # copies of the timed generate calls: the start position in,
                    # the step count, error word and generated ids out
                    "h2d_bytes_per_step": 8 * ROUNDS,
                    "d2h_bytes_per_step": ROUNDS * (8 + 4 * DECODE)},
            "gpu_launches": int(launches),
            "kernels_per_decode_step": stats["kernels_per_step"],
            "wall_s": round(wall, 3),
        }
        if clocks is not None:
            line["clocks"] = clocks
        line["roofline"] = loop_roof
        if roof is not None:
            line["roofline_matvec"] = roof
            line["roofline_matvec_sweep"] = sweep
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()
    return 0


TP_MODEL, TP_PROMPT, TP_DECODE = "qwen3-8b", 1024, 128


def suite_bench(args):
    """The 0.6B and 4B workloads on one GPU, timed with CUDA events on the
    session stream (args.warmup untimed repetitions, then args.steps timed)."""
    import torch

    from rpgbarenginecuda_b200 import Model, SampleOptions, Session, synthetic

    torch.cuda.set_device(0)
    greedy = SampleOptions(0.0, 0, 1.0)

    def timed(sess, fn):
        stream = torch.cuda.ExternalStream(sess.stream_ptr, device=0)
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        tot, n = 0.0, 0
        for _ in range(args.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            k = fn()
            e1.record(stream)
            torch.cuda.synchronize()
            tot += e0.elapsed_time(e1)
            n += k
        return n / (tot * 1e-3)

    def line(name, metric, value, extra):
        d = {"metric": metric, "value": round(value, 2), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
             "warmup": args.warmup, "higher_is_better": True, "dtype": "f32", "data": "synthetic",
             "config": {"model": name, "global_batch": 1}}
        d.update(extra)
        print(json.dumps(d), flush=True)

    # 0.6B: 21-id prompt, 32 greedy steps
    m = Model(synthetic.cached_model("qwen3-0.6b", seed=0), 0, 4096)
    s = Session(m, 4096)
    prompt = synthetic.seeded_tokens(21, 0, m.vocab)

    def pre06():
        s.set_len(0)
        s.prefill(prompt, want_logits=False)
        return len(prompt)

    def dec06():
        s.set_len(0)
        s.prefill(prompt, want_logits=False)
        return len(s.generate(greedy, 0, 32))

    p06 = timed(s, pre06)
    # decode rate = 32 tokens over (prefill + decode) minus the prefill time
    t_all = 1.0 / timed(s, dec06) * 32
    t_pre = len(prompt) / p06
    line("qwen3-0.6b", "batch-1 greedy decode tok/s (qwen3-0.6b, 21-id prompt, 32 steps)", 32 / (t_all - t_pre),
         {"prefill_tok_s": round(p06, 1)})
    s.close()
    m.close()

    # 4B: prefill at several prompt lengths; 256 greedy steps from contexts 512 and 3840
    m = Model(synthetic.cached_model("qwen3-4b", seed=0), 0, 4096)
    s = Session(m, 4096)
    pre = {}
    for n in (1, 4, 16, 128, 2048):
        toks = synthetic.seeded_tokens(n, 7, m.vocab)

        def pf(toks=toks):
            s.set_len(0)
            s.prefill(toks, want_logits=False)
            return len(toks)

        pre[str(n)] = round(timed(s, pf), 1)
    dec = {}
    for ctx in (512, 3840):
        toks = synthetic.seeded_tokens(ctx, 9, m.vocab)
        stream = torch.cuda.ExternalStream(s.stream_ptr, device=0)
        rates = []
        for it in range(args.warmup + args.steps):
            s.set_len(0)
            s.prefill(toks, want_logits=False)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            k = len(s.generate(greedy, 0, 256))
            e1.record(stream)
            torch.cuda.synchronize()
            if it >= args.warmup:
                rates.append(k / (e0.elapsed_time(e1) * 1e-3))
        dec[str(ctx)] = round(sum(rates) / len(rates), 2)
    line("qwen3-4b", "batch-1 greedy decode tok/s (qwen3-4b, 256 steps from context 512)", dec["512"],
         {"decode_tok_s_by_context": dec, "prefill_tok_s_by_n": pre})
    s.close()
    m.close()
    return 0


def tp_bench(args):
    """The 8B configuration split over the torchrun ranks (one GPU each).

    One turn = a TP_PROMPT-token prefill and TP_DECODE greedy steps on every
    rank in lockstep (the ranks exchange partial sums after attn_output and
    ffn_down and gather the logits).  Decode and prefill are timed with CUDA
    events on each rank's session stream; the reported times are the max over
    ranks.  With one rank the whole model runs on one GPU (decode loop kernel).
    """
    import datetime

    import torch

    from rpgbarenginecuda_b200 import Model, SampleOptions, Session, TpGroup, synthetic

    world, rank, local = dist()
    torch.cuda.set_device(local)
    tdist = None
    if world > 1:
        import torch.distributed as tdist

        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device(f"cuda:{local}"))
    name = TP_MODEL if args.model == MODEL else args.model
    if rank == 0:
        synthetic.cached_model(name, seed=0)  # one rank writes the file
    if tdist is not None:
        tdist.barrier()
    path = synthetic.cached_model(name, seed=0)
    group = TpGroup.from_process_group(device=local) if world > 1 else None
    model = Model(path, device=local, max_pos=4096, tp=group)
    sess = Session(model, 4096)
    if group is not None:
        sess.attach_tp()  # greedy decode in the one-launch loop, partials exchanged over NVLink
    stream = torch.cuda.ExternalStream(sess.stream_ptr, device=local)
    prompt = synthetic.seeded_tokens(TP_PROMPT, 1000, model.vocab)
    greedy = SampleOptions(0.0, 0, 1.0)

    def turn():
        sess.set_len(0)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(stream)
        sess.prefill(prompt, want_logits=False)
        ev[1].record(stream)
        ids = sess.generate(greedy, 0, TP_DECODE)
        ev[2].record(stream)
        torch.cuda.synchronize()
        return ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), len(ids)

    for _ in range(args.warmup):
        turn()
    pre_ms = dec_ms = 0.0
    n_dec = 0
    with Clocks(local) as clk:
        for _ in range(args.steps):
            a, b, n = turn()
            pre_ms, dec_ms, n_dec = pre_ms + a, dec_ms + b, n_dec + n
    if tdist is not None:
        t = torch.tensor([pre_ms, dec_ms], device=f"cuda:{local}", dtype=torch.float64)
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        pre_ms, dec_ms = float(t[0]), float(t[1])
    shape = synthetic.PRESETS[name]
    w_tok, kv_pos = shape.weight_bytes_per_token(), shape.kv_bytes_per_position()
    # algorithmic bytes of one turn's decode steps, summed over ranks (weights split, K/V rows split by head)
    dec_bytes = sum(w_tok + kv_pos * (TP_PROMPT + i + 1) for i in range(TP_DECODE)) * args.steps
    hbm_peak, hbm_kind = peaks()
    per_rank_gbs = dec_bytes / world / (dec_ms * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": f"batch-1 greedy decode tok/s ({name} Q4_K_M, tensor parallel over {world} GPU(s))",
            "value": round(n_dec / (dec_ms * 1e-3), 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round((pre_ms + dec_ms) / args.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights quantised to Q4_K/Q6_K, seeded token ids)",
            "prefill_tok_s": round(TP_PROMPT * args.steps / (pre_ms * 1e-3), 1),
            "config": {"workload": f"{name}: {TP_PROMPT}-token prefill + {TP_DECODE} greedy steps per turn",
                       "model": name, "global_batch": 1, "seq_len": TP_PROMPT + TP_DECODE,
                       "parallelism": (f"tp{world}: decode loop kernel per GPU, partials over NVLink"
                                       if world > 1 else "one GPU (decode loop kernel)")},
            "roofline": {"bound": "hbm", "achieved": round(per_rank_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(per_rank_gbs / hbm_peak, 4), "traffic": None, "peak_kind": hbm_kind,
                         "note": "per rank: algorithmic decode bytes / ranks / decode time"},
            "clocks": clk.summary()}), flush=True)
    sess.close()
    model.close()
    if group is not None:
        group.close()
    if tdist is not None:
        tdist.barrier()
        tdist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.matvec_shapes:
        matvec_shapes(args)
        return
    if args.tcgemm_shape:
        tcgemm_shape(args)
        return
    if args.decode_loop_ctx > 0:
        decode_loop_ctx(args)
        return
    if args.decode_trace > 0:
        decode_trace(args)
        return
    if args.suite:
        return suite_bench(args)
    if args.tp:
        return tp_bench(args)
    if args.impl == "reference":
        return reference_arm(args)
    return ours(args)


if __name__ == "__main__":
    sys.exit(main())
