"""B200-native (sm_100a) token loop of RPGBarEngineCUDA.

Python view of the C ABI in include/rpg_b200.h.  Names follow the reference's
internal API that its own tools drive (tools/gen_check.cu, sample_check.cu,
matmul_bench.cu): a Model is GpuModel::Load, a Session is the KV cache plus
scratch (GpuKvCache + GpuScratch), ``prefill`` is GpuForwardFull with a cache,
``generate`` is GpuGenerate, ``Matrix.matvec`` is GpuMatMulQuant and
``sample`` is GpuSampleToken / GpuFilterToProbs.  The ten-function public ABI
(include/rpg_engine.h) is exported by the same library.
"""

from __future__ import annotations

import ctypes

import numpy as np

from ._lib import EngineError, SampleOptions, check, load_engine  # noqa: F401

__all__ = ["Model", "Session", "Matrix", "SampleOptions", "EngineError", "TpGroup", "shard_plan", "sample",
           "counter_uniform", "launch_count", "library_path", "GGML_Q4_K", "GGML_Q5_K", "GGML_Q6_K", "GGML_Q8_0"]

GGML_Q8_0 = 8
GGML_Q4_K = 12
GGML_Q5_K = 13
GGML_Q6_K = 14


def library_path() -> str:
    from ._lib import ENGINE_SO
    return ENGINE_SO


def shard_plan(shape: dict, rank: int, size: int) -> dict:
    """This rank's share of a model split over `size` GPUs (rpgb_tp_shard_plan).

    `shape` holds n_heads, n_kv_heads, head_dim, ffn and vocab; raises
    EngineError when the model does not split evenly."""
    lib = load_engine()
    src = (ctypes.c_int32 * 5)(shape["n_heads"], shape["n_kv_heads"], shape["head_dim"], shape["ffn"],
                               shape["vocab"])
    out = (ctypes.c_int32 * 5)()
    check(lib.rpgb_tp_shard_plan(src, rank, size, out), "tp_shard_plan")
    return dict(zip(["heads", "kv_heads", "ffn", "vocab0", "vocab_rows"], list(out)))


class TpGroup:
    """A tensor-parallel group: one rank per GPU, joined over NCCL.

    Every rank constructs it with the same `unique_id` (made once by rank 0
    with ``TpGroup.unique_id()`` and sent to the others, e.g. with
    ``torch.distributed.broadcast_object_list``); construction is collective.
    ``from_process_group`` does that exchange over an initialised
    torch.distributed group."""

    def __init__(self, unique_id: bytes, rank: int, size: int, device: int):
        self._lib = load_engine()
        if len(unique_id) != 128:
            raise ValueError("a group id is 128 bytes")
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id)
        self.rank, self.size, self.device = rank, size, device
        self.handle = check(self._lib.rpgb_tp_group_create(buf, rank, size, device), "tp_group_create")

    @staticmethod
    def unique_id() -> bytes:
        lib = load_engine()
        buf = (ctypes.c_uint8 * 128)()
        check(lib.rpgb_tp_unique_id(buf), "tp_unique_id")
        return bytes(buf)

    @staticmethod
    def exchange_id(rank: int, group=None) -> bytes:
        """Rank 0's fresh id, delivered to every rank of a torch.distributed group."""
        import torch.distributed as dist
        obj = [TpGroup.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return obj[0]

    @classmethod
    def from_process_group(cls, device: int, group=None) -> "TpGroup":
        import torch.distributed as dist
        rank, size = dist.get_rank(group), dist.get_world_size(group)
        return cls(cls.exchange_id(rank, group), rank, size, device)

    def close(self):
        if self.handle is not None and self.handle >= 0:
            self._lib.rpgb_tp_group_free(self.handle)
            self.handle = None


class Model:
    """Weights of one GGUF resident on one device (this rank's shard with `tp`)."""

    def __init__(self, path: str, device: int = 0, max_pos: int = 4096, tp: TpGroup | None = None):
        self._lib = load_engine()
        self.path = path
        self.tp = tp
        if tp is None:
            self.handle = check(self._lib.rpgb_model_load(path.encode(), device, max_pos), "model_load")
        else:
            self.handle = check(self._lib.rpgb_model_load_tp(path.encode(), device, max_pos, tp.handle),
                                "model_load_tp")
        out = (ctypes.c_int32 * 12)()
        check(self._lib.rpgb_model_shape(self.handle, out, 12), "model_shape")
        keys = ["n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab", "context_length",
                "rope_positions", "eos_id", "device", "num_sms"]
        self.shape = dict(zip(keys, list(out)))
        self.vocab = self.shape["vocab"]

    @property
    def device_bytes(self) -> int:
        return int(self._lib.rpgb_model_device_bytes(self.handle))

    def close(self):
        if self.handle is not None and self.handle >= 0:
            self._lib.rpgb_model_free(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class Session:
    """fp16 KV cache + decode state of one conversation."""

    def __init__(self, model: Model, max_seq: int = 4096):
        self._lib = load_engine()
        self.model = model
        self.max_seq = max_seq
        self.handle = check(self._lib.rpgb_session_create(model.handle, max_seq), "session_create")

    def attach_tp(self, group=None):
        """Joins the ranks' sessions for greedy decode in the one-launch loop
        (rpgb_session_tp_attach).  Collective over the model's tensor-parallel
        group: the 64-byte exchange-buffer handles go round over
        torch.distributed (`group`), except for a group of one."""
        tp = self.model.tp
        if tp is None:
            raise ValueError("the session's model is not tensor parallel")
        own = (ctypes.c_uint8 * 64)()
        check(self._lib.rpgb_session_tp_handle(self.handle, own), "session_tp_handle")
        if tp.size == 1:
            handles = [bytes(own)]
        else:
            import torch.distributed as dist
            handles = [None] * tp.size
            dist.all_gather_object(handles, bytes(own), group=group)
        buf = (ctypes.c_uint8 * (64 * tp.size)).from_buffer_copy(b"".join(handles))
        check(self._lib.rpgb_session_tp_attach(self.handle, buf), "session_tp_attach")

    def __len__(self) -> int:
        return int(self._lib.rpgb_session_len(self.handle))

    def set_len(self, n: int):
        check(self._lib.rpgb_session_set_len(self.handle, n), "session_set_len")

    def prefill(self, tokens, want_logits: bool = True):
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        out = np.empty(self.model.vocab, dtype=np.float32) if want_logits else None
        check(self._lib.rpgb_prefill(self.handle, toks.ctypes.data, toks.size,
                                     out.ctypes.data if out is not None else None), "prefill")
        return out

    def generate(self, opts: SampleOptions | None = None, seed: int = 0, max_tokens: int = 32, stop=(),
                 step_logits: bool = False):
        opts = opts or SampleOptions(0.0, 0, 1.0)
        stop_arr = np.ascontiguousarray(np.asarray(list(stop), dtype=np.int32))
        ids = np.empty(max_tokens, dtype=np.int32)
        n_out = ctypes.c_int32(0)
        steps = np.empty((max_tokens, self.model.vocab), dtype=np.float32) if step_logits else None
        check(self._lib.rpgb_generate(self.handle, ctypes.byref(opts), seed, max_tokens,
                                      stop_arr.ctypes.data if stop_arr.size else None, stop_arr.size,
                                      ids.ctypes.data, ctypes.byref(n_out),
                                      steps.ctypes.data if steps is not None else None), "generate")
        n = n_out.value
        return (ids[:n].copy(), steps[:n].copy()) if step_logits else ids[:n].copy()

    def stats(self):
        k, g, n = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int64()
        check(self._lib.rpgb_session_stats(self.handle, ctypes.byref(k), ctypes.byref(g), ctypes.byref(n)),
              "session_stats")
        return {"kernels_per_step": k.value, "graph_ready": bool(g.value), "graph_launches": n.value}

    def trace_enable(self, cap: int = 1 << 16):
        """Record a device timeline of every decode-step launch (0 turns it off)."""
        check(self._lib.rpgb_session_trace_enable(self.handle, cap), "session_trace_enable")

    TRACE_DTYPE = np.dtype([("launch", np.uint32), ("block", np.uint32), ("t_start", np.uint64),
                            ("t_ready", np.uint64), ("t_end", np.uint64)])

    def trace_take(self, cap: int = 1 << 16) -> np.ndarray:
        """Records gathered since the last take (structured array, ns times)."""
        out = np.zeros(cap, dtype=self.TRACE_DTYPE)
        n = check(self._lib.rpgb_session_trace_take(self.handle, out.ctypes.data, cap), "session_trace_take")
        return out[:n].copy()

    @property
    def stream_ptr(self) -> int:
        """The session's cudaStream_t (for CUDA-event timing of its work)."""
        return int(self._lib.rpgb_session_stream(self.handle) or 0)

    def close(self):
        if self.handle is not None and self.handle >= 0:
            self._lib.rpgb_session_free(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class Matrix:
    """One quantised matrix in the engine's device layout (operator entry)."""

    def __init__(self, qtype: int, rows: int, cols: int, gguf_bytes: np.ndarray, device: int = 0):
        self._lib = load_engine()
        b = np.ascontiguousarray(gguf_bytes, dtype=np.uint8)
        self.rows, self.cols, self.qtype = rows, cols, qtype
        self.handle = check(self._lib.rpgb_matrix_upload(device, qtype, rows, cols, b.ctypes.data), "matrix_upload")

    def dequant(self, row0: int, n_rows: int, dst_ptr: int, stream: int = 0):
        check(self._lib.rpgb_matrix_dequant(self.handle, row0, n_rows, dst_ptr, stream or None), "matrix_dequant")

    def matvec(self, x_ptr: int, n_tok: int, out_ptr: int, stream: int = 0):
        check(self._lib.rpgb_matrix_matvec(self.handle, x_ptr, n_tok, out_ptr, stream or None), "matrix_matvec")

    def close(self):
        if self.handle is not None and self.handle >= 0:
            self._lib.rpgb_matrix_free(self.handle)
            self.handle = None


def sample(logits_ptr: int, n: int, opts: SampleOptions, seed: int, counter: int, tok_ptr: int,
           probs_ptr: int | None = None, stream: int = 0):
    lib = load_engine()
    check(lib.rpgb_sample(logits_ptr, n, ctypes.byref(opts), seed, counter, probs_ptr, tok_ptr, stream or None),
          "sample")


def launch_count() -> int:
    """Kernels launched by the engine library so far (graph nodes counted per replay)."""
    return int(load_engine().rpgb_launch_count())


def counter_uniform(seed: int, counter: int) -> float:
    return float(load_engine().rpgb_counter_uniform(seed, counter))


class TextLayer:
    """The host text layer of rpg_engine_generate (tokenizer, ChatML prompt,
    output parse) over a GGUF's tokenizer; runs on the CPU."""

    def __init__(self, gguf_path: str):
        self.L = load_engine()
        self.h = self.L.rpgb_text_open(gguf_path.encode())
        if not self.h:
            raise EngineError(f"text layer: {self._err()}")

    def _err(self) -> str:
        m = self.L.rpg_engine_last_error()
        return m.decode(errors="replace") if m else ""

    def _take(self, p, n=None) -> bytes:
        if not p:
            raise EngineError(f"text layer: {self._err()}")
        b = ctypes.string_at(p, n) if n is not None else ctypes.string_at(p)
        self.L.rpg_engine_free(p)
        return b

    def encode(self, text: bytes, parse_special: bool = True) -> list:
        cap = 4 * len(text) + 16
        out = np.empty(cap, dtype=np.int32)
        n = self.L.rpgb_text_encode(self.h, text, len(text), int(parse_special), out.ctypes.data, cap)
        if n < 0:
            raise EngineError(f"text layer: {self._err()}")
        return [int(v) for v in out[:n]]

    def decode(self, ids) -> bytes:
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        n = ctypes.c_int64(0)
        return self._take(self.L.rpgb_text_decode(self.h, a.ctypes.data if a.size else None, a.size,
                                                  ctypes.byref(n)), n.value)

    def render(self, request_json: str) -> bytes:
        return self._take(self.L.rpgb_text_render(request_json.encode()))

    def parse(self, raw: bytes) -> str:
        return self._take(self.L.rpgb_text_parse(raw, len(raw))).decode()

    def close(self):
        if self.h:
            self.L.rpgb_text_close(self.h)
            self.h = None
