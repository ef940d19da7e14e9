"""ctypes wrapper of the test oracle.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, always as the checker, never as the thing that
is measured or shipped.

* ``Oracle`` -- liboracle.so, the CPU restatement of the reference token loop
  (rpg_oracle.c, see rpg_oracle.h for the reference lines each part follows).
* ``RefQuant`` -- the reference's own src/quant.cc compiled by oracle/Makefile
  (bit-exact dequant pin).
* ``RefEmu`` -- the reference engine and sampler, CUDA sources included,
  compiled by oracle/Makefile for the host CPU against the SIMT emulation
  layer in oracle/emu: the reference's own outputs with no GPU.
* ``RefText`` -- the reference's host text layer (tokenizer, chat template,
  tool parser).

The reference's GPU build is never run: its RopeKernel
(src/kernels_gpu.cu:598-621) has no bounds check and reads and writes one row
past the end of its k buffer whenever rows x KV heads x head_dim / 2 is not a
multiple of 256 (two KV heads and an odd token count) -- the illegal memory
access it once raised on a B200.  The emulation runs the same code on the
host with slack after every allocation.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_QUANT_SO = os.path.join(HERE, "_ref", "libref_quant.so")
REF_EMU_SO = os.path.join(HERE, "_ref", "libref_emu.so")
REF_ENGINE_EMU_SO = os.path.join(HERE, "_ref", "librpg_engine_emu.so")
REF_TEXT_SO = os.path.join(HERE, "_ref", "libref_text.so")

i32, i64, u32, u64, f32, vp = (ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float,
                               ctypes.c_void_p)


def _ptr(a):
    return a.ctypes.data if a is not None else None


class Oracle:
    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            raise RuntimeError(f"{ORACLE_SO} missing: run make -C oracle")
        L = ctypes.CDLL(ORACLE_SO)
        sig = {
            "orc_f16_to_f32": (f32, [ctypes.c_uint16]),
            "orc_f32_to_f16": (ctypes.c_uint16, [f32]),
            "orc_dequant_row": (ctypes.c_int, [u32, vp, i64, vp]),
            "orc_matvec": (ctypes.c_int, [u32, vp, i64, i64, vp, i64, vp, ctypes.c_int]),
            "orc_model_open": (vp, [ctypes.c_char_p, i32, ctypes.c_char_p, ctypes.c_int]),
            "orc_model_close": (None, [vp]),
            "orc_model_shape": (None, [vp, vp]),
            "orc_session_create": (vp, [vp, i32, ctypes.c_int]),
            "orc_session_free": (None, [vp]),
            "orc_session_len": (i64, [vp]),
            "orc_session_set_len": (None, [vp, i64]),
            "orc_prefill": (ctypes.c_int, [vp, vp, i64, vp, vp]),
            "orc_generate": (ctypes.c_int, [vp, f32, i32, f32, u64, i32, vp, i32, vp, vp]),
            "orc_counter_uniform": (f32, [u64, u64]),
            "orc_filter_to_probs": (None, [vp, i64, f32, i32, f32, vp]),
            "orc_sample_token": (i32, [vp, i64, f32, i32, f32, f32]),
        }
        for k, (r, a) in sig.items():
            fn = getattr(L, k)
            fn.restype, fn.argtypes = r, a
        self.L = L

    def dequant(self, qtype: int, data: np.ndarray, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        rc = self.L.orc_dequant_row(qtype, np.ascontiguousarray(data).ctypes.data, n, out.ctypes.data)
        assert rc == 0
        return out

    def matvec(self, qtype, wbytes, rows, cols, x, n_threads=0) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
        out = np.empty((x.shape[0], rows), dtype=np.float32)
        rc = self.L.orc_matvec(qtype, np.ascontiguousarray(wbytes).ctypes.data, rows, cols, x.ctypes.data,
                               x.shape[0], out.ctypes.data, n_threads or os.cpu_count())
        assert rc == 0
        return out

    def counter_uniform(self, seed, counter) -> float:
        return float(self.L.orc_counter_uniform(seed, counter))

    def filter_to_probs(self, logits, temperature, top_k, top_p) -> np.ndarray:
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        out = np.empty_like(lg)
        self.L.orc_filter_to_probs(lg.ctypes.data, lg.size, temperature, top_k, top_p, out.ctypes.data)
        return out

    def sample_token(self, logits, temperature, top_k, top_p, u) -> int:
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        return int(self.L.orc_sample_token(lg.ctypes.data, lg.size, temperature, top_k, top_p, u))


class OracleModel:
    def __init__(self, path: str, max_pos: int = 4096):
        self.o = Oracle()
        err = ctypes.create_string_buffer(256)
        self.h = self.o.L.orc_model_open(path.encode(), max_pos, err, 256)
        if not self.h:
            raise RuntimeError(f"oracle model open failed: {err.value.decode()}")
        out = (ctypes.c_int32 * 10)()
        self.o.L.orc_model_shape(self.h, out)
        self.shape = dict(zip(["n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab",
                               "context_length", "rope_positions", "eos_id"], list(out)))
        self.vocab = self.shape["vocab"]

    def close(self):
        if self.h:
            self.o.L.orc_model_close(self.h)
            self.h = None


class OracleSession:
    def __init__(self, model: OracleModel, max_seq: int = 4096, n_threads: int = 0):
        self.m = model
        self.L = model.o.L
        self.h = self.L.orc_session_create(model.h, max_seq, n_threads or os.cpu_count())
        if not self.h:
            raise RuntimeError("oracle session create failed")

    def __len__(self):
        return int(self.L.orc_session_len(self.h))

    def set_len(self, n):
        self.L.orc_session_set_len(self.h, n)

    def prefill(self, tokens, hidden: bool = False):
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        logits = np.empty(self.m.vocab, dtype=np.float32)
        hid = None
        if hidden:
            hid = np.empty((self.m.shape["n_layers"] + 1, toks.size, self.m.shape["hidden"]), dtype=np.float32)
        rc = self.L.orc_prefill(self.h, toks.ctypes.data, toks.size, logits.ctypes.data, _ptr(hid))
        if rc != 0:
            raise RuntimeError(f"oracle prefill failed ({rc})")
        return (logits, hid) if hidden else logits

    def generate(self, temperature=0.0, top_k=0, top_p=1.0, seed=0, max_tokens=32, stop=(), step_logits=False):
        out = np.empty(max_tokens, dtype=np.int32)
        st = np.ascontiguousarray(np.asarray(list(stop), dtype=np.int32))
        steps = np.empty((max_tokens, self.m.vocab), dtype=np.float32) if step_logits else None
        n = self.L.orc_generate(self.h, temperature, top_k, top_p, seed, max_tokens,
                                st.ctypes.data if st.size else None, st.size, out.ctypes.data, _ptr(steps))
        if n < 0:
            raise RuntimeError(f"oracle generate failed ({n})")
        return (out[:n].copy(), steps[:n].copy()) if step_logits else out[:n].copy()

    def close(self):
        if self.h:
            self.L.orc_session_free(self.h)
            self.h = None


class RefQuant:
    """The reference's src/quant.cc (bit-exact host dequantiser)."""

    def __init__(self):
        if not os.path.exists(REF_QUANT_SO):
            raise FileNotFoundError(REF_QUANT_SO)
        L = ctypes.CDLL(REF_QUANT_SO)
        L.ref_dequantize_row.restype = ctypes.c_int
        L.ref_dequantize_row.argtypes = [u32, vp, i64, vp]
        L.ref_f16_to_f32.restype = f32
        L.ref_f16_to_f32.argtypes = [ctypes.c_uint16]
        self.L = L

    def dequant(self, qtype, data, n) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        rc = self.L.ref_dequantize_row(qtype, np.ascontiguousarray(data).ctypes.data, n, out.ctypes.data)
        assert rc == 0
        return out


class RefEmu:
    """The reference engine and sampler compiled for the host (oracle/emu)."""

    def __init__(self):
        if not os.path.exists(REF_EMU_SO):
            raise FileNotFoundError(REF_EMU_SO)
        L = ctypes.CDLL(REF_EMU_SO)
        sig = {
            "ref_last_error": (ctypes.c_char_p, []),
            "ref_dequantize_row": (ctypes.c_int, [u32, vp, i64, vp]),
            "ref_kernel_dequant": (ctypes.c_int, [u32, vp, i64, vp]),
            "ref_counter_uniform": (f32, [u64, u64]),
            "ref_matmul": (ctypes.c_int, [u32, vp, i64, i64, vp, i64, vp]),
            "ref_sample": (ctypes.c_int, [vp, i64, f32, i32, f32, u64, u64, vp, vp]),
            "ref_session_open": (ctypes.c_int, [ctypes.c_char_p, i32, i32]),
            "ref_session_close": (None, [ctypes.c_int]),
            "ref_session_prefill": (ctypes.c_int, [ctypes.c_int, vp, i64, vp, vp]),
            "ref_session_generate": (ctypes.c_int, [ctypes.c_int, f32, i32, f32, u64, i32, vp, i32, vp, vp, vp]),
            "ref_session_len": (i64, [ctypes.c_int]),
        }
        for k, (r, a) in sig.items():
            fn = getattr(L, k)
            fn.restype, fn.argtypes = r, a
        self.L = L

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError(self.L.ref_last_error().decode(errors="replace"))

    def counter_uniform(self, seed, counter) -> float:
        return float(self.L.ref_counter_uniform(seed, counter))

    def kernel_dequant(self, qtype, data, n) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self._check(self.L.ref_kernel_dequant(qtype, np.ascontiguousarray(data).ctypes.data, n, out.ctypes.data))
        return out

    def matmul(self, qtype, wbytes, rows, cols, x) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
        out = np.empty((x.shape[0], rows), dtype=np.float32)
        self._check(self.L.ref_matmul(qtype, np.ascontiguousarray(wbytes).ctypes.data, rows, cols, x.ctypes.data,
                                      x.shape[0], out.ctypes.data))
        return out

    def sample(self, logits, temperature, top_k, top_p, seed, counter, want_probs=False):
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        probs = np.empty_like(lg) if want_probs else None
        tok = ctypes.c_int32(-1)
        self._check(self.L.ref_sample(lg.ctypes.data, lg.size, temperature, top_k, top_p, seed, counter, _ptr(probs),
                                      ctypes.byref(tok)))
        return tok.value, probs

    def session(self, gguf_path, max_pos, max_seq):
        return RefEmuSession(self, gguf_path, max_pos, max_seq)


class RefEmuSession:
    def __init__(self, ref: RefEmu, gguf_path: str, max_pos: int, max_seq: int):
        self.r = ref
        self.h = ref.L.ref_session_open(gguf_path.encode(), max_pos, max_seq)
        if self.h <= 0:
            raise RuntimeError(ref.L.ref_last_error().decode(errors="replace"))

    def __len__(self):
        return int(self.r.L.ref_session_len(self.h))

    def prefill(self, tokens, vocab, n_layers=None, hidden=None):
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        lg = np.empty(vocab, dtype=np.float32)
        hid = None
        if n_layers is not None:
            hid = np.empty((n_layers + 1, toks.size, hidden), dtype=np.float32)
        self.r._check(self.r.L.ref_session_prefill(self.h, toks.ctypes.data, toks.size, lg.ctypes.data, _ptr(hid)))
        return (lg, hid) if hid is not None else lg

    def generate(self, temperature, top_k, top_p, seed, max_tokens, vocab, stop=(), step_logits=False):
        out = np.empty(max_tokens, dtype=np.int32)
        n = ctypes.c_int32(0)
        st = np.ascontiguousarray(np.asarray(list(stop), dtype=np.int32))
        steps = np.empty((max_tokens, vocab), dtype=np.float32) if step_logits else None
        self.r._check(self.r.L.ref_session_generate(self.h, temperature, top_k, top_p, seed, max_tokens,
                                                    st.ctypes.data if st.size else None, st.size, out.ctypes.data,
                                                    ctypes.byref(n), _ptr(steps)))
        k = n.value
        return (out[:k].copy(), steps[:k].copy()) if step_logits else out[:k].copy()

    def close(self):
        if self.h > 0:
            self.r.L.ref_session_close(self.h)
            self.h = 0


class RefText:
    """The reference's host text layer (tokenizer, ChatML template, tool parser)."""

    def __init__(self, gguf_path: str):
        if not os.path.exists(REF_TEXT_SO):
            raise FileNotFoundError(REF_TEXT_SO)
        L = ctypes.CDLL(REF_TEXT_SO)
        sig = {
            "reft_last_error": (ctypes.c_char_p, []),
            "reft_free": (None, [vp]),
            "reft_open": (vp, [ctypes.c_char_p]),
            "reft_close": (None, [vp]),
            "reft_encode": (i64, [vp, ctypes.c_char_p, i64, ctypes.c_int, vp, i64]),
            "reft_decode": (vp, [vp, vp, i64, ctypes.c_int, ctypes.POINTER(i64)]),
            "reft_render": (vp, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_int]),
            "reft_parse": (vp, [ctypes.c_char_p, i64]),
        }
        for k, (r, a) in sig.items():
            fn = getattr(L, k)
            fn.restype, fn.argtypes = r, a
        self.L = L
        self.h = L.reft_open(gguf_path.encode())
        if not self.h:
            raise RuntimeError(L.reft_last_error().decode(errors="replace"))

    def _take(self, p, n=None) -> bytes:
        if not p:
            raise RuntimeError(self.L.reft_last_error().decode(errors="replace"))
        b = ctypes.string_at(p, n) if n is not None else ctypes.string_at(p)
        self.L.reft_free(p)
        return b

    def encode(self, text: bytes, parse_special=True) -> list:
        cap = 4 * len(text) + 16
        out = np.empty(cap, dtype=np.int32)
        n = self.L.reft_encode(self.h, text, len(text), int(parse_special), out.ctypes.data, cap)
        if n < 0:
            raise RuntimeError(self.L.reft_last_error().decode(errors="replace"))
        return [int(v) for v in out[:n]]

    def decode(self, ids, skip_special=False) -> bytes:
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        n = i64(0)
        p = self.L.reft_decode(self.h, a.ctypes.data if a.size else None, a.size, int(skip_special), ctypes.byref(n))
        return self._take(p, n.value)

    def render(self, messages_json: str, tools_json=None, add_generation_prompt=True, enable_thinking=True) -> bytes:
        p = self.L.reft_render(messages_json.encode(), tools_json.encode() if tools_json is not None else None,
                               int(add_generation_prompt), int(enable_thinking))
        return self._take(p)

    def parse(self, raw: bytes) -> str:
        return self._take(self.L.reft_parse(raw, len(raw))).decode()

    def close(self):
        if self.h:
            self.L.reft_close(self.h)
            self.h = None
