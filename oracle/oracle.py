"""ctypes wrapper of the test oracle.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, always as the checker, never as the thing that
is measured or shipped.

* ``Oracle`` -- liboracle.so, the CPU restatement of the reference token loop
  (rpg_oracle.c, see rpg_oracle.h for the reference lines each part follows).
* ``RefQuant`` -- the reference's own src/quant.cc compiled by oracle/Makefile
  (bit-exact dequant pin).
* ``RefShim`` -- the reference engine compiled from its own sources for
  sm_100a (GPU golden outputs; needs a GPU).
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_QUANT_SO = os.path.join(HERE, "_ref", "libref_quant.so")
REF_SHIM_SO = os.path.join(HERE, "_ref", "libref_shim.so")

# The reference's GPU engine raised an illegal memory access inside its own
# prefill on a B200 (GpuForwardFull on the tiny-g4 synthetic model, 21 valid
# token ids, after the same calls had passed in earlier runs), so no
# reference GPU code (engine, matmul, sampler, dequant kernels) is run from
# here any more; the shim's host functions (counter_uniform) stay in use.
REF_GPU_CLOSED = ("the reference's GPU engine raised an illegal memory access in its own prefill "
                  "(tiny-g4 synthetic model, valid ids); its GPU code is not run again")

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


class RefShim:
    """Host functions of the reference engine compiled from its own sources."""

    def __init__(self):
        if not os.path.exists(REF_SHIM_SO):
            raise FileNotFoundError(REF_SHIM_SO)
        L = ctypes.CDLL(REF_SHIM_SO)
        sig = {
            "ref_last_error": (ctypes.c_char_p, []),
            "ref_dequantize_row": (ctypes.c_int, [u32, vp, i64, vp]),
            "ref_counter_uniform": (f32, [u64, u64]),
        }
        for k, (r, a) in sig.items():
            fn = getattr(L, k)
            fn.restype, fn.argtypes = r, a
        self.L = L

    def counter_uniform(self, seed, counter):
        return float(self.L.ref_counter_uniform(seed, counter))

    # The shim's GPU entries (ref_gpu_dequant, ref_gpu_matmul, ref_gpu_sample,
    # ref_session_*) drive the reference's own GPU code, which is no longer run
    # (REF_GPU_CLOSED); they are not bound here.
