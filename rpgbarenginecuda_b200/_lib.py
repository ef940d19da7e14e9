"""ctypes loading of the in-tree shared libraries.

The engine library must exist (built by ``__graft_entry__.build()`` or
``make -C rpgbarenginecuda_b200/csrc``); there is deliberately no fallback.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
ENGINE_SO = os.path.join(_HERE, "librpg_engine_b200.so")
SYNTH_SO = os.path.join(_HERE, "librpg_synth.so")

_engine = None
_synth = None

c_i32, c_i64, c_u32, c_u64, c_f32, c_p = (ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint64,
                                          ctypes.c_float, ctypes.c_void_p)


class SampleOptions(ctypes.Structure):
    """rpgb_sample_options (include/rpg_b200.h); defaults of src/sampler.h:35-44."""

    _fields_ = [("temperature", c_f32), ("top_k", c_i32), ("top_p", c_f32)]

    def __init__(self, temperature=1.0, top_k=0, top_p=1.0):
        super().__init__(temperature, top_k, top_p)


# name -> (restype, argtypes)
_SIGS = {
    "rpgb_version": (ctypes.c_char_p, []),
    "rpgb_last_error": (ctypes.c_char_p, []),
    "rpgb_model_load": (c_i32, [ctypes.c_char_p, c_i32, c_i32]),
    "rpgb_model_free": (None, [c_i32]),
    "rpgb_tp_shard_plan": (c_i32, [c_p, c_i32, c_i32, c_p]),
    "rpgb_tp_unique_id": (c_i32, [c_p]),
    "rpgb_tp_group_create": (c_i32, [c_p, c_i32, c_i32, c_i32]),
    "rpgb_tp_group_free": (None, [c_i32]),
    "rpgb_model_load_tp": (c_i32, [ctypes.c_char_p, c_i32, c_i32, c_i32]),
    "rpgb_session_tp_handle": (c_i32, [c_i32, c_p]),
    "rpgb_session_tp_attach": (c_i32, [c_i32, c_p]),
    "rpgb_model_shape": (c_i32, [c_i32, c_p, c_i32]),
    "rpgb_model_device_bytes": (c_i64, [c_i32]),
    "rpgb_session_create": (c_i32, [c_i32, c_i64]),
    "rpgb_session_free": (None, [c_i32]),
    "rpgb_session_len": (c_i64, [c_i32]),
    "rpgb_session_set_len": (c_i32, [c_i32, c_i64]),
    "rpgb_prefill": (c_i32, [c_i32, c_p, c_i64, c_p]),
    "rpgb_generate": (c_i32, [c_i32, ctypes.POINTER(SampleOptions), c_u64, c_i32, c_p, c_i32, c_p, c_p, c_p]),
    "rpgb_session_stats": (c_i32, [c_i32, c_p, c_p, c_p]),
    "rpgb_session_stream": (c_p, [c_i32]),
    "rpgb_session_trace_enable": (c_i32, [c_i32, c_i32]),
    "rpgb_session_trace_take": (c_i32, [c_i32, c_p, c_i32]),
    "rpgb_launch_count": (c_i64, []),
    "rpgb_matrix_upload": (c_i32, [c_i32, c_u32, c_i64, c_i64, c_p]),
    "rpgb_matrix_free": (None, [c_i32]),
    "rpgb_matrix_dequant": (c_i32, [c_i32, c_i64, c_i64, c_p, c_p]),
    "rpgb_matrix_matvec": (c_i32, [c_i32, c_p, c_i64, c_p, c_p]),
    "rpgb_sample": (c_i32, [c_p, c_i32, ctypes.POINTER(SampleOptions), c_u64, c_u64, c_p, c_p, c_p]),
    "rpgb_sample_noalloc": (c_i32, [c_p, c_i32, ctypes.POINTER(SampleOptions), c_u64, c_u64, c_p, c_p]),
    "rpgb_counter_uniform": (c_f32, [c_u64, c_u64]),
    "rpgb_text_open": (c_p, [ctypes.c_char_p]),
    "rpgb_text_close": (None, [c_p]),
    "rpgb_text_encode": (c_i64, [c_p, ctypes.c_char_p, c_i64, c_i32, c_p, c_i64]),
    "rpgb_text_decode": (c_p, [c_p, c_p, c_i64, ctypes.POINTER(c_i64)]),
    "rpgb_text_render": (c_p, [ctypes.c_char_p]),
    "rpgb_text_parse": (c_p, [ctypes.c_char_p, c_i64]),
    # the public ten-function ABI (include/rpg_engine.h)
    "rpg_engine_version": (ctypes.c_char_p, []),
    "rpg_engine_last_error": (ctypes.c_char_p, []),
    "rpg_engine_load_model": (c_i32, [ctypes.c_char_p, ctypes.c_char_p]),
    "rpg_engine_unload_model": (None, [c_i32]),
    "rpg_engine_session_create": (c_i32, [c_i32, ctypes.c_char_p]),
    "rpg_engine_session_destroy": (None, [c_i32]),
    "rpg_engine_session_reset": (c_i32, [c_i32]),
    "rpg_engine_generate": (c_p, [c_i32, ctypes.c_char_p]),
    "rpg_engine_free": (None, [c_p]),
    "rpg_engine_model_info": (c_p, [c_i32]),
}

# Symbols every build must export (the drop-in boundary of include/*.h).
EXPORTED = sorted(_SIGS)


def load_engine():
    global _engine
    if _engine is None:
        if not os.path.exists(ENGINE_SO):
            raise RuntimeError(f"{ENGINE_SO} is missing: build it with __graft_entry__.build() "
                               "(the engine has no CPU fallback)")
        lib = ctypes.CDLL(ENGINE_SO)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _engine = lib
    return _engine


def load_synth():
    global _synth
    if _synth is None:
        if not os.path.exists(SYNTH_SO):
            raise RuntimeError(f"{SYNTH_SO} is missing: build it with __graft_entry__.build()")
        _synth = ctypes.CDLL(SYNTH_SO)
    return _synth


def last_error() -> str:
    msg = load_engine().rpgb_last_error()
    return msg.decode(errors="replace") if msg else ""


class EngineError(RuntimeError):
    pass


def check(rc: int, what: str) -> int:
    if rc < 0:
        raise EngineError(f"{what}: {last_error()}")
    return rc
