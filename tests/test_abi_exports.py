"""The C-ABI library loads without a GPU and exports every symbol include/*.h declares."""

import ctypes
import os
import re
import subprocess

from rpgbarenginecuda_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for hdr in ("rpg_engine.h", "rpg_b200.h"):
        text = open(os.path.join(ROOT, "include", hdr)).read()
        names |= set(re.findall(r"(?:RPG_API|RPGB_API)\s+[\w\s\*]+?\b(\w+)\s*\(", text))
    return names


def test_headers_declare_the_reference_abi():
    names = declared_symbols()
    # the ten functions of the reference's include/rpg_engine.h / src/rpg_engine.def
    ten = {"rpg_engine_version", "rpg_engine_last_error", "rpg_engine_load_model", "rpg_engine_unload_model",
           "rpg_engine_session_create", "rpg_engine_session_destroy", "rpg_engine_session_reset",
           "rpg_engine_generate", "rpg_engine_free", "rpg_engine_model_info"}
    assert ten <= names
    assert {"rpgb_prefill", "rpgb_generate", "rpgb_sample", "rpgb_matrix_matvec"} <= names


def test_library_exports_every_declared_symbol():
    lib = _lib.load_engine()
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, missing


def test_no_internal_symbols_leak():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.ENGINE_SO], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert exported <= declared_symbols(), sorted(exported - declared_symbols())


def test_version_and_errors_without_gpu():
    lib = _lib.load_engine()
    assert lib.rpg_engine_version().decode().startswith("0.1")
    assert lib.rpgb_version()
    # invalid handles fail cleanly with a message, no exception crosses the ABI
    assert lib.rpgb_session_len(12345) < 0
    assert b"invalid" in lib.rpgb_last_error()
    assert lib.rpg_engine_session_reset(777) < 0
    assert lib.rpg_engine_last_error()
    lib.rpg_engine_unload_model(999)  # no-op on an invalid handle
    lib.rpg_engine_session_destroy(999)
    assert lib.rpg_engine_model_info(999) is None
    assert lib.rpg_engine_generate(999, b"{}") is None


def test_counter_uniform_host_entry_matches_oracle(oracle):
    lib = _lib.load_engine()
    for seed in (0, 7, 2 ** 64 - 1):
        for c in range(40):
            assert lib.rpgb_counter_uniform(seed, c) == oracle.counter_uniform(seed, c)
    assert isinstance(ctypes.c_float(lib.rpgb_counter_uniform(1, 2)).value, float)
