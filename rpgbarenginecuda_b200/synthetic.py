"""Seeded synthetic Qwen3 GGUF models (the benchmark inputs).

The reference is measured on real Qwen3 Q4_K_M checkpoints (README.md,
CHANGELOG.md); none is available offline, so the benchmark configurations are
random-init models of the same shapes, quantised in the Q4_K_M mix by the
encoder in ``csrc/synth/synth_gguf.cc``:

* Q4_K for q, k, o, gate and up in every layer and for v / down in odd layers;
* Q6_K for attn_v and ffn_down in even layers and for the tied token_embd;
* F32 norms drawn 1 + N(0, 0.05); matrices N(0, 0.02).

Both this engine and the reference read the same bytes, so parity does not
depend on the encoder beyond its round trip through the reference's
``DequantizeRow`` (src/quant.cc:416).
"""

from __future__ import annotations

import ctypes
import hashlib
import os
from dataclasses import dataclass, replace

import numpy as np

from . import _lib


@dataclass(frozen=True)
class ModelShape:
    name: str
    n_layers: int
    hidden: int
    ffn: int
    n_heads: int
    n_kv_heads: int
    head_dim: int = 128
    vocab: int = 151936
    context: int = 4096
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    weight_std: float = 0.02
    norm_std: float = 0.05
    mix: str = "q4_k_m"  # "q4_k_m" (Q4_K + Q6_K), "q5_k_m" (Q5_K + Q6_K) or "q8_0"

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def weight_bytes_per_token(self) -> int:
        """Quantised bytes one decode step streams: every layer matrix, the tied
        lm_head and the f32 norms."""
        b4, b6 = {"q4_k_m": (144, 210), "q5_k_m": (176, 210), "q8_0": (272, 272)}[self.mix]
        q4 = lambda m, k: m * k // 256 * b4  # noqa: E731
        q6 = lambda m, k: m * k // 256 * b6  # noqa: E731
        total = 0
        for layer in range(self.n_layers):
            six = layer % 2 == 0
            total += q4(self.q_dim, self.hidden) + q4(self.kv_dim, self.hidden)
            total += (q6 if six else q4)(self.kv_dim, self.hidden)
            total += q4(self.hidden, self.q_dim)
            total += 2 * q4(self.ffn, self.hidden)
            total += (q6 if six else q4)(self.hidden, self.ffn)
            total += (2 * self.hidden + 2 * self.head_dim) * 4
        total += q6(self.vocab, self.hidden) + self.hidden * 4
        return total

    def kv_bytes_per_position(self) -> int:
        return 2 * self.n_layers * self.kv_dim * 2


PRESETS = {
    "qwen3-0.6b": ModelShape("qwen3-0.6b", 28, 1024, 3072, 16, 8),
    "qwen3-1.7b": ModelShape("qwen3-1.7b", 28, 2048, 6144, 16, 8),
    "qwen3-4b": ModelShape("qwen3-4b", 36, 2560, 9728, 32, 8),
    "qwen3-8b": ModelShape("qwen3-8b", 36, 4096, 12288, 32, 8),
    # Small shapes for tests: same code paths (GQA, Q4_K/Q6_K mix, head_dim 128).
    "tiny": ModelShape("tiny", 2, 512, 1024, 4, 2, vocab=4096, context=512),
    "small": ModelShape("small", 4, 1024, 3072, 16, 8, vocab=8192, context=1024),
    "tiny-g4": ModelShape("tiny-g4", 2, 512, 1536, 8, 2, vocab=4096, context=512),
    # the 8B model's widths with two layers: its tensor-parallel splits (up to
    # eight ranks) at a test's cost
    "wide": ModelShape("wide", 2, 4096, 12288, 32, 8, vocab=8192, context=1024),
}


class _Cfg(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("ffn", ctypes.c_int32),
        ("n_heads", ctypes.c_int32),
        ("n_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("vocab", ctypes.c_int32),
        ("context", ctypes.c_int32),
        ("rope_theta", ctypes.c_float),
        ("rms_eps", ctypes.c_float),
        ("seed", ctypes.c_uint64),
        ("q6k_parity", ctypes.c_int32),
        ("weight_std", ctypes.c_float),
        ("norm_std", ctypes.c_float),
        ("mix", ctypes.c_int32),
    ]


def _synth():
    lib = _lib.load_synth()
    lib.rpgs_write_qwen3_gguf.argtypes = [ctypes.c_char_p, ctypes.POINTER(_Cfg), ctypes.c_char_p, ctypes.c_int]
    lib.rpgs_write_qwen3_gguf.restype = ctypes.c_int
    lib.rpgs_quantize_q4k.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    lib.rpgs_quantize_q4k.restype = ctypes.c_int
    lib.rpgs_quantize_q6k.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    lib.rpgs_quantize_q5k.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    lib.rpgs_quantize_q5k.restype = ctypes.c_int
    lib.rpgs_quantize_q8_0.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    lib.rpgs_quantize_q8_0.restype = ctypes.c_int
    lib.rpgs_quantize_q6k.restype = ctypes.c_int
    lib.rpgs_normal.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64, ctypes.c_float,
                                ctypes.c_float, ctypes.c_void_p]
    lib.rpgs_normal.restype = None
    return lib


def shape(name_or_shape) -> ModelShape:
    if isinstance(name_or_shape, ModelShape):
        return name_or_shape
    return PRESETS[name_or_shape]


def write_model(path: str, model="qwen3-1.7b", seed: int = 0, **overrides) -> str:
    """Writes a synthetic GGUF for ``model`` (preset name or ModelShape)."""
    s = replace(shape(model), **overrides) if overrides else shape(model)
    cfg = _Cfg(s.n_layers, s.hidden, s.ffn, s.n_heads, s.n_kv_heads, s.head_dim, s.vocab, s.context,
               s.rope_theta, s.rms_eps, seed, 0, s.weight_std, s.norm_std, MIXES[s.mix])
    err = ctypes.create_string_buffer(256)
    rc = _synth().rpgs_write_qwen3_gguf(path.encode(), ctypes.byref(cfg), err, 256)
    if rc != 0:
        raise RuntimeError(f"synthetic GGUF writer failed: {err.value.decode()}")
    return path


def cached_model(model="qwen3-1.7b", seed: int = 0, cache_dir: str | None = None) -> str:
    """Path of the synthetic model, generated once per (shape, seed) into a cache dir."""
    s = shape(model)
    cache_dir = cache_dir or os.environ.get("RPGB_MODEL_CACHE", "/tmp/rpgb_models")
    os.makedirs(cache_dir, exist_ok=True)
    mix = "" if s.mix == "q4_k_m" else f"-{s.mix}"
    path = os.path.join(cache_dir,
                        f"{s.name}-L{s.n_layers}-H{s.hidden}-w{s.weight_std:g}-n{s.norm_std:g}{mix}-s{seed}.gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write_model(tmp, s, seed)
        os.replace(tmp, path)
    return path


MIXES = {"q4_k_m": 0, "q5_k_m": 1, "q8_0": 2}
# bytes per 256 elements, ggml type code
QTYPES = {"q4_k": (144, 12), "q5_k": (176, 13), "q6_k": (210, 14), "q8_0": (272, 8)}


def quantize(x: np.ndarray, qtype: str) -> np.ndarray:
    """Quantises a float32 row (length a multiple of 256) to Q4_K, Q5_K, Q6_K or Q8_0 bytes."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    nb = x.size // 256
    out = np.zeros(nb * QTYPES[qtype][0], dtype=np.uint8)
    lib = _synth()
    fn = {"q4_k": lib.rpgs_quantize_q4k, "q5_k": lib.rpgs_quantize_q5k, "q6_k": lib.rpgs_quantize_q6k,
          "q8_0": lib.rpgs_quantize_q8_0}[qtype]
    if fn(x.ctypes.data, x.size, out.ctypes.data) != 0:
        raise ValueError("length must be a positive multiple of 256")
    return out


def normal(seed: int, n: int, mean: float = 0.0, std: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    _synth().rpgs_normal(seed, offset, n, mean, std, out.ctypes.data)
    return out


def seeded_tokens(n: int, seed: int, vocab: int = 151936) -> np.ndarray:
    """Token ids drawn uniformly from [0, vocab) (the seeded benchmark prompts)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)


def file_digest(path: str, nbytes: int = 1 << 22) -> str:
    """Cheap identity of a generated model: sha256 of its head, tail and size."""
    h = hashlib.sha256()
    size = os.path.getsize(path)
    h.update(str(size).encode())
    with open(path, "rb") as f:
        h.update(f.read(nbytes))
        f.seek(max(0, size - nbytes))
        h.update(f.read(nbytes))
    return h.hexdigest()[:16]
