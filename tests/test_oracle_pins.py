"""Pins the CPU oracle to the reference's own code (no GPU needed).

Reference checks restated here (the reference's own tests):
* dequant bit-exact vs src/quant.cc::DequantizeRow (tools/dequant_check.cu:75-125);
* exhaustive f16 -> f32 sweep vs src/dtypes.h::F16ToF32 (tools/dequant_check.cu:186-210);
* counter RNG u table bit-exact vs DevCounterUniform (tools/sample_check.cu:228,
  tests/cmp_sample.py criterion 1).
The reference libraries are built from its sources into oracle/_ref by
oracle/Makefile; the tests skip when that build is absent.
"""

import os

import numpy as np
import pytest

from oracle.oracle import REF_EMU_SO, REF_QUANT_SO, Oracle, RefQuant
from rpgbarenginecuda_b200 import synthetic

needs_ref_quant = pytest.mark.skipif(not os.path.exists(REF_QUANT_SO), reason="oracle/_ref not built")
needs_ref_emu = pytest.mark.skipif(not os.path.exists(REF_EMU_SO), reason="oracle/_ref not built")


@needs_ref_quant
@pytest.mark.parametrize("qtype,code", [("q4_k", 12), ("q6_k", 14)])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_dequant_bitexact_vs_reference_quant_cc(qtype, code, seed):
    o, rq = Oracle(), RefQuant()
    x = synthetic.normal(seed, 256 * 96, 0.0, 0.02 * (1 + seed))
    b = synthetic.quantize(x, qtype)
    a = rq.dequant(code, b, x.size)
    c = o.dequant(code, b, x.size)
    assert np.array_equal(a.view(np.uint32), c.view(np.uint32))


# (type code, bytes per block, elements per block, byte offsets of fp16 scales)
BLOCKS = {12: (144, 256, (0, 2)), 13: (176, 256, (0, 2)), 14: (210, 256, (208,)), 8: (34, 32, (0,))}


@needs_ref_quant
@pytest.mark.parametrize("code", [12, 13, 14, 8])
def test_dequant_bitexact_random_bytes(code):
    """Arbitrary bytes (all scale / sign / subnormal-d patterns), not only
    encoder output.  Q5_K and Q8_0 are on the reference's host path only
    (src/quant.cc:29-45; its GPU loader rejects them, src/gpu_model.cu:26-38)."""
    o, rq = Oracle(), RefQuant()
    blk, per, halves = BLOCKS[code]
    n_blocks = 64 * 256 // per
    rng = np.random.default_rng(code)
    b = rng.integers(0, 256, size=blk * n_blocks, dtype=np.uint8)
    # keep the fp16 scales finite so the comparison is on numbers, not NaN payloads
    for i in range(n_blocks):
        for h in halves:
            b[i * blk + h + 1] &= 0x7B
    a = rq.dequant(code, b, per * n_blocks)
    c = o.dequant(code, b, per * n_blocks)
    assert np.array_equal(a.view(np.uint32), c.view(np.uint32))


@needs_ref_quant
def test_f16_sweep_exhaustive():
    o, rq = Oracle(), RefQuant()
    bad = 0
    for h in range(65536):
        a = np.float32(rq.L.ref_f16_to_f32(h)).view(np.uint32)
        c = np.float32(o.L.orc_f16_to_f32(h)).view(np.uint32)
        bad += int(a != c)
    assert bad == 0


def test_f32_to_f16_is_round_to_nearest_even(oracle):
    # numpy's float16 cast is IEEE RNE, the rounding of __float2half_rn
    rng = np.random.default_rng(5)
    vals = np.concatenate([rng.normal(0, 1, 4000), rng.normal(0, 1e-5, 2000), rng.normal(0, 3e4, 2000),
                           np.array([65504, 65519.99, 65520, -65520, 2 ** -25, 2 ** -24, 3 * 2 ** -26, 0.0, -0.0])])
    vals = vals.astype(np.float32)
    ours = np.array([oracle.L.orc_f32_to_f16(float(v)) for v in vals], dtype=np.uint16)
    assert np.array_equal(ours, vals.astype(np.float16).view(np.uint16))


@needs_ref_emu
def test_counter_uniform_bitexact_vs_reference():
    from oracle.oracle import RefEmu

    o, rs = Oracle(), RefEmu()
    for seed in (0, 11, 12, 22, 2 ** 63 + 5, 2 ** 64 - 1):
        for c in list(range(64)) + [4095, 151935, 2 ** 40 + 3]:
            assert o.counter_uniform(seed, c) == rs.counter_uniform(seed, c)


def test_quantiser_round_trip_error():
    """Our encoder (no reference quantiser exists) round-trips within 4/6-bit error."""
    o = Oracle()
    x = synthetic.normal(3, 256 * 512, 0.0, 0.02)
    rel = {}
    for qt, code in (("q4_k", 12), ("q6_k", 14)):
        y = o.dequant(code, synthetic.quantize(x, qt), x.size)
        rel[qt] = float(np.sqrt(np.mean((y - x) ** 2)) / np.sqrt(np.mean(x ** 2)))
    assert rel["q4_k"] < 0.10
    assert rel["q6_k"] < 0.03


@needs_ref_quant
@pytest.mark.parametrize("qtype,code,bound", [("q4_k", 12, 0.07), ("q5_k", 13, 0.035), ("q6_k", 14, 0.02),
                                               ("q8_0", 8, 0.005)])
def test_synthetic_encoders_decode_with_reference_quant(qtype, code, bound):
    """The synthetic writer's encoders (csrc/synth/synth_gguf.cc) produce blocks
    the reference's own dequantiser reads back close to the input (error under
    `bound` of the largest |x|), and the oracle reads them identically."""
    o, rq = Oracle(), RefQuant()
    x = synthetic.normal(11, 256 * 64, 0.0, 0.02)
    b = synthetic.quantize(x, qtype)
    a = rq.dequant(code, b, x.size)
    assert np.array_equal(a.view(np.uint32), o.dequant(code, b, x.size).view(np.uint32))
    assert np.abs(a - x).max() <= bound * np.abs(x).max()
