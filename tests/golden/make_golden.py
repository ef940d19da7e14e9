"""Writes tests/golden/reference_pins.npz: outputs of the reference's own code,
built from its sources by oracle/Makefile into oracle/_ref, on fixed inputs.

* Dequantisation by the reference's host dequantiser (src/quant.cc
  DequantizeRow, the bit-exact oracle of its dequant_check tool): encoder
  output of seeded N(0, 0.02) rows and arbitrary bytes with finite d / dmin,
  for Q4_K and Q6_K.
* The sampler's counter-based uniform draw (DevCounterUniform, the host copy
  of the device RNG that its sample_check tool compares bit for bit).

tests/test_golden.py checks the oracle against these values without needing
oracle/_ref.  Rerun after changing the inputs below:
    python tests/golden/make_golden.py
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import RefEmu, RefQuant  # noqa: E402
from rpgbarenginecuda_b200 import synthetic  # noqa: E402

SEEDS = [0, 11, 12, 22, 2 ** 63 + 5, 2 ** 64 - 1]
COUNTERS = list(range(64)) + [4095, 151935, 2 ** 40 + 3]


def blocks(code, blk, n_blocks, seed):
    """Encoder blocks followed by arbitrary-byte blocks with finite d / dmin."""
    qt = "q4_k" if code == 12 else "q6_k"
    enc = synthetic.quantize(synthetic.normal(seed, 256 * n_blocks, 0.0, 0.02), qt)
    rnd = np.random.default_rng(seed + code).integers(0, 256, size=blk * n_blocks, dtype=np.uint8)
    for i in range(n_blocks):
        if code == 12:
            rnd[i * blk + 1] &= 0x7B
            rnd[i * blk + 3] &= 0x7B
        else:
            rnd[i * blk + 209] &= 0x7B
    return np.concatenate([enc, rnd])


def main():
    rq, rs = RefQuant(), RefEmu()
    out = {}
    for code, blk in ((12, 144), (14, 210)):
        b = blocks(code, blk, 32, 5)
        n = 256 * (b.size // blk)
        out[f"bytes_{code}"] = b
        out[f"dequant_{code}"] = rq.dequant(code, b, n)
    out["rng_seeds"] = np.array(SEEDS, dtype=np.uint64)
    out["rng_counters"] = np.array(COUNTERS, dtype=np.uint64)
    out["rng_u"] = np.array([[rs.counter_uniform(s, c) for c in COUNTERS] for s in SEEDS], dtype=np.float32)
    np.savez_compressed(os.path.join(HERE, "reference_pins.npz"), **out)


if __name__ == "__main__":
    main()
