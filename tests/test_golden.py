"""The oracle against golden values made by the reference's own code.

tests/golden/reference_pins.npz holds outputs of the reference built from its
sources (tests/golden/make_golden.py): its host dequantiser (src/quant.cc) on
encoder and arbitrary-byte Q4_K / Q6_K blocks, and its counter-based uniform
draw.  These checks need no reference build, so the oracle stays pinned
wherever the tests run.
"""

import os

import numpy as np
import pytest

from oracle.oracle import Oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_pins.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("code", [12, 14])
def test_dequant_matches_reference_golden(golden, code):
    b = golden[f"bytes_{code}"]
    ref = golden[f"dequant_{code}"]
    ours = Oracle().dequant(code, b, ref.size)
    assert np.array_equal(ours.view(np.uint32), ref.view(np.uint32))


def test_counter_uniform_matches_reference_golden(golden):
    o = Oracle()
    seeds, counters, u = golden["rng_seeds"], golden["rng_counters"], golden["rng_u"]
    for i, s in enumerate(seeds):
        for j, c in enumerate(counters):
            assert np.float32(o.counter_uniform(int(s), int(c))) == u[i, j], (int(s), int(c))
