"""rpgb_sample_noalloc: the sampler entry point that allocates no device memory.

It serves hosts that cannot call cudaMalloc while they sample (a frame or UI
thread that must not block on the device-wide synchronisation of an
allocation, or a process whose GPU memory already belongs to another
allocator's pool).  Its scratch is a fixed array inside the library, shared by
all calls on a device, so this file checks two calls in a row against the
allocating entry point rpgb_sample: the second call must not be affected by
what the first one left in the shared array.  Token ids must be identical (the
sampler's token choice is exact).

The file name makes pytest collect it last.
"""

import ctypes

import numpy as np
import pytest

from rpgbarenginecuda_b200 import SampleOptions
from rpgbarenginecuda_b200._lib import load_engine

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

MAX_VOCAB = 262144  # RPGB_SAMPLE_NOALLOC_MAX_VOCAB in include/rpg_b200.h

# (temperature, top_k, top_p): greedy, the fast top-k path, the general path
CASES = [(0.0, 0, 1.0), (0.7, 20, 0.8), (1.0, 2, 1.0), (1.0, 0, 0.95), (0.7, 40, 1.0)]


def _lib():
    lib = load_engine()
    assert hasattr(lib, "rpgb_sample_noalloc")
    return lib


def _err(lib):
    return lib.rpgb_last_error().decode()


def _sample_alloc(lib, logits, opts, seed, counter):
    tok = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    rc = lib.rpgb_sample(logits.data_ptr(), logits.numel(), ctypes.byref(opts), seed, counter, None,
                         tok.data_ptr(), None)
    assert rc == 0, _err(lib)
    return int(tok.item())


def _sample_noalloc(lib, logits, opts, seed, counter):
    tok = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    rc = lib.rpgb_sample_noalloc(logits.data_ptr(), logits.numel(), ctypes.byref(opts), seed, counter,
                                 tok.data_ptr(), None)
    assert rc == 0, _err(lib)
    return int(tok.item())


@pytest.mark.parametrize("n", [4096, 151936])
@pytest.mark.parametrize("t,k,p", CASES)
def test_two_calls_match_allocating_sampler(n, t, k, p):
    lib = _lib()
    rng = np.random.default_rng(1000 + n + int(10 * t) + k)
    logits = torch.from_numpy((rng.standard_normal(n) * 3.0).astype(np.float32)).cuda()
    opts = SampleOptions(t, k, p)
    seed = 77
    for counter in (5, 6):  # two calls in a row on the shared scratch
        want = _sample_alloc(lib, logits, opts, seed, counter)
        got = _sample_noalloc(lib, logits, opts, seed, counter)
        assert got == want, (n, t, k, p, counter, got, want)
        assert 0 <= got < n


def test_overflowing_fast_path_then_fast_path():
    """A call whose candidate slices overflow (ties) followed by a clean one."""
    lib = _lib()
    n = 151936
    tied = torch.zeros(n, dtype=torch.float32, device="cuda")  # every slice overflows the top-k buffer
    rng = np.random.default_rng(5)
    clean = torch.from_numpy((rng.standard_normal(n) * 3.0).astype(np.float32)).cuda()
    opts = SampleOptions(0.7, 20, 0.8)
    for logits in (tied, clean, tied, clean):
        assert _sample_noalloc(lib, logits, opts, 3, 9) == _sample_alloc(lib, logits, opts, 3, 9)


def test_rejects_vocabulary_beyond_limit():
    lib = _lib()
    logits = torch.zeros(8, dtype=torch.float32, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    opts = SampleOptions(0.0, 0, 1.0)
    rc = lib.rpgb_sample_noalloc(logits.data_ptr(), MAX_VOCAB + 1, ctypes.byref(opts), 0, 0, tok.data_ptr(), None)
    assert rc == -1
    assert "exceeds the fixed scratch limit" in _err(lib)


FRESH = r"""
import ctypes, sys
import numpy as np
import torch
sys.path.insert(0, {root!r})
from rpgbarenginecuda_b200 import SampleOptions
from rpgbarenginecuda_b200._lib import load_engine
lib = load_engine()
n = 151936
logits = torch.from_numpy((np.random.default_rng(3).standard_normal(n) * 3.0).astype(np.float32)).cuda()
toks = torch.full((8,), -1, dtype=torch.int32, device="cuda")
cases = [SampleOptions(0.7, 20, 0.8), SampleOptions(1.0, 0, 0.95), SampleOptions(0.0, 0, 1.0)]
torch.cuda.synchronize()
# the first sampler call of this process: it places the fixed array on the GPU
assert lib.rpgb_sample_noalloc(logits.data_ptr(), n, ctypes.byref(cases[0]), 9, 1, toks.data_ptr(), None) == 0
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
for i, o in enumerate(cases):
    for c in (2, 3):
        assert lib.rpgb_sample_noalloc(logits.data_ptr(), n, ctypes.byref(o), 9, c,
                                       toks[1 + 2 * i + c - 2:].data_ptr(), None) == 0
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
got = toks.cpu().tolist()
want = []
ref = torch.full((1,), -1, dtype=torch.int32, device="cuda")
for o, c in [(cases[0], 1)] + [(o, c) for o in cases for c in (2, 3)]:
    assert lib.rpgb_sample(logits.data_ptr(), n, ctypes.byref(o), 9, c, None, ref.data_ptr(), None) == 0
    want.append(int(ref.item()))
print("RESULT", free0, free1, got[:7], want)
assert free0 == free1, (free0, free1)
assert got[:7] == want, (got, want)
"""


def test_fresh_process_first_call_then_no_device_memory_change():
    """In a process whose first sampler call is rpgb_sample_noalloc: free device
    memory is unchanged across the calls after the first one, and the tokens
    equal rpgb_sample's."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", FRESH.format(root=root)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "RESULT" in r.stdout
