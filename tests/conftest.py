"""Shared fixtures.  GPU tests are marked ``gpu`` and run on a B200 box."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope="session")
def model_cache(tmp_path_factory):
    d = os.environ.get("RPGB_MODEL_CACHE") or str(tmp_path_factory.mktemp("models"))
    os.environ["RPGB_MODEL_CACHE"] = d
    return d


# The toy models carry weights N(0, 0.06) instead of the benchmark's N(0, 0.02):
# with the smaller weights a two-layer model's residual stream is dominated by
# the token embedding, the tied lm_head then favours the input token, and
# greedy decoding repeats one id -- a comparison that proves little.  These
# are the models of the reference fixtures in tests/golden/ref_engine.npz.
TOY_STD = 0.06


def toy_model(name, seed, model_cache):
    from dataclasses import replace

    from rpgbarenginecuda_b200 import synthetic

    return synthetic.cached_model(replace(synthetic.PRESETS[name], weight_std=TOY_STD), seed=seed,
                                  cache_dir=model_cache)


@pytest.fixture(scope="session")
def tiny_model(model_cache):
    return toy_model("tiny", 1, model_cache)


@pytest.fixture(scope="session")
def tiny_g4_model(model_cache):
    return toy_model("tiny-g4", 2, model_cache)


@pytest.fixture(scope="session")
def small_model(model_cache):
    return toy_model("small", 3, model_cache)


@pytest.fixture(scope="session")
def wide_model(model_cache):
    return toy_model("wide", 4, model_cache)


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle

    return Oracle()
