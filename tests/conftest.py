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


@pytest.fixture(scope="session")
def tiny_model(model_cache):
    from rpgbarenginecuda_b200 import synthetic

    return synthetic.cached_model("tiny", seed=1, cache_dir=model_cache)


@pytest.fixture(scope="session")
def tiny_g4_model(model_cache):
    from rpgbarenginecuda_b200 import synthetic

    return synthetic.cached_model("tiny-g4", seed=2, cache_dir=model_cache)


@pytest.fixture(scope="session")
def small_model(model_cache):
    from rpgbarenginecuda_b200 import synthetic

    return synthetic.cached_model("small", seed=3, cache_dir=model_cache)


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle

    return Oracle()
