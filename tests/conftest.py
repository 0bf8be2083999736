import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: long-running parity case")


def _has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def native():
    from hobbylm_b200 import _native

    _native.lib()
    return _native


@pytest.fixture(scope="session")
def model130():
    from hobbylm_b200 import synth

    return synth.cached_model("130M", 0)


@pytest.fixture(scope="session")
def model500():
    from hobbylm_b200 import synth

    return synth.cached_model("500M", 0)


@pytest.fixture(scope="session")
def oracle130(oracle_mod, model130):
    return oracle_mod.Engine(model130, quant=True)


@pytest.fixture(scope="session")
def engine130(model130):
    from hobbylm_b200 import Engine

    eng = Engine.load(model130, max_batch=8)
    yield eng
    eng.close()
