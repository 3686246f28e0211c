import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

MODEL_CACHE = os.environ.get("STRASGPT_MODEL_CACHE", "/tmp/strasgpt_models")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")
    config.addinivalue_line("markers", "slow: full-size benchmark configurations")


def _ensure_built():
    from strasgpt_b200 import _paths
    import oracle
    if not (os.path.exists(_paths.main_lib()) and os.path.exists(_paths.synth_lib())):
        from strasgpt_b200 import build
        build.build()
    if not os.path.exists(oracle.ORACLE_LIB):
        oracle.build()


@pytest.fixture(scope="session", autouse=True)
def built_libraries():
    _ensure_built()


def model_dir(cfg, seed: int = 0) -> str:
    """Write (or reuse) the synthetic model of `cfg` and return its path."""
    from strasgpt_b200 import synth
    return synth.write_model(os.path.join(MODEL_CACHE, f"{cfg.name}_s{seed}"),
                             cfg, seed=seed)


@pytest.fixture(scope="session")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch
