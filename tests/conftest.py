import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (run with -m gpu on a B200)")


@pytest.fixture(scope="session")
def orc():
    import oracle as O
    return O.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle as O
    if not O.Reference.available():
        pytest.skip("reference build oracle/_ref is not present on this machine")
    return O.Reference()


@pytest.fixture(scope="session")
def golden():
    cache = {}

    def load(name):
        if name not in cache:
            cache[name] = dict(np.load(GOLDEN / f"{name}.npz"))
        return cache[name]
    return load


@pytest.fixture(scope="session")
def gguf_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("gguf")


@pytest.fixture(scope="session")
def be():
    from smallm_engine_b200 import CUDABackend
    b = CUDABackend(0)
    yield b
    b.close()

