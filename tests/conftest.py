import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    """The committed golden fixtures (reference CPU functions executed by tests/golden/jsmini.py)."""
    import json

    import numpy as np

    here = os.path.join(ROOT, "tests", "golden")
    arrays = np.load(os.path.join(here, "golden.npz"))
    cases = json.load(open(os.path.join(here, "golden.json")))["cases"]
    return {c["name"]: (c, {k.split("/", 1)[1]: arrays[k] for k in arrays.files if k.startswith(c["name"] + "/")})
            for c in cases}


@pytest.fixture(scope="session")
def eng():
    """One AttentionEngine (library context) on cuda:0 for the GPU tests."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from brimkern_b200.engine import AttentionEngine
    e = AttentionEngine(0)
    yield e
    e.close()
