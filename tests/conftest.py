import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "conformance.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    o.build()
    return o


@pytest.fixture(scope="session")
def golden():
    z = np.load(GOLDEN)
    meta = json.loads(bytes(z["__meta__"]).decode())

    class G:
        def __init__(self):
            self.meta = meta

        def raw(self, op, name):
            return z[f"{op}/{name}"]

        def arr(self, op, name, dtype):
            return self.raw(op, name).view(dtype)

        def uniform(self, op):
            return self.raw(op, "uniform").view(np.uint32)

    return G()


@pytest.fixture(scope="session")
def cuda_lib():
    """libtextsift_cuda.so, built if needed (fails loudly if it cannot load)."""
    from textsift_b200 import build
    build.build()
    from textsift_b200 import abi
    return abi.lib()
