"""pytest configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs here without a GPU: the oracle against the golden vectors,
host-side logic (shard planning, LSE merge, gloo ranks) and that the C-ABI
library loads and exports every declared symbol.  `-m gpu` runs the parity
tests proper through the C ABI on a B200.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "engine")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def lib():
    from llama3pure_b200.build import build
    from llama3pure_b200.attn import load_library

    build()
    return load_library()


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(os.path.join(ROOT, "tests", "golden", "attn_golden.npz"))
