"""pytest configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs on a CPU-only machine: the oracle against the
reference's known-answer tests, the host-side validation of the C ABI, and
the multi-rank host logic on gloo.  `-m gpu` runs the parity tests proper,
which call the CUDA library through its C ABI on a B200.
"""
import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def kats():
    with open(os.path.join(GOLDEN, "reference_kats.json")) as f:
        return json.load(f)["cases"]


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    o.lib()
    return o
