"""Test configuration: the `gpu` marker, import paths, and shared fixtures.

`-m "not gpu"` runs on any machine (oracle against the golden vectors, host-side checks, the C-ABI
library's exports and argument checks). `-m gpu` needs a B200 and runs the CUDA path against the
oracle through the C-ABI.
"""

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
for path in (REPO, REPO / "inference-performance-engineering_b200"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import torch

    cache = {}

    def load(name):
        if name not in cache:
            cache[name] = torch.load(GOLDEN / f"{name}.pt", weights_only=True)
        return cache[name]

    return load
