import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def lcg(seed):
    """The reference tests' 64-bit LCG (crates/voxrt/tests/kernels.rs:7-12): returns (next_seed, value)."""
    seed = (seed * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
    return seed, seed >> 33


class LCG:
    def __init__(self, seed):
        self.seed = seed

    def next(self):
        self.seed, v = lcg(self.seed)
        return v


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle

    oracle.build()
    return oracle
