"""Test configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs on any host (oracle vs golden vectors, host logic, library
symbol checks, multi-process gloo logic); `-m gpu` needs a B200 and calls the
CUDA library through its C-ABI, comparing against the CPU oracle.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / 'tests' / 'golden'
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA GPU (B200, sm_100a)')


@pytest.fixture(scope='session')
def golden():
    cache = {}

    def load(name):
        if name not in cache:
            cache[name] = dict(np.load(GOLDEN / name))
        return cache[name]
    return load


@pytest.fixture(scope='session')
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail('GPU test collected without a CUDA device')
    import odie_b200
    odie_b200.build()
    return torch.device('cuda:0')
