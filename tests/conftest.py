import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / 'tests' / 'golden'


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200, sm_100a)')


@pytest.fixture(scope='session')
def golden_dir():
    return GOLDEN


def max_rel(x, ref):
    """max|x - ref| / max|ref|  (the tolerance form of the parity contract)."""
    x, ref = x.float().cpu(), ref.float().cpu()
    return ((x - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()
