import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, 'tests', 'golden')


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA GPU (B200)')
    config.addinivalue_line('markers', 'slow: long-running CPU test')


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN, name + '.npz')))


def golden_layers(g):
    n = int(g['n_layers'])
    return [(g[f'W{i}'], g[f'b{i}']) for i in range(n)]


def close(a, b, rtol=1e-5, atol=1e-6):
    """Reference-parity tolerance: |a - b| <= atol + rtol * |b|."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.allclose(a, b, rtol=rtol, atol=atol)


def max_excess(a, b, rtol=1e-5, atol=1e-6):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b) - (atol + rtol * np.abs(b)), initial=-1))


@pytest.fixture(scope='session')
def cuda_available():
    import torch
    return torch.cuda.is_available()
