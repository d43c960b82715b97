"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on CPU."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the CUDA library")


def cuda_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def fc():
    """The CUDA backend.  Fails loudly (no skip, no fallback) when a GPU test
    runs without the library or without a device."""
    import floyd_b200
    floyd_b200.lib()
    return floyd_b200


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def top_margin(logits):
    """Top-1 minus top-2 logit of a row."""
    part = np.partition(logits, -2)
    return float(part[-1] - part[-2])
