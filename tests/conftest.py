"""Shared test configuration.

Markers: ``gpu`` tests need a CUDA device (run with ``-m gpu`` on a B200);
everything else runs on a CPU-only host (``-m "not gpu"``).
"""

import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def golden_cases():
    """The EM fit / inference cases (make_golden.py); the operator cases
    (ops_*.npz, make_operator_golden.py) are loaded by name."""
    names = (os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))
    return sorted(n for n in names if not n.startswith("ops_"))


def load_golden(name):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test collected on a host without CUDA")
    from gmmxx_b200 import _native

    _native.load()  # the engine must be built; no fallback
    return torch.device("cuda:0")
