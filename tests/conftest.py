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


def golden_cases(prefix=None):
    """The EM fit / inference cases (make_golden.py); the operator cases
    (ops_*.npz, make_operator_golden.py) are loaded by name.  With ``prefix``,
    the cases of that family instead (e.g. "init_kmeanspp_",
    make_kmeans_golden.py)."""
    names = (os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))
    if prefix is not None:
        return sorted(n for n in names if n.startswith(prefix))
    return sorted(n for n in names if not n.startswith(("ops_", "init_")))


def kmeans_pp_reference_draws(x, k, seed):
    """The random draws of the reference's k-means++ for rows ``x`` (B, N, D)
    (CPU torch tensor) after ``torch.manual_seed(seed)``, in its order
    (torch_fallback.py:1400-1420): the row sample (``randperm`` when it is a
    strict subset), the first centres (``randint``), then (B, L) uniforms per
    further centre.  Returns (sample, first_idx, uniforms (K-1, B, L))."""
    import math

    import torch

    import oracle

    b, n, d = x.shape
    s = oracle.kmeans_pp_sample_size(n, k)
    torch.manual_seed(seed)
    sample = x if s == n else x.index_select(1, torch.randperm(n)[:s])
    first = torch.randint(0, s, (b,))
    trials = 2 + int(math.log(float(k)))
    u = [torch.rand((b, trials), dtype=torch.float32) for _ in range(k - 1)]
    u = torch.stack(u) if u else torch.zeros((0, b, trials))
    return sample, first, u


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
