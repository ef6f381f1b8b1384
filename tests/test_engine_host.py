"""Host-side parts of the EM driver that need no kernel: initial parameters
(the reference's user-init and random-init rules, torch_fallback.py:1348-1894)
on CPU tensors, checked against the oracle's restatement, and the
approx_top_k / window checks."""

import numpy as np
import pytest
import torch

import oracle
from gmmxx_b200 import _native as nat
from gmmxx_b200 import engine


def _data(seed=0, b=2, n=300, d=4):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(b, n, d, generator=g) * 3.0 + 1.0


@pytest.mark.parametrize("cov", ["spherical", "diag", "tied", "full"])
def test_global_covariance_matches_oracle(cov):
    x = _data()
    got = engine.global_covariance(cov, x, 5, 1e-6).numpy()
    fn = {"spherical": lambda: oracle.global_spherical_variance(x.numpy(), 5, 1e-6),
          "diag": lambda: oracle.global_diag_variance(x.numpy(), 5, 1e-6),
          "tied": lambda: oracle.global_tied_covariance(x.numpy(), 1e-6),
          "full": lambda: oracle.global_full_covariance(x.numpy(), 5, 1e-6)}[cov]
    np.testing.assert_allclose(got, fn(), rtol=1e-5, atol=1e-6)


def test_user_init_clamps_and_renormalises():
    """User weights are clamped to 1e-8 and renormalised; spherical / diag
    variances clamped to reg_covar (torch_fallback.py:1634-1643, 1646-1742)."""
    x = _data()
    means = torch.zeros(2, 3, 4)
    w = torch.tensor([[0.0, 1.0, 3.0], [1.0, 1.0, 2.0]])
    var = torch.tensor([[1e-9, 2.0, 3.0], [1.0, 1.0, 1.0]])
    m, c, wt, source = engine.initial_parameters("spherical", x, 3, means, var, w, 1e-6)
    assert source == "user"
    np.testing.assert_allclose(wt.sum(-1).numpy(), 1.0, rtol=1e-6)
    assert wt[0, 0] > 0 and abs(float(wt[0, 2]) - 0.75) < 1e-6
    assert float(c[0, 0]) == pytest.approx(1e-6)
    with pytest.raises(ValueError):
        engine.initial_parameters("spherical", x, 3, means, var[:, :2], w, 1e-6)
    with pytest.raises(ValueError):
        engine.initial_parameters("diag", x, 3, means[:, :, :3], None, None, 1e-6)
    with pytest.raises(ValueError):
        engine.initial_parameters("spherical", x, 3, means, var, w[:, :2], 1e-6)


def test_user_matrix_init_is_symmetrised():
    x = _data()
    a = torch.randn(2, 4, 4)
    m, c, w, _ = engine.initial_parameters("tied", x, 3, torch.zeros(2, 3, 4), a, None, 1e-6)
    assert torch.allclose(c, c.transpose(-1, -2))
    assert torch.allclose(c, 0.5 * (a + a.transpose(-1, -2)))
    np.testing.assert_allclose(w.numpy(), 1.0 / 3)


def test_random_init_draws_rows():
    """init_params "random" draws K rows of x (torch_fallback.py:1384-1387);
    covariances are the global ones and the weights uniform.  ("kmeans" runs
    on the device; host rows, as here, take the same random draw.)"""
    x = _data()
    torch.manual_seed(0)
    m, c, w, source = engine.initial_parameters("diag", x, 5, None, None, None, 1e-6, "kmeans")
    assert source == "random"
    for b in range(2):
        for k in range(5):
            assert (x[b] == m[b, k]).all(-1).any()
    np.testing.assert_allclose(c.numpy(), engine.global_covariance("diag", x, 5, 1e-6).numpy())
    np.testing.assert_allclose(w.numpy(), 0.2)
    with pytest.raises(ValueError, match="init_params"):
        engine.initial_parameters("diag", x, 5, None, None, None, 1e-6, "k-means++")


def test_engine_windows():
    engine.check_window("diag", nat.MAX_D)
    with pytest.raises(nat.UnsupportedShape):
        engine.check_window("diag", nat.MAX_D + 1)
    with pytest.raises(nat.UnsupportedShape):
        engine.check_window("full", nat.MAX_D_FULL + 1)
    with pytest.raises(ValueError):
        engine.cov_code("banded")
    with pytest.raises(ValueError, match="CUDA"):
        engine.check_x(torch.zeros(1, 4, 2))
    with pytest.raises(ValueError, match="shape"):
        engine.check_x(torch.zeros(4, 2))
    with pytest.raises(TypeError):
        engine.check_x([[0.0]])


def test_kernel_path_names():
    from gmmxx_b200 import engine

    assert engine.kernel_path_name({1}) == "tensor-core"
    assert engine.kernel_path_name({0}) == "cuda-core"
    assert "no co-resident cluster" in engine.kernel_path_name({2})
    assert engine.kernel_path_name({1, 2}).startswith("tensor-core + cuda-core")
    assert engine.kernel_path_name(set()) == "none"


def test_accumulate_records_the_no_cluster_fallback(monkeypatch):
    """CudaOps.accumulate keeps what the library reports after each call
    (gmmxx_last_accumulate_path); a tensor-core launch that found no
    co-resident cluster and ran the CUDA-core kernels is named in fit_info's
    kernel_path."""
    import types

    from gmmxx_b200 import _native as nat
    from gmmxx_b200 import engine

    ops = object.__new__(engine.CudaOps)
    ops.top_k, ops.paths = None, set()
    ops.covc, ops.xdt, ops.b, ops.n, ops.d, ops.k = nat.DIAG, nat.BFLOAT16, 1, 70_000, 64, 128
    ops.x = types.SimpleNamespace(data_ptr=lambda: 0)
    ops.ws = torch.zeros(16, dtype=torch.uint8)
    ops.stream = 0
    calls = []
    monkeypatch.setattr(nat, "call", lambda name, *a: calls.append(name))
    monkeypatch.setattr(nat, "last_accumulate_path", lambda: 2)
    ops.accumulate(torch.zeros(4), torch.zeros(1, dtype=torch.float64))
    assert calls == ["gmmxx_em_accumulate"]
    assert ops.kernel_path() == nat.PATH_NAMES[2]
