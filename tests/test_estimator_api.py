"""Host-side contract of the GMMXX estimator (no kernel runs): constructor
validation and aliases, the backend / use_triton keywords, sklearn-style
get_params / set_params / clone, input validation and the no-fallback rule.
Mirrors the reference's own estimator tests (tests/test_backend_kwarg.py,
tests/test_gmmxx.py:106-201) where the behaviour is the same; where it
differs the test says why."""

import warnings

import pytest
import torch

from gmmxx_b200 import GMMXX
from gmmxx_b200 import _native as nat


def test_constructor_aliases_and_defaults():
    m = GMMXX(n_components=4)
    assert m.k == 4 and m.niter == 100 and m.tol == 1e-4 and m.seed == 0
    assert m.covariance_type == "spherical" and m.init_params == "kmeans" and m.backend == "auto"
    m = GMMXX(k=3, max_iter=7, random_state=5, n_features=2, covariance_type="diagonal")
    assert (m.k, m.niter, m.seed, m.d, m.covariance_type) == (3, 7, 5, 2, "diag")
    # the same value through both names is accepted; conflicting values are not
    assert GMMXX(k=3, n_components=3).k == 3
    with pytest.raises(ValueError, match="conflicting"):
        GMMXX(k=3, n_components=4)
    with pytest.raises(ValueError):
        GMMXX()  # k is required


@pytest.mark.parametrize("kwargs", [
    dict(k=0), dict(k=2, niter=0), dict(k=2, tol=-1.0), dict(k=2, reg_covar=-1e-6), dict(k=2, d=0),
    dict(k=2, chunk_size_data=0), dict(k=2, covariance_type="banded"), dict(k=2, matmul_precision="low"),
    dict(k=2, approx_top_k=0), dict(k=2, init_kmeans_iters=0), dict(k=2, init_kmeans_tol=-1.0),
])
def test_invalid_constructor_arguments(kwargs):
    with pytest.raises(ValueError):
        GMMXX(**kwargs)


def test_backend_keyword_and_use_triton_shim():
    assert GMMXX(n_components=4, backend="cuda").backend == "cuda"
    with pytest.raises(ValueError, match="backend"):
        GMMXX(n_components=4, backend="bogus")
    with warnings.catch_warnings(record=True) as caught:
        warnings.simplefilter("always")
        m = GMMXX(n_components=4, use_triton=False)
    assert m.backend == "auto" and m._legacy_no_triton is True
    assert any(issubclass(w.category, DeprecationWarning) for w in caught)
    with pytest.raises(ValueError, match="backend.*use_triton"):
        GMMXX(n_components=4, backend="cuda", use_triton=False)
    # this engine has no Triton path, so the property is False for every backend
    # (the reference reports True under "auto" / "triton", interface.py:271-283)
    for backend in ("auto", "cuda", "triton", "torch"):
        assert GMMXX(n_components=4, backend=backend).use_triton is False


def test_fit_attributes_start_none():
    m = GMMXX(n_components=4)
    for name in ("means_", "covariances_", "weights_", "labels_", "lower_bound_", "n_iter_",
                 "last_backend_used_", "cuda_estep_enabled_", "cuda_fused_update_enabled_",
                 "cuda_approx_topk_enabled_", "approximate_em_enabled_", "approx_top_k_"):
        assert getattr(m, name) is None, name


def test_get_params_clone_and_set_params():
    m = GMMXX(n_components=8, backend="torch", covariance_type="full", reg_covar=1e-4, approx_top_k=3)
    params = m.get_params()
    assert "backend" in params and "use_triton" not in params
    clone = type(m)(**params)
    assert clone.get_params() == params
    m.set_params(n_components=5, max_iter=3, random_state=9, covariance_type="diagonal", tol=0.0)
    assert (m.k, m.niter, m.seed, m.covariance_type, m.tol) == (5, 3, 9, "diag", 0.0)
    with pytest.raises(ValueError, match="Invalid parameter"):
        m.set_params(bogus=1)
    with pytest.raises(ValueError, match="backend"):
        m.set_params(backend="bogus")
    with pytest.raises(ValueError):
        m.set_params(reg_covar=-1.0)
    assert m.set_params() is m


def test_set_params_use_triton_shim():
    m = GMMXX(n_components=4)
    with warnings.catch_warnings(record=True) as caught:
        warnings.simplefilter("always")
        m.set_params(use_triton=False)
    assert m.backend == "auto" and m._legacy_no_triton is True
    assert any(issubclass(w.category, DeprecationWarning) for w in caught)
    m = GMMXX(n_components=4, backend="cuda")
    with pytest.raises(ValueError, match="backend is already explicit"):
        m.set_params(use_triton=True)
    assert m.backend == "cuda" and m._legacy_no_triton is False


@pytest.mark.parametrize("data,exc", [
    ([[0.0, 1.0]], TypeError),                                     # not a tensor
    (torch.zeros((4, 2), dtype=torch.int64), TypeError),           # not floating point
    (torch.zeros((4,)), ValueError),                               # 1-D
    (torch.zeros((0, 2)), ValueError),                             # no samples
    (torch.zeros((2, 0, 3)), ValueError),
    (torch.zeros((4, 3)), ValueError),                             # d mismatch (d=2)
])
def test_input_validation_before_any_kernel(data, exc):
    m = GMMXX(n_components=2, d=2, device="cpu")
    with pytest.raises(exc):
        m.fit(data)


def test_no_fallback_without_the_engine():
    """A CPU device, or a backend this engine does not provide, raises instead
    of silently running another implementation."""
    x = torch.randn(16, 2)
    with pytest.raises(nat.CudaBackendUnavailable):
        GMMXX(n_components=2, device="cpu").fit(x)
    for backend in ("torch", "triton"):
        with pytest.raises(ValueError, match="not provided"):
            GMMXX(n_components=2, device="cpu", backend=backend).fit(x)


def test_inference_needs_a_fit():
    m = GMMXX(n_components=2, device="cpu")
    for call in (m.predict, m.predict_proba, m.score_samples, m.score, m.bic, m.aic):
        with pytest.raises(RuntimeError, match="not trained"):
            call(torch.randn(4, 2))


def test_gmmxx_backend_environment_variable(monkeypatch):
    """GMMXX_BACKEND picks the backend when the keyword is "auto" (the
    reference's _dispatch.py:128-144); an explicit keyword wins and invalid
    values are ignored.  A backend this engine does not provide raises."""
    x = torch.randn(16, 2)
    monkeypatch.setenv("GMMXX_BACKEND", "torch")
    with pytest.raises(ValueError, match="not provided"):
        GMMXX(n_components=2, device="cpu").fit(x)
    with pytest.raises(nat.CudaBackendUnavailable):  # explicit keyword wins
        GMMXX(n_components=2, device="cpu", backend="cuda").fit(x)
    monkeypatch.setenv("GMMXX_BACKEND", "bogus")
    assert GMMXX(n_components=2)._effective_backend() == "auto"
    with pytest.raises(nat.CudaBackendUnavailable):
        GMMXX(n_components=2, device="cpu").fit(x)
