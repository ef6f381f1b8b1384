"""The operator-level API (gmmxx_b200.cuda_ops) on the host: the reference's
public names (gmmxx/cuda_ops.py:55-87), its argument checks
(gmmxx/_cuda.py:67-74), the hard-EM operators this engine does not provide,
and the finalize / projection algebra against golden vectors recorded from
the reference's own operators (tests/golden/make_operator_golden.py).  The
algebra runs here on CPU tensors with the operators' CUDA-device check
replaced for the test.  The GPU operator tests (tests/test_gpu_cuda_ops.py)
also run here once with the kernel calls replaced by host fakes, which
checks each operator's own argument handling and finalize rules; the GPU run
checks the kernels."""

import numpy as np
import pytest
import torch

from conftest import load_golden
from gmmxx_b200 import cuda_ops

REFERENCE_NAMES = [
    "canary_add_offset", "spherical_assign", "spherical_logsumexp", "spherical_resp", "soft_update_spherical",
    "blocked_update_spherical", "blocked_update_spherical_sorted", "finalize_spherical", "fused_spherical",
    "approx_topk_update_spherical", "diag_assign", "diag_logsumexp", "diag_resp", "blocked_update_diag",
    "blocked_update_diag_sorted", "finalize_diag", "tied_project", "tied_log_det", "tied_assign", "tied_logsumexp",
    "tied_resp", "tied_finalize", "full_assign", "full_logsumexp", "full_resp", "full_blocked_update",
    "full_finalize", "has_cuda", "require_cuda", "CudaBackendUnavailable", "CudaRuntimeFallback",
]


def test_public_names_match_the_reference():
    assert sorted(cuda_ops.__all__) == sorted(REFERENCE_NAMES)
    for name in REFERENCE_NAMES:
        assert hasattr(cuda_ops, name), name


@pytest.mark.parametrize("name", ["blocked_update_spherical", "blocked_update_spherical_sorted",
                                  "finalize_spherical", "blocked_update_diag", "blocked_update_diag_sorted",
                                  "finalize_diag", "full_blocked_update"])
def test_hard_em_operators_are_not_provided(name):
    with pytest.raises(NotImplementedError, match="hard-assignment"):
        getattr(cuda_ops, name)(torch.zeros(1, 4, 2), torch.zeros(1, 4, dtype=torch.int32), 2)


def test_argument_checks_match_the_reference():
    x = torch.zeros(1, 4, 2)
    means = torch.zeros(1, 3, 2)
    var = torch.ones(1, 3)
    log_w = torch.zeros(1, 3)
    with pytest.raises(ValueError, match="x: must be on a CUDA device"):
        cuda_ops.spherical_assign(x, means, var, log_w)
    with pytest.raises(ValueError, match="canary input: must be on a CUDA device"):
        cuda_ops.canary_add_offset(torch.zeros(4, dtype=torch.int32), 1)
    with pytest.raises(ValueError, match="sums: must be on a CUDA device"):
        cuda_ops.tied_finalize(torch.zeros(1, 3, 2), torch.zeros(1, 2, 2), torch.ones(1, 3), 4, 1e-6)
    if not torch.cuda.is_available():
        assert cuda_ops.has_cuda() is False
    assert issubclass(cuda_ops.CudaRuntimeFallback, RuntimeError)


@pytest.fixture
def host_checks(monkeypatch):
    """Let the operators take CPU tensors (the algebra below launches no kernel)."""
    def check(t, name, dtype=None):
        if dtype is not None and t.dtype != dtype:
            raise ValueError(f"{name}: dtype must be {dtype}, got {t.dtype}")
        return t.contiguous()

    monkeypatch.setattr(cuda_ops, "_check_input", check)
    monkeypatch.setattr(cuda_ops, "require_cuda", lambda: None)


def _t(g, key):
    return torch.from_numpy(np.ascontiguousarray(g[key]))


@pytest.mark.parametrize("case", ["tied_finalize_soft", "tied_finalize_hard"])
def test_tied_finalize_matches_reference(host_checks, case):
    g = load_golden("ops_" + case)
    m, L, w = cuda_ops.tied_finalize(_t(g, "sums"), _t(g, "xx_total"), _t(g, "counts"), int(g["total_n"]),
                                     float(g["reg_covar"]))
    np.testing.assert_allclose(m.numpy(), g["means"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(L.numpy(), g["L"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(w.numpy(), g["weights"], rtol=1e-6, atol=1e-7)


def test_full_finalize_matches_reference(host_checks):
    """Including an empty component and one whose covariance has no Cholesky
    factor: both keep their old mean and factor with weight 0."""
    g = load_golden("ops_full_finalize")
    m, L, w = cuda_ops.full_finalize(_t(g, "sums"), _t(g, "outer_sums"), _t(g, "counts"), _t(g, "old_means"),
                                     _t(g, "old_L"), int(g["total_n"]), float(g["reg_covar"]))
    np.testing.assert_allclose(m.numpy(), g["means"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(L.numpy(), g["L"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(w.numpy(), g["weights"], rtol=1e-6, atol=1e-7)
    assert w[0, 2] == 0 and w[0, 3] == 0
    assert torch.equal(L[0, 3], _t(g, "old_L")[0, 3])


def test_tied_project_and_log_det_match_reference(host_checks):
    g = load_golden("ops_tied_project")
    y = cuda_ops.tied_project(_t(g, "x"), _t(g, "L"))
    np.testing.assert_allclose(y.numpy(), g["y"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(cuda_ops.tied_log_det(_t(g, "L")).numpy(), g["log_det"], rtol=1e-6)


class _FakeOps:
    """Stand-in for engine.CudaOps on the host: the per-iteration prologue
    (variance floor, weight floor and renormalisation) and the spherical
    statistics of exact or top-k EM, from the oracle's float32 logits."""

    def __init__(self, cov, x, k, top_k=None):
        self.cov, self.x, self.k, self.top_k = cov, x, k, top_k
        self.stat_width = x.shape[-1] + 2

    def prepare(self, m, v, w, reg, mw):
        v.clamp_(min=reg)
        w.clamp_(min=mw)
        w /= w.sum(-1, keepdim=True)
        self.params = (m, v, w)

    def accumulate(self, stats, ll):
        lg = _oracle_logits(self.cov, self.x, *self.params).double()
        if self.top_k:
            vals, idx = lg.topk(self.top_k, -1)
            lse = torch.logsumexp(vals, -1)
            r = torch.zeros_like(lg).scatter_(-1, idx, torch.exp(vals - lse[..., None]))
        else:
            lse = torch.logsumexp(lg, -1)
            r = torch.exp(lg - lse[..., None])
        x = self.x.double()
        d = x.shape[-1]
        stats[..., 0] += r.sum(1).float()
        stats[..., 1:1 + d] += (r.transpose(1, 2) @ x).float()
        stats[..., 1 + d] += (r * x.square().sum(-1)[..., None]).sum(1).float()
        ll += lse.sum()


def _oracle_logits(cov, x, means, c, w):
    import oracle

    return torch.from_numpy(oracle.component_logits(cov, x.float().numpy(), means.float().numpy(),
                                                    c.float().numpy(), w.float().numpy()))


@pytest.fixture
def fake_engine(monkeypatch, host_checks):
    """The kernel calls of cuda_ops replaced by host fakes built on the oracle
    (test infrastructure), so that each operator's own argument handling and
    finalize algebra run on the CPU."""
    import contextlib

    from gmmxx_b200 import engine

    monkeypatch.setattr(engine, "assign", lambda cov, x, m, c, w: _oracle_logits(cov, x, m, c, w).argmax(-1))
    monkeypatch.setattr(engine, "score_samples",
                        lambda cov, x, m, c, w: torch.logsumexp(_oracle_logits(cov, x, m, c, w), -1))
    monkeypatch.setattr(engine, "resp",
                        lambda cov, x, m, c, w, ln: torch.exp(_oracle_logits(cov, x, m, c, w) - ln[..., None]))
    monkeypatch.setattr(engine, "canary_add_offset", lambda t, o: t + o)
    monkeypatch.setattr(engine, "CudaOps", _FakeOps)
    monkeypatch.setattr(cuda_ops, "has_cuda", lambda: True)
    monkeypatch.setattr(torch.cuda, "device", lambda d: contextlib.nullcontext())


@pytest.mark.parametrize("name,kwargs", [
    ("test_spherical_and_diag_estep", dict(cov="spherical", dtype=torch.float32)),
    ("test_spherical_and_diag_estep", dict(cov="diag", dtype=torch.bfloat16)),
    ("test_tied_estep", {}),
    ("test_full_estep_matches_reference_golden", {}),
    ("test_soft_update_spherical", {}),
    ("test_fused_spherical", {}),
    ("test_approx_topk_matches_reference_golden", dict(case="approx_small")),
    ("test_approx_topk_matches_reference_golden", dict(case="approx_k150")),
    ("test_approx_topk_arguments", {}),
    ("test_finalize_operators_on_device", dict(case="full_finalize")),
    ("test_canary_and_availability", {}),
])
def test_operator_host_logic_with_a_fake_engine(fake_engine, name, kwargs):
    """The GPU operator tests (tests/test_gpu_cuda_ops.py) run on the CPU with
    the engine faked: this checks the operators' own host logic and the
    tests' expectations; the GPU run checks the kernels behind them."""
    import test_gpu_cuda_ops as gpu_tests

    getattr(gpu_tests, name)(torch.device("cpu"), **kwargs)
