"""The operator-level API (gmmxx_b200.cuda_ops) on the GPU, against float64
torch references of the reference operators' definitions (gmmxx/_cuda.py:
100-147, 328-412, 783-889, 897-959, 1056-1088, 1100-1243, 1246-1416) and the
golden vectors recorded from the reference's own torch operators
(tests/golden/make_operator_golden.py).  Shapes and checks follow the
reference's operator tests (tests/test_cuda_spherical_safe.py,
test_cuda_diag_safe.py, test_cuda_tied.py, test_cuda_full.py,
test_cuda_approx_topk_spherical.py).

Tolerances: fp32 log-sum-exp and statistics within 1e-4 relative / 1e-4
absolute, responsibilities within 5e-5 absolute (fp32 logits of magnitude
~100 carry ~1e-5 of rounding), labels equal on >= 99.9 % of rows (rows whose
two best logits tie to fp32 rounding may differ)."""

import math

import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu

TOL = dict(rtol=1e-4, atol=1e-4)


def _setup(dev, b=2, n=500, d=12, k=7, dtype=torch.float32, seed=0, cov="spherical"):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(b, n, d, generator=g) * 2.0).to(dtype)
    means = (torch.randn(b, k, d, generator=g) * 2.0).to(dtype)
    shape = (b, k) if cov == "spherical" else (b, k, d)
    var = torch.rand(*shape, generator=g).clamp_min(0.5)
    log_w = torch.log_softmax(torch.randn(b, k, generator=g), dim=-1)
    return [t.to(dev) for t in (x, means, var, log_w)]


def _logits_ref(cov, x, means, var, log_w):
    """float64 logits of the reference's operator definitions."""
    x, means, var, log_w = (t.double().cpu() for t in (x, means, var, log_w))
    d = x.shape[-1]
    diff2 = (x[:, :, None, :] - means[:, None, :, :]).square()
    if cov == "spherical":
        return log_w[:, None] - 0.5 * (diff2.sum(-1) / var[:, None] + d * torch.log(2 * math.pi * var)[:, None])
    return log_w[:, None] - 0.5 * ((diff2 / var[:, None]).sum(-1) + torch.log(2 * math.pi * var).sum(-1)[:, None])


def _tied_logits_ref(x, means, L, log_w):
    x, means, L, log_w = (t.double().cpu() for t in (x, means, L, log_w))
    d = x.shape[-1]
    y = torch.linalg.solve_triangular(L, x.transpose(1, 2), upper=False).transpose(1, 2)
    nu = torch.linalg.solve_triangular(L, means.transpose(1, 2), upper=False).transpose(1, 2)
    logdet = L.diagonal(dim1=-2, dim2=-1).abs().log().sum(-1)
    dist = (y[:, :, None, :] - nu[:, None, :, :]).square().sum(-1)
    return log_w[:, None] - 0.5 * d * math.log(2 * math.pi) - logdet[:, None, None] - 0.5 * dist


def _check_estep(lg, ids, lse, r):
    ref_lse = torch.logsumexp(lg, -1)
    assert ids.dtype == torch.int32 and ids.shape == lg.shape[:2]
    assert (ids.cpu().long() == lg.argmax(-1)).double().mean() >= 0.999
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse.numpy(), **TOL)
    np.testing.assert_allclose(r.cpu().numpy(), torch.exp(lg - ref_lse[..., None]).numpy(), atol=5e-5)


@pytest.mark.parametrize("cov", ["spherical", "diag"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_spherical_and_diag_estep(cuda_device, cov, dtype):
    from gmmxx_b200 import cuda_ops as ops

    x, means, var, log_w = _setup(cuda_device, dtype=dtype, cov=cov)
    assign, lse_fn, resp = {"spherical": (ops.spherical_assign, ops.spherical_logsumexp, ops.spherical_resp),
                            "diag": (ops.diag_assign, ops.diag_logsumexp, ops.diag_resp)}[cov]
    ids = assign(x, means, var, log_w)
    lse = lse_fn(x, means, var, log_w)
    r = resp(x, means, var, log_w, lse)
    _check_estep(_logits_ref(cov, x, means, var, log_w), ids, lse, r)
    # caller-provided outputs are filled and returned
    out_i = torch.empty_like(ids)
    out_l = torch.empty_like(lse)
    out_r = torch.empty_like(r)
    assert assign(x, means, var, log_w, out_i) is out_i and torch.equal(out_i, ids)
    assert lse_fn(x, means, var, log_w, out_l) is out_l and torch.equal(out_l, lse)
    assert resp(x, means, var, log_w, lse, out_r) is out_r and torch.equal(out_r, r)
    with pytest.raises(ValueError, match="var: dtype"):
        assign(x, means, var.double(), log_w)


def test_tied_estep(cuda_device):
    from gmmxx_b200 import cuda_ops as ops

    g = torch.Generator().manual_seed(4)
    b, n, d, k = 2, 400, 6, 5
    x = torch.randn(b, n, d, generator=g) * 2.0
    means = torch.randn(b, k, d, generator=g) * 2.0
    L = torch.tril(torch.randn(b, d, d, generator=g))
    i = torch.arange(d)
    L[:, i, i] = L[:, i, i].abs() + 1.0
    log_w = torch.log_softmax(torch.randn(b, k, generator=g), dim=-1)
    x, means, L, log_w = (t.to(cuda_device) for t in (x, means, L, log_w))
    lse = ops.tied_logsumexp(x, means, L, log_w)
    _check_estep(_tied_logits_ref(x, means, L, log_w), ops.tied_assign(x, means, L, log_w), lse,
                 ops.tied_resp(x, means, L, log_w, lse))
    y = ops.tied_project(x, L)
    np.testing.assert_allclose((L @ y.transpose(1, 2)).transpose(1, 2).cpu().numpy(), x.cpu().numpy(), atol=1e-4)


def test_full_estep_matches_reference_golden(cuda_device):
    from gmmxx_b200 import cuda_ops as ops

    g = load_golden("ops_full_estep")
    x, means, L, log_w = (torch.from_numpy(g[k]).to(cuda_device) for k in ("x", "means", "L", "log_w"))
    ids = ops.full_assign(x, means, L, log_w)
    lse = ops.full_logsumexp(x, means, L, log_w)
    r = ops.full_resp(x, means, L, log_w, lse)
    assert ids.dtype == torch.int32
    assert (ids.cpu().numpy() == g["assign"]).mean() >= 0.999
    np.testing.assert_allclose(lse.cpu().numpy(), g["lse"], **TOL)
    np.testing.assert_allclose(r.cpu().numpy(), g["resp"], atol=5e-5)


def _soft_stats_ref(x, means, var, log_w):
    lg = _logits_ref("spherical", x, means, var, log_w)
    r = torch.softmax(lg, -1)
    xd = x.double().cpu()
    return r.sum(1), r.transpose(1, 2) @ xd, (r * xd.square().sum(-1)[..., None]).sum(1), lg


def test_soft_update_spherical(cuda_device):
    """Finalize rules of the reference operator: mu = sum_x / max(n_k, 1e-8),
    var = max((sum_x2 - n_k |mu|^2) / (max(n_k, 1e-8) D), reg),
    weights = max(n_k / N, 1e-8)."""
    from gmmxx_b200 import cuda_ops as ops

    x, means, var, log_w = _setup(cuda_device, b=1, n=3000, d=8, k=6, seed=3)
    nk, sx, sxx, lg = _soft_stats_ref(x, means, var, log_w)
    n, d = x.shape[1], x.shape[2]
    n_safe = nk.clamp_min(1e-8)
    mu = sx / n_safe[..., None]
    v = ((sxx - nk * mu.square().sum(-1)) / (n_safe * d)).clamp_min(1e-6)
    w = (nk / n).clamp_min(1e-8)
    m2, v2, w2, lse, ids = ops.soft_update_spherical(x, means, var, log_w, 1e-6)
    np.testing.assert_allclose(m2.cpu().numpy(), mu.numpy(), **TOL)
    np.testing.assert_allclose(v2.cpu().numpy(), v.numpy(), **TOL)
    np.testing.assert_allclose(w2.cpu().numpy(), w.numpy(), rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(lse.cpu().numpy(), torch.logsumexp(lg, -1).numpy(), **TOL)
    assert ids.dtype == torch.int32 and (ids.cpu().long() == lg.argmax(-1)).double().mean() >= 0.999
    out = ops.soft_update_spherical(x, means, var, log_w, 1e-6, compute_ids=False, compute_lse=False)
    assert out[3] is None and out[4] is None
    xb, mb = x.to(torch.bfloat16), means.to(torch.bfloat16)
    assert ops.soft_update_spherical(xb, mb, var, log_w, 1e-6)[0].dtype == torch.bfloat16


def test_fused_spherical(cuda_device):
    """The fused operator's rules: mu = sum_x / n_k, var = max((sum_x2 / n_k -
    |mu|^2) / D, reg), weights = n_k / N; a component with n_k = 0 keeps its
    mean and variance with weight 0; the D <= 64, K <= 128 window."""
    from gmmxx_b200 import cuda_ops as ops

    x, means, var, log_w = _setup(cuda_device, b=2, n=2000, d=10, k=5, seed=5)
    means[:, 4] = 1.0e3  # no row reaches it: n_k = 0 exactly
    nk, sx, sxx, lg = _soft_stats_ref(x, means, var, log_w)
    n, d = x.shape[1], x.shape[2]
    live = nk > 0
    mu = sx / torch.where(live, nk, torch.ones_like(nk))[..., None]
    v = ((sxx / torch.where(live, nk, torch.ones_like(nk)) - mu.square().sum(-1)) / d).clamp_min(1e-6)
    m2, v2, w2, lse, ids = ops.fused_spherical(x, means, var, log_w, 1e-6)
    assert not live[:, 4].any()
    np.testing.assert_allclose(m2[:, :4].cpu().numpy(), mu[:, :4].numpy(), **TOL)
    np.testing.assert_allclose(v2[:, :4].cpu().numpy(), v[:, :4].numpy(), **TOL)
    np.testing.assert_allclose(w2.cpu().numpy(), (nk / n).numpy(), rtol=1e-4, atol=1e-6)
    assert torch.equal(m2[:, 4], means[:, 4]) and torch.equal(v2[:, 4], var[:, 4]) and (w2[:, 4] == 0).all()
    np.testing.assert_allclose(lse.cpu().numpy(), torch.logsumexp(lg, -1).numpy(), **TOL)
    assert ids.dtype == torch.int32
    with pytest.raises(ValueError, match="D <= 64"):
        ops.fused_spherical(*_setup(cuda_device, b=1, n=10, d=65, k=3), 1e-6)
    with pytest.raises(ValueError, match="K <= 128"):
        ops.fused_spherical(*_setup(cuda_device, b=1, n=10, d=4, k=129), 1e-6)
    with pytest.raises(ValueError, match="same dtype"):
        ops.fused_spherical(x, means.double(), var, log_w, 1e-6)


@pytest.mark.parametrize("case", ["approx_small", "approx_k150"])
def test_approx_topk_matches_reference_golden(cuda_device, case):
    from gmmxx_b200 import cuda_ops as ops

    g = load_golden("ops_" + case)
    x, means, var, log_w = (torch.from_numpy(g[k]).to(cuda_device) for k in ("x", "means", "var", "log_w"))
    top_k = int(g["top_k"])
    nk, sx, sxx, ll = ops.approx_topk_update_spherical(x, means, var, log_w, top_k=top_k)
    np.testing.assert_allclose(nk.cpu().numpy(), g["nk"], **TOL)
    np.testing.assert_allclose(sx.cpu().numpy(), g["sum_x"], rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(sxx.cpu().numpy(), g["sum_x_sq"], rtol=1e-4, atol=1e-2)
    assert ll.dim() == 0 and ll.dtype == torch.float32
    assert abs(float(ll) - float(g["ll"])) <= 1e-5 * abs(float(g["ll"])) + 1e-2
    # unnormalised log-weights shift every logit, not the selection
    nk2, _, _, ll2 = ops.approx_topk_update_spherical(x, means, var, log_w + 1.5, top_k=top_k)
    np.testing.assert_allclose(nk2.cpu().numpy(), nk.cpu().numpy(), rtol=1e-5, atol=1e-5)
    b, n = x.shape[:2]
    assert abs(float(ll2) - float(ll) - 1.5 * b * n) <= 1e-5 * abs(float(ll)) + 1e-2


def test_approx_topk_arguments(cuda_device):
    from gmmxx_b200 import cuda_ops as ops
    from gmmxx_b200 import _native as nat

    args = _setup(cuda_device, b=1, n=16, d=4, k=8)
    for bad in (0, 8):
        with pytest.raises(ValueError, match="top_k"):
            ops.approx_topk_update_spherical(*args, top_k=bad)
    with pytest.raises(ValueError, match="chunk_size_K"):
        ops.approx_topk_update_spherical(*args, top_k=3, chunk_size_K=0)
    small = ops.approx_topk_update_spherical(*args, top_k=3, chunk_size_K=2)
    full = ops.approx_topk_update_spherical(*args, top_k=3, chunk_size_K=10)
    for a, b in zip(small, full):
        assert torch.equal(a, b)
    with pytest.raises(nat.UnsupportedShape):
        ops.approx_topk_update_spherical(*_setup(cuda_device, b=1, n=16, d=4, k=100), top_k=65)


@pytest.mark.parametrize("case", ["tied_finalize_soft", "tied_finalize_hard", "full_finalize"])
def test_finalize_operators_on_device(cuda_device, case):
    from gmmxx_b200 import cuda_ops as ops

    g = load_golden("ops_" + case)
    t = lambda k: torch.from_numpy(np.ascontiguousarray(g[k])).to(cuda_device)
    if case.startswith("tied"):
        m, L, w = ops.tied_finalize(t("sums"), t("xx_total"), t("counts"), int(g["total_n"]), float(g["reg_covar"]))
    else:
        m, L, w = ops.full_finalize(t("sums"), t("outer_sums"), t("counts"), t("old_means"), t("old_L"),
                                    int(g["total_n"]), float(g["reg_covar"]))
    np.testing.assert_allclose(m.cpu().numpy(), g["means"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(L.cpu().numpy(), g["L"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(w.cpu().numpy(), g["weights"], rtol=1e-6, atol=1e-7)


def test_canary_and_availability(cuda_device):
    from gmmxx_b200 import cuda_ops as ops

    assert ops.has_cuda()
    ops.require_cuda()
    x = torch.arange(100, dtype=torch.int32, device=cuda_device)
    assert torch.equal(ops.canary_add_offset(x, 3), x + 3)
    with pytest.raises(ValueError, match="dtype"):
        ops.canary_add_offset(x.float(), 3)
