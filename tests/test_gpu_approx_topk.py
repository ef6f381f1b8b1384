"""Approximate top-k EM on the CUDA-core kernels (topk_rows_kernel,
topk_mstep_kernel) against the numpy oracle of the reference's
_topk_logits_for_chunk / _accumulate_topk_stats (torch_fallback.py:667-767).

* the per-row lists the selection pass leaves in scratch: the oracle's top_k
  components on rows whose k-th and (k+1)-th logits are more than
  1e-3 + 2e-5 |logit| apart (fp32 rounding cannot swap them there), in
  descending logit order, and in the oracle's order where the listed logits
  are that far apart; responsibilities within 2e-5;
* the statistics: equal (rtol 1e-4) to the sums of r * psi(x) over the
  kernel's own lists, computed in float64 on the host;
* the log-likelihood: the sum of the rows' top_k log-sum-exps within 1e-5
  relative;
* whole fits: parameters within the parity tolerance of the oracle's
  approximate EM (1e-4 relative, atol 1e-4);
* equal logits rank the lower component index first.
The golden cases recorded from the reference with approx_top_k run through
tests/test_gpu_parity.py::test_fit_matches_reference_golden."""

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

PARAM_TOL = dict(rtol=1e-4, atol=1e-4)


def _mixture(seed, b, n, d, k, spread=6.0):
    rng = np.random.default_rng(seed)
    centers = rng.uniform(-spread, spread, size=(b, k, d)).astype(np.float32)
    sig = rng.uniform(0.5, 1.5, size=(b, k)).astype(np.float32)
    comp = rng.integers(0, k, size=(b, n))
    x = np.take_along_axis(centers, comp[..., None], 1) + np.take_along_axis(sig, comp, 1)[..., None] * \
        rng.standard_normal((b, n, d)).astype(np.float32)
    init = np.stack([x[i, rng.choice(n, k, replace=False)] for i in range(b)]).astype(np.float32)
    return x.astype(np.float32), init


def _init_cov(cov, x, k):
    if cov == "tied":
        return oracle.global_tied_covariance(x, 1e-6)
    return {"spherical": oracle.global_spherical_variance, "diag": oracle.global_diag_variance,
            "full": oracle.global_full_covariance}[cov](x, k, 1e-6)


def _psi(cov, x):
    """Per-row statistic features in the C ABI's stats layout."""
    x = x.astype(np.float64)
    one = np.ones(x.shape[:-1] + (1,))
    if cov == "spherical":
        return np.concatenate([one, x, np.square(x).sum(-1, keepdims=True)], -1)
    if cov == "diag":
        return np.concatenate([one, x, np.square(x)], -1)
    if cov == "tied":
        return np.concatenate([one, x], -1)
    i, j = np.triu_indices(x.shape[-1])
    return np.concatenate([one, x, x[..., i] * x[..., j]], -1)


def _lists(ops, b, n, top_k):
    nb = b * n * top_k * 4
    half = ops.scratch.numel() // 2
    idx = ops.scratch[:nb].view(torch.int32).reshape(b, n, top_k).cpu().numpy()
    r = ops.scratch[half:half + nb].view(torch.float32).reshape(b, n, top_k).cpu().numpy()
    return idx, r


def _accumulate(cuda_device, cov, xt, means, covt, weights, k, top_k):
    from gmmxx_b200 import engine

    b = xt.shape[0]
    ops = engine.CudaOps(cov, xt, k, top_k)
    ops.prepare(means, covt, weights, 1e-6, 1e-8)  # clamps / renormalises in place, as each iteration does
    stats = torch.zeros((b, k, ops.stat_width), dtype=torch.float32, device=cuda_device)
    ll = torch.zeros((1,), dtype=torch.float64, device=cuda_device)
    ops.accumulate(stats, ll)
    ops.check_status()
    torch.cuda.synchronize()
    return ops, stats.cpu().numpy().astype(np.float64), float(ll.item())


@pytest.mark.parametrize("cov,b,n,d,k,top_k,dtype", [
    ("spherical", 2, 5000, 16, 150, 6, torch.float32),   # three component tiles, the last one partial
    ("diag", 1, 7000, 8, 70, 3, torch.bfloat16),
    ("tied", 2, 3000, 12, 90, 4, torch.float32),
    ("full", 1, 3000, 5, 65, 2, torch.float16),
    ("diag", 1, 4000, 24, 200, 64, torch.float32),       # the largest top_k
    ("spherical", 1, 2000, 4, 3, 2, torch.float32),      # K inside one tile
    ("spherical", 1, 1000, 8, 40, 1, torch.float32),     # top_k = 1: hard responsibilities
])
def test_topk_lists_and_statistics(cuda_device, cov, b, n, d, k, top_k, dtype):
    x, init = _mixture(31 + k + top_k, b, n, d, k)
    xt = torch.from_numpy(x).to(dtype).to(cuda_device)
    xf = xt.float().cpu().numpy()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)
    means, covt, weights = t(init), t(_init_cov(cov, xf, k)), t(np.full((b, k), 1.0 / k, np.float32))
    ops, stats, ll = _accumulate(cuda_device, cov, xt, means, covt, weights, k, top_k)
    idx, r = _lists(ops, b, n, top_k)

    assert ((idx >= 0) & (idx < k)).all()
    assert (np.diff(np.sort(idx, -1), axis=-1) > 0).all()  # distinct components per row
    np.testing.assert_allclose(r.sum(-1), 1.0, atol=1e-5)

    lg = oracle.component_logits(cov, xf, means.cpu().numpy(), covt.cpu().numpy(), weights.cpu().numpy())
    order = np.argsort(-lg, axis=-1, kind="stable")
    srt = np.take_along_axis(lg, order, -1).astype(np.float64)
    # rows whose list boundary is unambiguous: the oracle's components
    margin = 1e-3 + 2e-5 * np.abs(srt[..., :1])  # fp32 rounding of the two implementations' logits
    safe = srt[..., top_k - 1] - srt[..., top_k] > margin[..., 0]
    assert safe.mean() > 0.9
    np.testing.assert_array_equal(np.sort(idx, -1)[safe], np.sort(order[..., :top_k], -1)[safe])
    # every list in descending logit order (to fp32 rounding), and in the
    # oracle's order where its logits are separated
    lk = np.take_along_axis(lg, idx.astype(np.int64), -1).astype(np.float64)
    assert (np.diff(lk, axis=-1) <= margin).all()
    strict = safe
    if top_k > 1:
        strict = safe & (np.diff(srt[..., :top_k], axis=-1) < -margin).all(-1)
    np.testing.assert_array_equal(idx[strict], order[..., :top_k][strict])
    vals = srt[..., :top_k]
    mx = vals[..., :1]
    lse = (mx + np.log(np.exp(vals - mx).sum(-1, keepdims=True)))[..., 0]
    np.testing.assert_allclose(r[safe], np.exp(lk - lse[..., None])[safe], atol=2e-5)

    # statistics from the kernel's own lists, in float64
    psi = _psi(cov, xf)
    want = np.zeros((b, k, psi.shape[-1]))
    for bb in range(b):
        contrib = r[bb].astype(np.float64)[..., None] * psi[bb][:, None, :]
        np.add.at(want[bb], idx[bb].ravel(), contrib.reshape(-1, psi.shape[-1]))
    np.testing.assert_allclose(stats, want, rtol=1e-4, atol=1e-5 * np.abs(want).max())
    assert abs(ll - lse.sum()) <= 1e-5 * abs(lse.sum()) + 1e-3


@pytest.mark.parametrize("cov,b,n,d,k,top_k", [
    ("spherical", 1, 8000, 16, 100, 4),
    ("diag", 2, 6000, 8, 70, 3),
    ("tied", 1, 5000, 12, 80, 2),
    ("full", 1, 4000, 5, 66, 3),
])
def test_approx_fit_matches_oracle(cuda_device, cov, b, n, d, k, top_k):
    from gmmxx_b200 import engine

    x, init = _mixture(51 + k, b, n, d, k)
    icov = _init_cov(cov, x, k)
    w = np.full((b, k), 1.0 / k, np.float32)
    ref = oracle.fit(cov, x, k, 3, 0.0, init, icov, w, approx_top_k=top_k)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)
    labels, means, c, wt, info = engine.em_fit(cov, t(x), k, max_iters=3, tol=0.0, init_means=t(init),
                                               init_variances=t(icov), init_weights=t(w), approx_top_k=top_k)
    assert info["approximate_em_enabled"] and info["approx_top_k"] == top_k
    np.testing.assert_allclose(means.cpu().numpy(), ref[1], **PARAM_TOL)
    np.testing.assert_allclose(c.cpu().numpy(), ref[2], **PARAM_TOL)
    np.testing.assert_allclose(wt.cpu().numpy(), ref[3], **PARAM_TOL)
    assert abs(info["lower_bound"] - ref[4]["lower_bound"]) <= 1e-4 * abs(ref[4]["lower_bound"])
    assert (labels.cpu().numpy() == ref[0]).mean() >= 0.999


def test_equal_logits_rank_lower_index_first(cuda_device):
    """A populated component a is copied into b = a + 64 (another component
    tile) and a populated a2 into b2 = a2 + 1 (the same tile): their logits
    are equal, the lower index ranks first, and with top_k = 1 the copy is
    never chosen."""
    k, d = 80, 8
    x, init = _mixture(7, 1, 4000, d, k)
    icov = _init_cov("diag", x, k)
    w = np.full((1, k), 1.0 / k, np.float32)
    counts = np.bincount(oracle.assign("diag", x, init, icov, w)[0], minlength=k)
    a = int(np.argmax(counts[:16]))
    a2 = 16 + int(np.argmax(counts[16:62]))
    pairs = ((a, a + 64), (a2, a2 + 1))
    for lo, hi in pairs:
        init[0, hi] = init[0, lo]
        icov[0, hi] = icov[0, lo]
    t = lambda a_: torch.from_numpy(np.ascontiguousarray(a_)).to(cuda_device)
    xt = t(x)
    ops, _, _ = _accumulate(cuda_device, "diag", xt, t(init), t(icov), t(w), k, 1)
    idx, r = _lists(ops, 1, x.shape[1], 1)
    assert not np.isin(idx, [hi for _, hi in pairs]).any()
    ops, _, _ = _accumulate(cuda_device, "diag", xt, t(init), t(icov), t(w), k, 2)
    idx, r = _lists(ops, 1, x.shape[1], 2)
    for lo, hi in pairs:
        rows = np.isin(idx[0, :, 0], [lo, hi])
        assert counts[lo] > 5 and rows.sum() >= 0.9 * counts[lo]
        assert (idx[0, rows, 0] == lo).all() and (idx[0, rows, 1] == hi).all()
        np.testing.assert_allclose(r[0, rows], 0.5, atol=1e-6)


def test_estimator_approx_flags_and_exact_when_top_k_covers_k(cuda_device):
    """GMMXX(approx_top_k=...) reports the approximation like the reference
    (interface.py:388-392); approx_top_k >= K is exact EM, bit for bit."""
    from gmmxx_b200 import GMMXX

    x, _ = _mixture(12, 1, 4000, 8, 12)
    xt = torch.from_numpy(x[0]).to(cuda_device)
    g = GMMXX(k=12, niter=4, covariance_type="diag", backend="cuda", seed=3, approx_top_k=3).fit(xt)
    assert g.approximate_em_enabled_ and g.approx_top_k_ == 3 and g.cuda_approx_topk_enabled_
    assert torch.isfinite(g.means_).all() and torch.isfinite(g.covariances_).all()
    p = g.predict_proba(xt)  # prediction stays exact
    assert torch.allclose(p.sum(-1), torch.ones(4000, device=cuda_device), atol=1e-4)
    e = GMMXX(k=12, niter=4, covariance_type="diag", backend="cuda", seed=3, approx_top_k=12).fit(xt)
    assert not e.approximate_em_enabled_ and e.approx_top_k_ is None and not e.cuda_approx_topk_enabled_
    f = GMMXX(k=12, niter=4, covariance_type="diag", backend="cuda", seed=3).fit(xt)
    assert torch.equal(e.means_, f.means_) and torch.equal(e.covariances_, f.covariances_)


def test_streamed_approx_fit_matches_resident(cuda_device):
    """Host-streamed chunks give the same lists per row; only the statistics'
    summation order differs."""
    from gmmxx_b200 import engine, large_n

    x, init = _mixture(9, 1, 10000, 12, 70)
    icov = oracle.global_diag_variance(x, 70, 1e-6)
    w = np.full((1, 70), 1 / 70, np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    a = engine.em_fit("diag", t(x).to(cuda_device), 70, max_iters=3, tol=0.0, init_means=t(init),
                      init_variances=t(icov), init_weights=t(w), approx_top_k=4)
    b = large_n.em_fit_streamed("diag", t(x), 70, device=cuda_device, chunk_rows=1500, max_iters=3, tol=0.0,
                                init_means=t(init), init_variances=t(icov), init_weights=t(w), approx_top_k=4)
    assert b[4]["approximate_em_enabled"] and b[4]["approx_top_k"] == 4
    for u, v in zip(a[1:4], b[1:4]):
        np.testing.assert_allclose(u.cpu().numpy(), v.cpu().numpy(), **PARAM_TOL)
    assert (a[0] == b[0]).float().mean().item() >= 0.999
