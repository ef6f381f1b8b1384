"""Numpy restatement of the reference's soft-EM GMM path (TEST INFRASTRUCTURE).

Every function here restates one function of the reference's PyTorch
implementation, ``gmmxx/torch_fallback.py`` (cited per function as
``torch_fallback.py:<lines>``).  Arithmetic follows the reference: float32
storage and float32 arithmetic, the expanded-distance logits with the distance
clamped at zero, a streaming logsumexp over component chunks, and the exact
M-step finalize / empty-cluster rules.  ``dtype=np.float64`` runs the same
algorithm in double precision, which the tests use to measure the float32 noise
floor.

This module is the parity checker.  It is imported only by tests, by the smoke
entry and by the benchmark's CPU-baseline leg; the CUDA engine never calls it.
Parity pin: ``tests/test_oracle_golden.py`` compares it with golden vectors
recorded from the reference (``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import math
from typing import Dict, Tuple

import numpy as np

__all__ = [
    "LOG_2PI",
    "precision_and_logdet",
    "spherical_logits",
    "diag_logits",
    "tied_logits",
    "full_logits",
    "component_logits",
    "stream_logsumexp",
    "fit",
    "fit_spherical",
    "fit_diag",
    "fit_tied",
    "fit_full",
    "assign",
    "score_samples",
    "predict_proba",
    "global_spherical_variance",
    "global_diag_variance",
    "global_tied_covariance",
    "global_full_covariance",
    "kmeans_pp_sample_size",
    "kmeans_plus_plus",
    "nearest_centroid",
    "lloyd",
    "hard_label_init",
]

LOG_2PI = math.log(2.0 * math.pi)


def _sym(m: np.ndarray) -> np.ndarray:
    """torch_fallback.py:304-305 (_symmetrize_matrix)."""
    return 0.5 * (m + np.swapaxes(m, -1, -2))


def _chol_ok(a: np.ndarray) -> Tuple[np.ndarray, bool]:
    try:
        return np.linalg.cholesky(a), True
    except np.linalg.LinAlgError:
        return np.zeros_like(a), False


def precision_and_logdet(cov: np.ndarray, dtype=np.float32) -> Tuple[np.ndarray, np.ndarray]:
    """torch_fallback.py:316-334 (_precision_and_logdet).

    Symmetrise, Cholesky-factor every matrix of the batch; if any matrix is not
    positive definite, retry the whole batch with ``cov + jitter*I`` for
    jitter = 1e-6, 1e-5, ... 1e-1 and keep the first jitter at which every
    matrix factors.  Returns ``(cholesky_inverse(L), 2*sum(log(diag(L))))``.
    """
    cov = _sym(np.asarray(cov, dtype=dtype))
    d = cov.shape[-1]
    flat = cov.reshape(-1, d, d)
    chol = np.empty_like(flat)
    ok_all = True
    for i in range(flat.shape[0]):
        chol[i], ok = _chol_ok(flat[i])
        ok_all &= ok
    if not ok_all:
        eye = np.eye(d, dtype=dtype)
        jitter = 1e-6
        for _ in range(6):
            ok_all = True
            for i in range(flat.shape[0]):
                chol[i], ok = _chol_ok((flat[i] + dtype(jitter) * eye).astype(dtype))
                ok_all &= ok
            if ok_all:
                break
            jitter *= 10.0
        if not ok_all:
            raise np.linalg.LinAlgError("covariance not positive definite after jitter ladder")
    chol = chol.reshape(cov.shape)
    linv = np.linalg.inv(chol).astype(dtype)
    precision = (np.swapaxes(linv, -1, -2) @ linv).astype(dtype)
    logdet = (2.0 * np.log(np.diagonal(chol, axis1=-2, axis2=-1)).sum(axis=-1)).astype(dtype)
    return precision, logdet


# ---------------------------------------------------------------------------
# Logits (expanded distance, clamped at zero)
# ---------------------------------------------------------------------------


def spherical_logits(x, x_sq, means, variances, log_weights, dtype=np.float32):
    """torch_fallback.py:337-354 (_compute_chunk_logits)."""
    d = x.shape[-1]
    means_sq = np.square(means).sum(axis=-1)
    dist = x_sq[:, :, None] - dtype(2.0) * (x @ np.swapaxes(means, 1, 2)) + means_sq[:, None, :]
    dist = np.maximum(dist, dtype(0.0))
    log_norm = (d * (LOG_2PI + np.log(variances)))[:, None, :].astype(dtype)
    return (log_weights[:, None, :] - dtype(0.5) * (dist / variances[:, None, :] + log_norm)).astype(dtype)


def _diag_terms(means, variances, dtype=np.float32):
    """Loop-invariant diag terms, torch_fallback.py:2491-2494."""
    precision = (dtype(1.0) / np.maximum(variances, dtype(1e-30))).astype(dtype)
    weighted_means = (means * precision).astype(dtype)
    mpm = (means * weighted_means).sum(axis=-1).astype(dtype)
    logdet = np.log(np.maximum(variances, dtype(1e-30))).sum(axis=-1).astype(dtype)
    return precision, weighted_means, mpm, logdet


def diag_logits(x, means, variances, log_weights, terms=None, dtype=np.float32):
    """torch_fallback.py:357-397 (_compute_diag_chunk_logits)."""
    d = x.shape[-1]
    precision, wm, mpm, logdet = terms if terms is not None else _diag_terms(means, variances, dtype)
    dist = (np.square(x) @ np.swapaxes(precision, 1, 2)) - dtype(2.0) * (x @ np.swapaxes(wm, 1, 2)) + mpm[:, None, :]
    dist = np.maximum(dist, dtype(0.0))
    log_norm = (dtype(d * LOG_2PI) + logdet).astype(dtype)
    return (log_weights[:, None, :] - dtype(0.5) * (dist + log_norm[:, None, :])).astype(dtype)


def _matrix_terms(means, covariances, cov_type, dtype=np.float32):
    """Loop-invariant tied/full terms, torch_fallback.py:2868-2873."""
    precision, logdet = precision_and_logdet(covariances, dtype)
    if cov_type == "full":
        pm = np.einsum("bkde,bke->bkd", precision, means).astype(dtype)
    else:
        pm = (means @ np.swapaxes(precision, 1, 2)).astype(dtype)
    mpm = (means * pm).sum(axis=-1).astype(dtype)
    return precision, logdet, pm, mpm


def full_logits(x, means, covariances, log_weights, terms=None, dtype=np.float32):
    """torch_fallback.py:400-432 (_compute_full_chunk_logits)."""
    d = x.shape[-1]
    precision, logdet, pm, mpm = terms if terms is not None else _matrix_terms(means, covariances, "full", dtype)
    xpx = np.einsum("bnd,bkde,bne->bnk", x, precision, x, optimize=True).astype(dtype)
    cross = x @ np.swapaxes(pm, 1, 2)
    quad = np.maximum(xpx - dtype(2.0) * cross + mpm[:, None, :], dtype(0.0))
    log_norm = (dtype(d * LOG_2PI) + logdet).astype(dtype)
    return (log_weights[:, None, :] - dtype(0.5) * (quad + log_norm[:, None, :])).astype(dtype)


def tied_logits(x, means, covariance, log_weights, terms=None, dtype=np.float32):
    """torch_fallback.py:435-465 (_compute_tied_chunk_logits)."""
    d = x.shape[-1]
    precision, logdet, pm, mpm = terms if terms is not None else _matrix_terms(means, covariance, "tied", dtype)
    xpx = np.einsum("bnd,bde,bne->bn", x, precision, x, optimize=True).astype(dtype)
    cross = x @ np.swapaxes(pm, 1, 2)
    quad = np.maximum(xpx[:, :, None] - dtype(2.0) * cross + mpm[:, None, :], dtype(0.0))
    log_norm = (dtype(d * LOG_2PI) + logdet).astype(dtype)
    return (log_weights[:, None, :] - dtype(0.5) * (quad + log_norm[:, None, None])).astype(dtype)


class _Model:
    """Loop-invariant per-parameter-set terms so chunked calls do not redo them."""

    def __init__(self, cov_type, means, cov, weights, dtype=np.float32):
        self.cov_type = cov_type
        self.dtype = dtype
        self.means = np.asarray(means, dtype=dtype)
        self.cov = np.asarray(cov, dtype=dtype)
        self.log_weights = np.log(np.asarray(weights, dtype=dtype)).astype(dtype)
        self.terms = None
        if cov_type == "diag":
            self.terms = _diag_terms(self.means, self.cov, dtype)
        elif cov_type in ("tied", "full"):
            self.terms = _matrix_terms(self.means, self.cov, cov_type, dtype)

    def logits(self, x, x_sq, k0, k1):
        dt = self.dtype
        m = self.means[:, k0:k1]
        lw = self.log_weights[:, k0:k1]
        if self.cov_type == "spherical":
            return spherical_logits(x, x_sq, m, self.cov[:, k0:k1], lw, dt)
        if self.cov_type == "diag":
            p, wm, mpm, ld = self.terms
            return diag_logits(x, m, None, lw, (p[:, k0:k1], wm[:, k0:k1], mpm[:, k0:k1], ld[:, k0:k1]), dt)
        p, ld, pm, mpm = self.terms
        if self.cov_type == "full":
            return full_logits(x, m, None, lw, (p[:, k0:k1], ld[:, k0:k1], pm[:, k0:k1], mpm[:, k0:k1]), dt)
        return tied_logits(x, m, None, lw, (p, ld, pm[:, k0:k1], mpm[:, k0:k1]), dt)


def component_logits(cov_type, x, means, cov, weights, dtype=np.float32):
    """All (B, N, K) logits for one parameter set (test helper)."""
    x = np.asarray(x, dtype=dtype)
    model = _Model(cov_type, means, cov, weights, dtype)
    x_sq = np.square(x).sum(axis=-1).astype(dtype)
    return model.logits(x, x_sq, 0, model.means.shape[1])


def stream_logsumexp(model: _Model, x, x_sq, chunk_size_K):
    """torch_fallback.py:468-499 / 502-563 / 566-596 (streaming log-normaliser).

    Online max / rescaled exp-sum across component chunks of ``chunk_size_K``.
    """
    dt = model.dtype
    bsz, n, _ = x.shape
    k = model.means.shape[1]
    mx = np.full((bsz, n), -np.inf, dtype=dt)
    s = np.zeros((bsz, n), dtype=dt)
    for k0 in range(0, k, chunk_size_K):
        lg = model.logits(x, x_sq, k0, min(k0 + chunk_size_K, k))
        new_mx = np.maximum(mx, lg.max(axis=-1))
        with np.errstate(invalid="ignore"):
            s = s * np.exp(mx - new_mx) + np.exp(lg - new_mx[:, :, None]).sum(axis=-1)
        mx = new_mx
    return (mx + np.log(s)).astype(dt)


def _logsumexp(lg):
    """torch.logsumexp over the last axis."""
    mx = lg.max(axis=-1)
    return (mx + np.log(np.exp(lg - mx[..., None]).sum(axis=-1))).astype(lg.dtype)


# ---------------------------------------------------------------------------
# Initial-parameter helpers (used when a caller injects only init means)
# ---------------------------------------------------------------------------


def global_spherical_variance(x, n_components, reg_covar, dtype=np.float32):
    """torch_fallback.py:1348-1363 (_global_spherical_variance)."""
    x = np.asarray(x, dtype=dtype)
    d = x.shape[-1]
    mean = x.mean(axis=1)
    second = np.square(x).sum(axis=-1).mean(axis=1)
    gv = np.maximum(second - np.square(mean).sum(axis=-1), 0.0) / float(d)
    gv = np.maximum(gv, reg_covar).astype(dtype)
    return np.repeat(gv[:, None], n_components, axis=1)


def global_diag_variance(x, n_components, reg_covar, dtype=np.float32):
    """torch_fallback.py:1366-1369 (_global_diag_variance)."""
    x = np.asarray(x, dtype=dtype)
    c = x - x.mean(axis=1, keepdims=True)
    gv = np.maximum(np.square(c).mean(axis=1), reg_covar).astype(dtype)
    return np.repeat(gv[:, None, :], n_components, axis=1)


def global_tied_covariance(x, reg_covar, dtype=np.float32):
    """torch_fallback.py:1372-1376 (_global_tied_covariance)."""
    x = np.asarray(x, dtype=dtype)
    n, d = x.shape[1], x.shape[2]
    c = x - x.mean(axis=1, keepdims=True)
    cov = (np.swapaxes(c, 1, 2) @ c) / float(n)
    return (_sym(cov) + reg_covar * np.eye(d, dtype=dtype)).astype(dtype)


def global_full_covariance(x, n_components, reg_covar, dtype=np.float32):
    """torch_fallback.py:1379-1381 (_global_full_covariance)."""
    cov = global_tied_covariance(x, reg_covar, dtype)
    return np.repeat(cov[:, None], n_components, axis=1)


def _init_params(cov_type, x, k, init_means, init_cov, init_weights, reg_covar, dtype):
    """User-init branches of torch_fallback.py:1646-1682 (spherical), 1706-1720
    (diag), 1776-1790 (full), 1836-1850 (tied) with _validate_init_weights
    (1634-1643)."""
    bsz = x.shape[0]
    if init_means is None:
        raise ValueError("the oracle needs injected init_means (identical-init parity)")
    means = np.array(init_means, dtype=dtype, copy=True)
    if means.ndim != 3:
        raise ValueError("init_means must have shape (B, K, D)")
    weights = (
        np.full((bsz, k), 1.0 / float(k), dtype=dtype)
        if init_weights is None
        else np.array(init_weights, dtype=dtype, copy=True)
    )
    weights = np.maximum(weights, dtype(1e-8))
    weights = (weights / weights.sum(axis=-1, keepdims=True)).astype(dtype)
    if cov_type == "spherical":
        cov = global_spherical_variance(x, k, reg_covar, dtype) if init_cov is None else np.array(init_cov, dtype=dtype)
        cov = np.maximum(cov, dtype(reg_covar))
    elif cov_type == "diag":
        cov = global_diag_variance(x, k, reg_covar, dtype) if init_cov is None else np.array(init_cov, dtype=dtype)
        cov = np.maximum(cov, dtype(reg_covar))
    elif cov_type == "tied":
        cov = global_tied_covariance(x, reg_covar, dtype) if init_cov is None else np.array(init_cov, dtype=dtype)
        cov = _sym(cov).astype(dtype)
    else:
        cov = global_full_covariance(x, k, reg_covar, dtype) if init_cov is None else np.array(init_cov, dtype=dtype)
        cov = _sym(cov).astype(dtype)
    return means, cov.astype(dtype), weights


# ---------------------------------------------------------------------------
# EM loops
# ---------------------------------------------------------------------------


def fit(
    cov_type: str,
    x,
    n_components: int,
    max_iters: int = 100,
    tol: float = 1e-4,
    init_means=None,
    init_variances=None,
    init_weights=None,
    *,
    reg_covar: float = 1e-6,
    chunk_size_N: int = 32768,
    chunk_size_K: int = 1024,
    min_weight: float = 1e-8,
    compute_labels: bool = True,
    dtype=np.float32,
    approx_top_k=None,
):
    """Soft EM, following the four reference loops:

    * spherical: torch_fallback.py:2060-2330 (torch path of
      batch_gmm_Spherical_torch_native), finalize 2293-2305;
    * diag: torch_fallback.py:2486-2696, finalize 2654-2666;
    * tied / full: torch_fallback.py:2864-3200 (_batch_gmm_matrix_torch_native),
      finalize 3141-3167.

    ``approx_top_k`` (1 <= top_k < K) runs the reference's approximate EM
    (_resolve_approx_top_k, torch_fallback.py:599-607; _topk_logits_for_chunk
    and _accumulate_topk_stats, 667-767): each row's responsibilities are the
    softmax of its top_k logits and zero elsewhere, and the log-likelihood sums
    the log-sum-exp of those top_k logits.  Equal logits rank the lower
    component index first.  top_k >= K is exact EM.

    Returns ``(labels, means, covariances, weights, info)`` like the reference.
    """
    if cov_type not in ("spherical", "diag", "tied", "full"):
        raise ValueError("covariance_type must be spherical, diag, tied or full")
    x = np.asarray(x, dtype=dtype)
    if x.ndim != 3:
        raise ValueError("x must have shape (B, N, D)")
    bsz, n, d = x.shape
    k = int(n_components)
    if k <= 0:
        raise ValueError("n_components must be positive")
    if n == 0:
        raise ValueError("x must contain at least one sample")
    if max_iters <= 0:
        raise ValueError("max_iters must be positive")
    top_k = None
    if approx_top_k is not None:
        top_k = int(approx_top_k)
        if top_k <= 0:
            raise ValueError("approx_top_k must be positive or None")
        if top_k >= k:
            top_k = None
    means, cov, weights = _init_params(cov_type, x, k, init_means, init_variances, init_weights, reg_covar, dtype)
    dt = dtype
    x_sq_all = np.square(x).sum(axis=-1).astype(dt)
    eye = np.eye(d, dtype=dt)
    total_xx = None
    if cov_type == "tied":
        # torch_fallback.py:2856-2862: X^T X once per fit
        total_xx = np.zeros((bsz, d, d), dtype=dt)
        for n0 in range(0, n, chunk_size_N):
            xc = x[:, n0:n0 + chunk_size_N]
            total_xx += np.swapaxes(xc, 1, 2) @ xc
    history = []
    prev_lb = None
    it = 0
    for it in range(max_iters):
        if cov_type in ("spherical", "diag"):
            cov = np.maximum(cov, dt(reg_covar))
        weights = np.maximum(weights, dt(min_weight))
        weights = (weights / weights.sum(axis=-1, keepdims=True)).astype(dt)
        model = _Model(cov_type, means, cov, weights, dt)
        nk = np.zeros((bsz, k), dtype=dt)
        sum_x = np.zeros((bsz, k, d), dtype=dt)
        if cov_type == "spherical":
            sum_sq = np.zeros((bsz, k), dtype=dt)
        elif cov_type == "diag":
            sum_sq = np.zeros((bsz, k, d), dtype=dt)
        elif cov_type == "full":
            sum_sq = np.zeros((bsz, k, d, d), dtype=dt)
        else:
            sum_sq = None
        total_ll = dt(0.0)
        for n0 in range(0, n, chunk_size_N):
            n1 = min(n0 + chunk_size_N, n)
            xc = x[:, n0:n1]
            xsq = x_sq_all[:, n0:n1]
            if top_k is not None:
                lg = model.logits(xc, xsq, 0, k)
                order = np.argsort(-lg, axis=-1, kind="stable")[..., :top_k]
                vals = np.take_along_axis(lg, order, axis=-1)
                lse = _logsumexp(vals)
                total_ll = dt(total_ll + lse.sum(dtype=dt))
                r = np.zeros_like(lg)
                np.put_along_axis(r, order, np.exp(vals - lse[..., None]).astype(dt), axis=-1)
                _accumulate(cov_type, r, xc, xsq, 0, k, nk, sum_x, sum_sq, dt)
                continue
            if cov_type == "spherical" or k > chunk_size_K:
                lse = stream_logsumexp(model, xc, xsq, chunk_size_K)
            else:
                lse = _logsumexp(model.logits(xc, xsq, 0, k))
            total_ll = dt(total_ll + lse.sum(dtype=dt))
            for k0 in range(0, k, chunk_size_K):
                k1 = min(k0 + chunk_size_K, k)
                r = np.exp(model.logits(xc, xsq, k0, k1) - lse[:, :, None]).astype(dt)
                _accumulate(cov_type, r, xc, xsq, k0, k1, nk, sum_x, sum_sq, dt)
        active = nk > dt(min_weight)
        nk_safe = np.maximum(nk, dt(min_weight))
        means_new = (sum_x / nk_safe[..., None]).astype(dt)
        means_new = np.where(active[..., None], means_new, means)
        if cov_type == "spherical":
            # torch_fallback.py:2298-2301
            msq = np.square(means_new).sum(axis=-1)
            v = np.maximum(sum_sq - nk * msq, dt(0.0)) / (nk_safe * dt(d))
            v = np.maximum(v, dt(reg_covar))
            cov_new = np.where(active, v, cov).astype(dt)
        elif cov_type == "diag":
            # torch_fallback.py:2659-2661
            second = sum_sq / nk_safe[..., None]
            v = np.maximum(second - np.square(means_new), dt(reg_covar))
            cov_new = np.where(active[..., None], v, cov).astype(dt)
        else:
            outer = means_new[..., :, None] * means_new[..., None, :]
            if cov_type == "full":
                # torch_fallback.py:3150-3158
                scatter = sum_sq - nk[..., None, None] * outer
                c = scatter / nk_safe[..., None, None]
                c = _sym(c) + dt(reg_covar) * eye
                cov_new = np.where(active[..., None, None], c, cov).astype(dt)
            else:
                # torch_fallback.py:3159-3162
                scatter = total_xx - (nk[..., None, None] * outer).sum(axis=1)
                c = scatter / dt(n)
                cov_new = (_sym(c) + dt(reg_covar) * eye).astype(dt)
        w = nk / dt(n)
        w = np.maximum(w, dt(min_weight))
        weights_new = (w / w.sum(axis=-1, keepdims=True)).astype(dt)
        lb = float(dt(total_ll / dt(bsz * n)))
        if cov_type != "spherical" and not (tol > 0.0 or it + 1 == max_iters):
            # torch_fallback.py:2487/2865 (collect_lower_bound): the diag /
            # tied / full loops record 0.0 for iterations whose bound is not
            # needed (tol == 0 and not the last iteration).
            lb = 0.0
        history.append(lb)
        means, cov, weights = means_new.astype(dt), cov_new, weights_new
        if tol > 0.0 and prev_lb is not None and it + 1 < max_iters and abs(lb - prev_lb) < tol:
            break
        if tol > 0.0:
            prev_lb = lb
    labels = assign(cov_type, x, means, cov, weights, chunk_size_N=chunk_size_N, chunk_size_K=chunk_size_K, dtype=dt) if compute_labels else None
    info: Dict[str, object] = {
        "n_iter": it + 1,
        "lower_bound": history[-1],
        "lower_bound_history": history,
        "init_source": "user",
        "approximate_em_enabled": top_k is not None,
        "approx_top_k": top_k,
    }
    return labels, means, cov, weights, info


def _accumulate(cov_type, r, xc, xsq, k0, k1, nk, sum_x, sum_sq, dt):
    """Sufficient statistics of responsibilities ``r`` (B, n, k1 - k0) for
    components k0..k1 (torch_fallback.py:2255-2291 and the per-type loops)."""
    nk[:, k0:k1] += r.sum(axis=1)
    sum_x[:, k0:k1] += np.swapaxes(r, 1, 2) @ xc
    if cov_type == "spherical":
        sum_sq[:, k0:k1] += (r * xsq[:, :, None]).sum(axis=1)
    elif cov_type == "diag":
        sum_sq[:, k0:k1] += np.swapaxes(r, 1, 2) @ np.square(xc)
    elif cov_type == "full":
        sum_sq[:, k0:k1] += np.einsum("bnk,bnd,bne->bkde", r, xc, xc, optimize=True).astype(dt)


def fit_spherical(x, n_components, max_iters=100, tol=1e-4, init_means=None, init_variances=None, init_weights=None, **kw):
    return fit("spherical", x, n_components, max_iters, tol, init_means, init_variances, init_weights, **kw)


def fit_diag(x, n_components, max_iters=100, tol=1e-4, init_means=None, init_variances=None, init_weights=None, **kw):
    return fit("diag", x, n_components, max_iters, tol, init_means, init_variances, init_weights, **kw)


def fit_tied(x, n_components, max_iters=100, tol=1e-4, init_means=None, init_variances=None, init_weights=None, **kw):
    return fit("tied", x, n_components, max_iters, tol, init_means, init_variances, init_weights, **kw)


def fit_full(x, n_components, max_iters=100, tol=1e-4, init_means=None, init_variances=None, init_weights=None, **kw):
    return fit("full", x, n_components, max_iters, tol, init_means, init_variances, init_weights, **kw)


# ---------------------------------------------------------------------------
# Inference
# ---------------------------------------------------------------------------


def assign(cov_type, x, means, cov, weights, *, chunk_size_N=32768, chunk_size_K=1024, dtype=np.float32):
    """torch_fallback.py:780-821 / 824-871 / 874-965 (*_assign_torch_native_chunked).

    Argmax over components; the first maximal component wins inside a chunk
    (torch ``max``) and a later chunk replaces the best only on a strictly
    larger logit.
    """
    x = np.asarray(x, dtype=dtype)
    model = _Model(cov_type, means, cov, weights, dtype)
    bsz, n, _ = x.shape
    k = model.means.shape[1]
    x_sq = np.square(x).sum(axis=-1).astype(dtype)
    labels = np.empty((bsz, n), dtype=np.int64)
    for n0 in range(0, n, chunk_size_N):
        n1 = min(n0 + chunk_size_N, n)
        best = np.full((bsz, n1 - n0), -np.inf, dtype=dtype)
        best_idx = np.zeros((bsz, n1 - n0), dtype=np.int64)
        for k0 in range(0, k, chunk_size_K):
            lg = model.logits(x[:, n0:n1], x_sq[:, n0:n1], k0, min(k0 + chunk_size_K, k))
            tl = lg.max(axis=-1)
            ti = lg.argmax(axis=-1)
            upd = tl > best
            best = np.where(upd, tl, best)
            best_idx = np.where(upd, ti + k0, best_idx)
        labels[:, n0:n1] = best_idx
    return labels


def score_samples(cov_type, x, means, cov, weights, *, chunk_size_N=32768, chunk_size_K=1024, dtype=np.float32):
    """torch_fallback.py:983-1130 (*_score_samples_torch_native_chunked)."""
    x = np.asarray(x, dtype=dtype)
    model = _Model(cov_type, means, cov, weights, dtype)
    bsz, n, _ = x.shape
    x_sq = np.square(x).sum(axis=-1).astype(dtype)
    out = np.empty((bsz, n), dtype=dtype)
    for n0 in range(0, n, chunk_size_N):
        n1 = min(n0 + chunk_size_N, n)
        out[:, n0:n1] = stream_logsumexp(model, x[:, n0:n1], x_sq[:, n0:n1], chunk_size_K)
    return out


def predict_proba(cov_type, x, means, cov, weights, *, chunk_size_N=32768, chunk_size_K=1024, dtype=np.float32):
    """torch_fallback.py:1133-1345 (*_predict_proba_torch_native_chunked):
    ``exp(logit - streaming_lse)``."""
    x = np.asarray(x, dtype=dtype)
    model = _Model(cov_type, means, cov, weights, dtype)
    bsz, n, _ = x.shape
    k = model.means.shape[1]
    x_sq = np.square(x).sum(axis=-1).astype(dtype)
    out = np.empty((bsz, n, k), dtype=dtype)
    for n0 in range(0, n, chunk_size_N):
        n1 = min(n0 + chunk_size_N, n)
        xc, xs = x[:, n0:n1], x_sq[:, n0:n1]
        lse = stream_logsumexp(model, xc, xs, chunk_size_K)
        for k0 in range(0, k, chunk_size_K):
            k1 = min(k0 + chunk_size_K, k)
            out[:, n0:n1, k0:k1] = np.exp(model.logits(xc, xs, k0, k1) - lse[:, :, None])
    return out


# ---------------------------------------------------------------------------
# k-means initialisation (init_params="kmeans")
# ---------------------------------------------------------------------------


def kmeans_pp_sample_size(n, n_components):
    """torch_fallback.py:1392-1398: rows of the k-means++ sample, or None
    where the reference declines (K > 256 or K > sample size)."""
    target = max(4096, 64 * n_components)
    sample_n = min(n, 65536, target)
    if n_components <= 0 or n_components > sample_n or n_components > 256:
        return None
    return sample_n


def kmeans_plus_plus(sample, n_components, first_idx, uniforms, dtype=np.float32):
    """torch_fallback.py:1390-1451 (_kmeans_plus_plus_init_means) with its
    random draws given: ``sample`` (B, S, D) is the row sample, ``first_idx``
    (B,) the first centres' rows, ``uniforms`` (K-1, B, L) the per-centre
    draws in [0, 1).  Candidate t of centre c is the first row whose running
    sum of closest squared distances reaches u * total (clamped to the last
    row, row 0 when the total is 0); the candidate of least potential (first
    on ties) is kept.  The running sums are accumulated in float64 and
    rounded to float32 per row, as torch's CPU cumsum of float32 does (its
    accumulator type is double); totals and potentials likewise."""
    s = np.asarray(sample, dtype)
    b, n, d = s.shape
    centers = np.empty((b, n_components, d), dtype)
    for bi in range(b):
        sf = s[bi]
        centers[bi, 0] = sf[first_idx[bi]]
        closest = np.square(sf - sf[first_idx[bi]]).sum(axis=-1, dtype=dtype)
        for c in range(1, n_components):
            total = np.asarray(closest.sum(dtype=np.float64), dtype)
            cum = np.cumsum(closest, dtype=np.float64).astype(dtype)
            cand = np.searchsorted(cum, np.asarray(uniforms[c - 1, bi], dtype) * total, side="left")
            cand = np.minimum(cand, n - 1)
            if not total > 0:
                cand[:] = 0
            new = np.square(sf[None, :, :] - sf[cand][:, None, :]).sum(axis=-1, dtype=dtype)
            trial = np.minimum(closest[None], new)
            best = int(np.argmin(trial.sum(axis=1, dtype=np.float64).astype(dtype)))
            centers[bi, c] = sf[cand[best]]
            closest = trial[best]
    return centers


def nearest_centroid(x, means, dtype=np.float32):
    """Index of each row's nearest centroid in the expanded-distance form of
    the spherical logits (torch_fallback.py:337-354 with unit variances and
    equal weights), first on ties."""
    xf = np.asarray(x, dtype)
    m = np.asarray(means, dtype)
    dist = np.square(xf).sum(-1, dtype=dtype)[..., None] - 2.0 * np.einsum("bnd,bkd->bnk", xf, m) + \
        np.square(m).sum(-1, dtype=dtype)[:, None, :]
    return np.argmin(np.maximum(dist, 0.0), axis=-1)


def lloyd(x, means, max_iters, tol, dtype=np.float32):
    """Lloyd's k-means (the algorithm of the reference's flash-kmeans step,
    torch_fallback.py:1585-1623): nearest-centroid labels, every centroid moved
    to the mean of its rows (an empty one stays), at most ``max_iters`` rounds,
    stopping once no centroid moves by more than ``tol``; returns (labels of
    the final centroids, centroids)."""
    xf = np.asarray(x, dtype)
    m = np.asarray(means, dtype).copy()
    b, n, d = xf.shape
    k = m.shape[1]
    for _ in range(max(0, int(max_iters))):
        lab = nearest_centroid(xf, m, dtype)
        new = m.copy()
        for bi in range(b):
            cnt = np.bincount(lab[bi], minlength=k).astype(dtype)
            sums = np.zeros((k, d), dtype)
            np.add.at(sums, lab[bi], xf[bi])
            live = cnt > 0
            new[bi, live] = sums[live] / cnt[live, None]
        shift = float(np.sqrt(np.square(new - m).sum(-1)).max())
        m = new
        if shift <= tol:
            break
    return nearest_centroid(xf, m, dtype), m


def hard_label_init(cov_type, x, means, labels, reg_covar, dtype=np.float32):
    """(weights, covariances) from hard labels: torch_fallback.py:1454-1481
    (spherical), 1483-1508 (diag), 1511-1543 (full), 1546-1569 (tied)."""
    xf = np.asarray(x, dtype)
    m = np.asarray(means, dtype)
    b, n, d = xf.shape
    k = m.shape[1]
    counts = np.zeros((b, k), dtype)
    for bi in range(b):
        counts[bi] = np.bincount(labels[bi], minlength=k)
    safe = np.maximum(counts, 1.0)
    weights = safe / safe.sum(-1, keepdims=True)
    diffs = xf - np.take_along_axis(m, labels[..., None], axis=1)
    eye = np.eye(d, dtype=dtype)
    if cov_type in ("spherical", "diag"):
        sq = np.zeros((b, k, d), dtype)
        for bi in range(b):
            np.add.at(sq[bi], labels[bi], np.square(diffs[bi]))
        if cov_type == "spherical":
            var = sq.sum(-1) / safe / float(d)
            gv = global_spherical_variance(xf, k, reg_covar, dtype)
            cov = np.where(counts > 0, var, gv)
        else:
            var = sq / safe[..., None]
            gv = global_diag_variance(xf, k, reg_covar, dtype)
            cov = np.where(counts[..., None] > 0, var, gv)
        return weights, np.maximum(cov, reg_covar).astype(dtype)
    if cov_type == "tied":
        cov = np.einsum("bnd,bne->bde", diffs, diffs) / float(n) + reg_covar * eye
        return weights, _sym(cov).astype(dtype)
    onehot = np.zeros((b, n, k), dtype)
    for bi in range(b):
        onehot[bi, np.arange(n), labels[bi]] = 1.0
    sum_x = np.einsum("bnk,bnd->bkd", onehot, xf)
    sum_xx = np.einsum("bnk,bnd,bne->bkde", onehot, xf, xf)
    mc, mr = m[..., :, None], m[..., None, :]
    scatter = sum_xx - mc * sum_x[..., None, :] - sum_x[..., :, None] * mr + counts[..., None, None] * (mc * mr)
    cov = scatter / safe[..., None, None] + reg_covar * eye
    cov = np.where(counts[..., None, None] > 0, cov, global_full_covariance(xf, k, reg_covar, dtype))
    return weights, _sym(cov).astype(dtype)
