"""Operator-level API with the reference's names: ``gmmxx.cuda_ops``
(gmmxx/cuda_ops.py:1-87), the wrappers of ``gmmxx._cuda``
(gmmxx/_cuda.py:46-1416).

Same function names, argument order and meaning, return shapes and dtypes,
and the same input checks (``ValueError`` for a tensor that is not on a CUDA
device or has the wrong dtype, ``CudaBackendUnavailable`` when the native
library is missing), so code written against the reference's operators runs
unchanged.  The work runs on this engine's kernels through its C ABI:

* E-step operators (``*_assign``, ``*_logsumexp``, ``*_resp``) call
  ``gmmxx_assign`` / ``gmmxx_logsumexp`` / ``gmmxx_resp`` with the weights
  ``exp(log_w)``; tied and full take the reference's Cholesky factors ``L``
  and pass ``L L^T`` (the engine re-factors it).  Labels come back int32 as in
  the reference.
* ``soft_update_spherical``, ``fused_spherical`` and
  ``approx_topk_update_spherical`` accumulate their statistics with
  ``gmmxx_em_accumulate`` / ``gmmxx_em_accumulate_topk`` and apply the
  reference operator's own finalize rules to them (those rules differ from
  the EM loops': see each function).
* ``tied_project``, ``tied_log_det``, ``tied_finalize`` and ``full_finalize``
  are small (K x D x D) tensor algebra in the reference too and are the same
  algebra here (triangular solves and Cholesky through torch.linalg).

The reference's hard-assignment operators (``blocked_update_*``,
``finalize_spherical``, ``finalize_diag``, ``full_blocked_update``) serve its
hard-EM path, which this engine does not implement; they raise
``NotImplementedError``.  Nothing falls back: ``CudaRuntimeFallback`` exists
so that ``except`` clauses written for the reference still import, but no
operator raises it -- a failing call raises ``GmmxxError``.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _native as nat
from . import engine

CudaBackendUnavailable = nat.CudaBackendUnavailable


class CudaRuntimeFallback(RuntimeError):
    """The reference raises this to fall back to another backend
    (gmmxx/_cuda.py:40-43).  This engine never falls back and never raises it."""


def has_cuda() -> bool:
    """True when the native library loads and a CUDA device is visible
    (gmmxx/_cuda.py:46-48)."""
    return nat.available() and torch.cuda.is_available()


def require_cuda() -> None:
    """Raise CudaBackendUnavailable when the native library is missing
    (gmmxx/_cuda.py:57-64)."""
    nat.load()


def _check_input(t: torch.Tensor, name: str, *, dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """The reference's argument check (gmmxx/_cuda.py:67-74): CUDA device,
    contiguous (copied when not), optional exact dtype."""
    if not t.is_cuda:
        raise ValueError(f"{name}: must be on a CUDA device, got {t.device}")
    if not t.is_contiguous():
        t = t.contiguous()
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name}: dtype must be {dtype}, got {t.dtype}")
    return t


def _into(result: torch.Tensor, out: Optional[torch.Tensor]) -> torch.Tensor:
    if out is None:
        return result
    out.copy_(result)
    return out


def _weights(log_w: torch.Tensor) -> torch.Tensor:
    return log_w.to(torch.float32).exp()


def _cov_from_factor(L: torch.Tensor) -> torch.Tensor:
    lf = L.to(torch.float32)
    return lf @ lf.transpose(-1, -2)


def canary_add_offset(input: torch.Tensor, offset: int) -> torch.Tensor:  # noqa: A002 (reference name)
    """input + offset through the smoke kernel (gmmxx/_cuda.py:77-97)."""
    require_cuda()
    input = _check_input(input, "canary input", dtype=torch.int32)  # noqa: A001
    return engine.canary_add_offset(input, offset)


# ---------------------------------------------------------------------------
# spherical (gmmxx/_cuda.py:328-412, 415-682, 783-889, 1056-1088)
# ---------------------------------------------------------------------------


def _e_args(x, means, var, log_w):
    require_cuda()
    x = _check_input(x, "x")
    means = _check_input(means, "means")
    var = _check_input(var, "var", dtype=torch.float32)
    log_w = _check_input(log_w, "log_w", dtype=torch.float32)
    return x, means, var, log_w


def spherical_assign(x, means, var, log_w, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Labels (B, N) int32: argmax of the logits, the first maximal component."""
    x, means, var, log_w = _e_args(x, means, var, log_w)
    return _into(engine.assign("spherical", x, means, var, _weights(log_w)).to(torch.int32), out)


def spherical_logsumexp(x, means, var, log_w, out: Optional[torch.Tensor] = None,
                        x_sq: Optional[torch.Tensor] = None, c_sq: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-row log-sum-exp of the logits, (B, N) fp32.  ``x_sq`` / ``c_sq``
    (precomputed |x|^2, |mu|^2 in the reference) are accepted and not needed."""
    del x_sq, c_sq
    x, means, var, log_w = _e_args(x, means, var, log_w)
    return _into(engine.score_samples("spherical", x, means, var, _weights(log_w)), out)


def spherical_resp(x, means, var, log_w, log_norm, out: Optional[torch.Tensor] = None,
                   x_sq: Optional[torch.Tensor] = None, c_sq: Optional[torch.Tensor] = None) -> torch.Tensor:
    """exp(logit - log_norm), (B, N, K) fp32."""
    del x_sq, c_sq
    x, means, var, log_w = _e_args(x, means, var, log_w)
    log_norm = _check_input(log_norm, "log_norm", dtype=torch.float32)
    return _into(engine.resp("spherical", x, means, var, _weights(log_w), log_norm), out)


def _spherical_stats(x, means, var, log_w, top_k: Optional[int] = None):
    """(n_k, sum r x, sum r |x|^2, sum of the rows' log-sum-exp) for the
    parameters as given: the engine's per-iteration prologue runs on copies
    with a negligible weight floor (the weights it renormalises are corrected
    for in the log-likelihood).  The variances are floored at 1e-30 only for
    approximate top-k EM (the reference's clamp in
    approx_topk_update_spherical, _cuda.py:829-830); the exact operators take
    log(var) unclamped as the reference's do (_cuda.py:581), apart from a
    floor at 0 for negative variances."""
    b, n, d = x.shape
    k = means.shape[1]
    ops = engine.CudaOps("spherical", x, k, top_k)
    m = means.to(torch.float32).clone()
    v = var.clone()
    w = _weights(log_w).clone()
    with torch.cuda.device(x.device):
        ops.prepare(m, v, w, 1e-30 if top_k is not None else 0.0, 1e-30)
        stats = torch.zeros((b, k, ops.stat_width), dtype=torch.float32, device=x.device)
        ll = torch.zeros((1,), dtype=torch.float64, device=x.device)
        ops.accumulate(stats, ll)
    ll = ll[0] + float(n) * torch.logsumexp(log_w.to(torch.float64), dim=-1).sum()
    return stats[..., 0], stats[..., 1:1 + d], stats[..., 1 + d], ll


def soft_update_spherical(
    x: torch.Tensor,
    means: torch.Tensor,
    var: torch.Tensor,
    log_w: torch.Tensor,
    reg_covar: float,
    x_f_cached: Optional[torch.Tensor] = None,
    x_sq_cached: Optional[torch.Tensor] = None,
    x_aug_cached: Optional[torch.Tensor] = None,
    x_estep_aug_cached: Optional[torch.Tensor] = None,
    x_estep_aug_bf16_cached: Optional[torch.Tensor] = None,
    x_aug_bf16_cached: Optional[torch.Tensor] = None,
    persistent_partial_buf: Optional[torch.Tensor] = None,
    compute_ids: bool = True,
    compute_lse: bool = True,
):
    """One exact spherical soft-EM update; returns (means, var, weights,
    lse_per_sample or None, labels int32 or None).  The cache arguments of the
    reference are accepted and not needed.  Finalize rules of the reference
    operator (its fp32 finalize kernel, csrc/mstep/finalize_spherical.cu:
    129-176): n_safe = max(n_k, 1e-8), mu = sum_x / n_safe,
    var = max((sum_x2 - n_k |mu|^2) / (n_safe D), reg_covar),
    weights = max(n_k / N, 1e-8) (not renormalised, no empty-cluster keep);
    means are cast to x's dtype."""
    del x_f_cached, x_sq_cached, x_aug_cached, x_estep_aug_cached, x_estep_aug_bf16_cached
    del x_aug_bf16_cached, persistent_partial_buf
    x, means, var, log_w = _e_args(x, means, var, log_w)
    b, n, d = x.shape
    nk, sx, sxx, _ = _spherical_stats(x, means, var, log_w)
    n_safe = nk.clamp_min(1e-8)
    mu = sx / n_safe.unsqueeze(-1)
    v = ((sxx - nk * mu.square().sum(-1)) / (n_safe * float(d))).clamp_min(float(reg_covar))
    w = (nk / float(n)).clamp_min(1e-8)
    if x.dtype != torch.float32:
        mu = mu.to(x.dtype)
    lse = spherical_logsumexp(x, means, var, log_w) if compute_lse else None
    ids = spherical_assign(x, means, var, log_w) if compute_ids else None
    return mu, v, w, lse, ids


def fused_spherical(x, means, var, log_w, reg_covar: float):
    """One spherical soft-EM step with the reference's fused-kernel rules
    (csrc/fused/spherical_fused.cu:189-229, 239-350): returns (new_means in
    means' dtype, new_var fp32 >= reg_covar, new_weights = n_k / N fp32,
    lse_per_sample (B, N) fp32, labels (B, N) int32); a component with
    n_k <= 0 keeps its mean and variance and gets weight 0.  The reference
    kernel's window (D <= 64, K <= 128, means in x's dtype) is enforced."""
    x, means, var, log_w = _e_args(x, means, var, log_w)
    if x.ndim != 3:
        raise ValueError("fused_safe: x must be (B, N, D)")
    if means.dtype != x.dtype:
        raise ValueError("fused_safe: means must be contiguous CUDA, same dtype as x")
    b, n, d = x.shape
    k = means.shape[1]
    if d > 64:
        raise ValueError(f"fused_safe requires D <= 64; got {d}")
    if k > 128:
        raise ValueError(f"fused_safe requires K <= 128; got {k}")
    if n == 0:
        return (means.clone(), var.clone(), torch.zeros_like(var), torch.zeros((b, 0), device=x.device),
                torch.empty((b, 0), dtype=torch.int32, device=x.device))
    nk, sx, sxx, _ = _spherical_stats(x, means, var, log_w)
    live = nk > 0.0
    n_inv = 1.0 / torch.where(live, nk, torch.ones_like(nk))
    mu = sx * n_inv.unsqueeze(-1)
    v = ((sxx * n_inv - mu.square().sum(-1)) / float(d)).clamp_min(float(reg_covar))
    new_means = torch.where(live.unsqueeze(-1), mu, means.to(torch.float32)).to(means.dtype)
    new_var = torch.where(live, v, var)
    new_w = torch.where(live, nk / float(n), torch.zeros_like(nk))
    lse = spherical_logsumexp(x, means, var, log_w)
    labels = spherical_assign(x, means, var, log_w)
    return new_means, new_var, new_w, lse, labels


def approx_topk_update_spherical(x, means, var, log_w, *, top_k: int, chunk_size_K: int = 64):
    """Approximate spherical soft-EM statistics over each row's top_k
    components (gmmxx/_cuda.py:783-889): returns (n_k (B, K), sum r x
    (B, K, D), sum r |x|^2 (B, K), sum of the rows' top_k log-sum-exp as a
    0-dim fp32 tensor).  ``chunk_size_K`` only steers the reference's
    streaming and is validated, not needed."""
    x, means, var, log_w = _e_args(x, means, var, log_w)
    if x.ndim != 3:
        raise ValueError("x must have shape (B, N, D)")
    if means.ndim != 3:
        raise ValueError("means must have shape (B, K, D)")
    b, n, d = x.shape
    bm, k, dm = means.shape
    if (bm, dm) != (b, d):
        raise ValueError("means shape mismatch")
    if var.shape != (b, k):
        raise ValueError("var shape mismatch")
    if log_w.shape != (b, k):
        raise ValueError("log_w shape mismatch")
    top_k = int(top_k)
    if top_k <= 0 or top_k >= k:
        raise ValueError("top_k must be in [1, K - 1]")
    if int(chunk_size_K) <= 0:
        raise ValueError("chunk_size_K must be positive")
    if top_k > engine.MAX_APPROX_TOP_K:
        raise nat.UnsupportedShape(nat.ERR_UNSUPPORTED,
                                   f"top_k={top_k} exceeds the engine window (<= {engine.MAX_APPROX_TOP_K})")
    nk, sx, sxx, ll = _spherical_stats(x, means, var, log_w, top_k)
    return nk.contiguous(), sx.contiguous(), sxx.contiguous(), ll.to(torch.float32)


# ---------------------------------------------------------------------------
# diagonal (gmmxx/_cuda.py:897-959)
# ---------------------------------------------------------------------------


def diag_assign(x, means, var, log_w, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Labels (B, N) int32; ``var`` (B, K, D)."""
    x, means, var, log_w = _e_args(x, means, var, log_w)
    return _into(engine.assign("diag", x, means, var, _weights(log_w)).to(torch.int32), out)


def diag_logsumexp(x, means, var, log_w, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-row log-sum-exp, (B, N) fp32."""
    x, means, var, log_w = _e_args(x, means, var, log_w)
    return _into(engine.score_samples("diag", x, means, var, _weights(log_w)), out)


def diag_resp(x, means, var, log_w, log_norm, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """exp(logit - log_norm), (B, N, K) fp32."""
    x, means, var, log_w = _e_args(x, means, var, log_w)
    log_norm = _check_input(log_norm, "log_norm", dtype=torch.float32)
    return _into(engine.resp("diag", x, means, var, _weights(log_w), log_norm), out)


# ---------------------------------------------------------------------------
# tied: the reference's projected-coordinate operators (gmmxx/_cuda.py:1100-1243)
# ---------------------------------------------------------------------------


def tied_project(x: torch.Tensor, L: torch.Tensor) -> torch.Tensor:
    """y = L^-1 x row by row for lower-triangular L (B, D, D); x (B, N, D)."""
    require_cuda()
    x = _check_input(x, "x")
    L = _check_input(L, "L")
    rhs = x.transpose(-1, -2).to(L.dtype)
    return torch.linalg.solve_triangular(L, rhs, upper=False).transpose(-1, -2).contiguous()


def tied_log_det(L: torch.Tensor) -> torch.Tensor:
    """log|L| = sum_d log |L_dd|, (B,)."""
    return torch.diagonal(L, dim1=-2, dim2=-1).abs().log().sum(-1)


def _tied_args(x, means, L, log_w):
    require_cuda()
    x = _check_input(x, "x")
    means = _check_input(means, "means")
    log_w = _check_input(log_w, "log_w", dtype=torch.float32)
    return x, means, _cov_from_factor(L), log_w


def tied_assign(x, means, L, log_w) -> torch.Tensor:
    """Labels (B, N) int32 for the shared covariance L L^T."""
    x, means, cov, log_w = _tied_args(x, means, L, log_w)
    return engine.assign("tied", x, means, cov, _weights(log_w)).to(torch.int32)


def tied_logsumexp(x, means, L, log_w) -> torch.Tensor:
    """The tied log-likelihood per row, (B, N) fp32."""
    x, means, cov, log_w = _tied_args(x, means, L, log_w)
    return engine.score_samples("tied", x, means, cov, _weights(log_w))


def tied_resp(x, means, L, log_w, log_norm) -> torch.Tensor:
    """exp(tied logit - log_norm), (B, N, K) fp32; ``log_norm`` as returned by
    tied_logsumexp."""
    x, means, cov, log_w = _tied_args(x, means, L, log_w)
    log_norm = _check_input(log_norm, "log_norm", dtype=torch.float32)
    return engine.resp("tied", x, means, cov, _weights(log_w), log_norm)


def tied_finalize(sums, xx_total, counts, total_n: int, reg_covar: float):
    """(means (B, K, D), Cholesky factor of the new shared covariance
    (B, D, D), weights (B, K)) from the statistics, the reference operator's
    rules: mu = sums / max(n_k, 1e-30), weights = n_k / N (not renormalised),
    Sigma = sym((X^T X - sum_k n_k mu mu^T) / N + reg I).  ``counts`` may be
    int32 (hard) or fp32 (soft)."""
    require_cuda()
    sums = _check_input(sums, "sums", dtype=torch.float32)
    xx_total = _check_input(xx_total, "xx_total", dtype=torch.float32)
    counts = _check_input(counts, "counts")
    d = sums.shape[-1]
    n_k = counts.to(torch.float32)
    mu = sums / n_k.clamp_min(1e-30).unsqueeze(-1)
    weights = n_k / float(total_n)
    scatter = (mu * n_k.unsqueeze(-1)).transpose(-1, -2) @ mu
    sigma = (xx_total - scatter) / float(total_n) + float(reg_covar) * torch.eye(d, device=sums.device)
    sigma = 0.5 * (sigma + sigma.transpose(-1, -2))
    return mu, torch.linalg.cholesky(sigma), weights


# ---------------------------------------------------------------------------
# full (gmmxx/_cuda.py:1246-1416)
# ---------------------------------------------------------------------------


def _full_args(x, means, L, log_w):
    require_cuda()
    x = _check_input(x, "x")
    means = _check_input(means, "means")
    L = _check_input(L, "L")
    log_w = _check_input(log_w, "log_w", dtype=torch.float32)
    return x, means, _cov_from_factor(L), log_w


def full_assign(x, means, L, log_w) -> torch.Tensor:
    """Labels (B, N) int32; ``L`` (B, K, D, D) per-component Cholesky factors."""
    x, means, cov, log_w = _full_args(x, means, L, log_w)
    return engine.assign("full", x, means, cov, _weights(log_w)).to(torch.int32)


def full_logsumexp(x, means, L, log_w) -> torch.Tensor:
    """Per-row log-sum-exp, (B, N) fp32."""
    x, means, cov, log_w = _full_args(x, means, L, log_w)
    return engine.score_samples("full", x, means, cov, _weights(log_w))


def full_resp(x, means, L, log_w, log_norm) -> torch.Tensor:
    """exp(logit - log_norm), (B, N, K) fp32."""
    x, means, cov, log_w = _full_args(x, means, L, log_w)
    log_norm = _check_input(log_norm, "log_norm", dtype=torch.float32)
    return engine.resp("full", x, means, cov, _weights(log_w), log_norm)


def full_finalize(sums, outer_sums, counts, old_means, old_L, total_n: int, reg_covar: float):
    """(means (B, K, D), Cholesky factors (B, K, D, D), weights (B, K)), the
    reference operator's rules: mu = sums / max(n_k, 1e-30),
    Sigma = sym(outer / n_k - mu mu^T + reg I); a component whose count is
    <= 0 or whose Sigma has no Cholesky factor keeps its old mean and factor
    and gets weight 0; outputs are cast to the dtypes of old_means / old_L."""
    require_cuda()
    sums = _check_input(sums, "sums", dtype=torch.float32)
    outer_sums = _check_input(outer_sums, "outer_sums", dtype=torch.float32)
    counts = _check_input(counts, "counts")
    old_means = _check_input(old_means, "old_means")
    old_L = _check_input(old_L, "old_L")
    d = sums.shape[-1]
    n_k = counts.to(torch.float32)
    n_safe = n_k.clamp_min(1e-30)
    mu = sums / n_safe.unsqueeze(-1)
    weights = n_k / float(total_n)
    sigma = outer_sums / n_safe[..., None, None] - mu.unsqueeze(-1) * mu.unsqueeze(-2)
    sigma = sigma + float(reg_covar) * torch.eye(d, device=sums.device)
    sigma = 0.5 * (sigma + sigma.transpose(-1, -2))
    factor, info = torch.linalg.cholesky_ex(sigma)
    failed = (info != 0) | (n_k <= 0.0)
    mu = torch.where(failed.unsqueeze(-1), old_means.to(torch.float32), mu)
    factor = torch.where(failed[..., None, None], old_L.to(torch.float32), factor)
    weights = torch.where(failed, torch.zeros_like(weights), weights)
    return mu.to(old_means.dtype), factor.to(old_L.dtype), weights


# ---------------------------------------------------------------------------
# hard-assignment operators of the reference's hard-EM path (not provided)
# ---------------------------------------------------------------------------


def _hard_em(name: str):
    def op(*args, **kwargs):
        raise NotImplementedError(
            f"{name}: hard-assignment EM operators are not part of the gmmxx_b200 engine (it runs soft EM); "
            "use soft_update_spherical / fused_spherical or the batch_gmm_* API")

    op.__name__ = name
    op.__doc__ = f"The reference's hard-EM operator {name}; not provided (raises NotImplementedError)."
    return op


blocked_update_spherical = _hard_em("blocked_update_spherical")
blocked_update_spherical_sorted = _hard_em("blocked_update_spherical_sorted")
finalize_spherical = _hard_em("finalize_spherical")
blocked_update_diag = _hard_em("blocked_update_diag")
blocked_update_diag_sorted = _hard_em("blocked_update_diag_sorted")
finalize_diag = _hard_em("finalize_diag")
full_blocked_update = _hard_em("full_blocked_update")


__all__ = [
    "canary_add_offset",
    "spherical_assign",
    "spherical_logsumexp",
    "spherical_resp",
    "soft_update_spherical",
    "blocked_update_spherical",
    "blocked_update_spherical_sorted",
    "finalize_spherical",
    "fused_spherical",
    "approx_topk_update_spherical",
    "diag_assign",
    "diag_logsumexp",
    "diag_resp",
    "blocked_update_diag",
    "blocked_update_diag_sorted",
    "finalize_diag",
    "tied_project",
    "tied_log_det",
    "tied_assign",
    "tied_logsumexp",
    "tied_resp",
    "tied_finalize",
    "full_assign",
    "full_logsumexp",
    "full_resp",
    "full_blocked_update",
    "full_finalize",
    "has_cuda",
    "require_cuda",
    "CudaBackendUnavailable",
    "CudaRuntimeFallback",
]
