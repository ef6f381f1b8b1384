"""Functional API with the reference's signatures, served by the CUDA engine.

``batch_gmm_{Spherical,Diagonal,Tied,Full}`` keep the argument names, order,
defaults and return value ``(labels, means, covariances, weights, info)`` of
the reference (gmmxx/torch_fallback.py:3339-3513).  Arguments that only steer
the reference's Triton / chunking heuristics (``chunk_size_N``,
``chunk_size_K``, ``kmeans_*``, ``use_triton``) are accepted and validated but
do not change the result: the engine streams rows and components itself.
``approx_top_k`` in [1, K - 1] runs approximate top-k EM (each row's
responsibilities restricted to its top_k components, as the reference's
torch_fallback.py:667-767); None or >= K is exact EM.

Half-precision ``x`` (bf16 / fp16) is read as stored and every parameter and
logit is computed and returned in fp32: the estimator's upcast semantics
(interface.py:426-433), exact because the conversion to fp32 is exact.  The
reference's torch functions instead keep the parameters in ``x.dtype``
between iterations (torch_fallback.py:2295, 2656-2666, 3145-3167) and, for
spherical, form the cross term ``x @ means^T`` in ``x.dtype``
(torch_fallback.py:348); those roundings are not reproduced.

Inference functions mirror the reference's ``*_torch_native_chunked``
functions (torch_fallback.py:780-1345) without the torch-specific suffix.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import engine


def _validate(x, n_components, max_iters, chunk_size_N, chunk_size_K, min_weight, approx_top_k):
    if not torch.is_tensor(x) or x.ndim != 3:
        raise ValueError("x must have shape (B, N, D)")
    if n_components <= 0:
        raise ValueError("n_components must be positive")
    if x.shape[1] == 0:
        raise ValueError("x must contain at least one sample")
    if max_iters <= 0:
        raise ValueError("max_iters must be positive")
    if chunk_size_N <= 0 or chunk_size_K <= 0:
        raise ValueError("chunk_size_N and chunk_size_K must be positive")
    if min_weight <= 0.0:
        raise ValueError("min_weight must be positive")
    if approx_top_k is not None and int(approx_top_k) <= 0:
        raise ValueError("approx_top_k must be positive or None")


def _fit(cov_type, x, n_components, max_iters, tol, init_means, init_variances, init_weights, verbose,
         init_params, reg_covar, chunk_size_N, chunk_size_K, min_weight, compute_labels, approx_top_k,
         kmeans=(10, 1e-4)):
    _validate(x, n_components, max_iters, chunk_size_N, chunk_size_K, min_weight, approx_top_k)
    return engine.em_fit(
        cov_type, x, n_components, max_iters=max_iters, tol=tol, init_means=init_means,
        init_variances=init_variances, init_weights=init_weights, init_params=init_params,
        reg_covar=reg_covar, min_weight=min_weight, compute_labels=compute_labels, verbose=verbose,
        approx_top_k=approx_top_k, kmeans_init_iters=int(kmeans[0]), kmeans_init_tol=float(kmeans[1]))


def batch_gmm_Spherical(
    x: torch.Tensor,
    n_components: int,
    max_iters: int = 100,
    tol: float = 1e-4,
    init_means: Optional[torch.Tensor] = None,
    init_variances: Optional[torch.Tensor] = None,
    init_weights: Optional[torch.Tensor] = None,
    verbose: bool = False,
    *,
    init_params: str = "kmeans",
    reg_covar: float = 1e-6,
    chunk_size_N: int = 32768,
    chunk_size_K: int = 1024,
    kmeans_init_iters: int = 10,
    kmeans_init_tol: float = 1e-4,
    use_triton: bool = True,
    min_weight: float = 1e-8,
    compute_labels: bool = True,
    approx_top_k: Optional[int] = None,
):
    """Spherical soft EM (reference: torch_fallback.py:3339-3380, loop 1897-2397)."""
    return _fit("spherical", x, n_components, max_iters, tol, init_means, init_variances, init_weights, verbose,
                init_params, reg_covar, chunk_size_N, chunk_size_K, min_weight, compute_labels, approx_top_k,
                (kmeans_init_iters, kmeans_init_tol))


def batch_gmm_Diagonal(
    x: torch.Tensor,
    n_components: int,
    max_iters: int = 100,
    tol: float = 1e-4,
    init_means: Optional[torch.Tensor] = None,
    init_variances: Optional[torch.Tensor] = None,
    init_weights: Optional[torch.Tensor] = None,
    verbose: bool = False,
    *,
    init_params: str = "kmeans",
    reg_covar: float = 1e-6,
    chunk_size_N: int = 32768,
    chunk_size_K: int = 1024,
    kmeans_init_iters: int = 10,
    kmeans_init_tol: float = 1e-4,
    use_triton: bool = True,
    min_weight: float = 1e-8,
    compute_labels: bool = True,
    approx_top_k: Optional[int] = None,
):
    """Diagonal soft EM (reference: torch_fallback.py:3383-3424, loop 2401-2728)."""
    return _fit("diag", x, n_components, max_iters, tol, init_means, init_variances, init_weights, verbose,
                init_params, reg_covar, chunk_size_N, chunk_size_K, min_weight, compute_labels, approx_top_k,
                (kmeans_init_iters, kmeans_init_tol))


def batch_gmm_Full(
    x: torch.Tensor,
    n_components: int,
    max_iters: int = 100,
    tol: float = 1e-4,
    init_means: Optional[torch.Tensor] = None,
    init_variances: Optional[torch.Tensor] = None,
    init_weights: Optional[torch.Tensor] = None,
    verbose: bool = False,
    *,
    init_params: str = "kmeans",
    reg_covar: float = 1e-6,
    chunk_size_N: int = 32768,
    chunk_size_K: int = 1024,
    kmeans_init_iters: int = 10,
    kmeans_init_tol: float = 1e-4,
    use_triton: bool = True,
    min_weight: float = 1e-8,
    compute_labels: bool = True,
    approx_top_k: Optional[int] = None,
):
    """Full-covariance soft EM (reference: torch_fallback.py:3427-3468, loop 2732-3244)."""
    return _fit("full", x, n_components, max_iters, tol, init_means, init_variances, init_weights, verbose,
                init_params, reg_covar, chunk_size_N, chunk_size_K, min_weight, compute_labels, approx_top_k,
                (kmeans_init_iters, kmeans_init_tol))


def batch_gmm_Tied(
    x: torch.Tensor,
    n_components: int,
    max_iters: int = 100,
    tol: float = 1e-4,
    init_means: Optional[torch.Tensor] = None,
    init_variances: Optional[torch.Tensor] = None,
    init_weights: Optional[torch.Tensor] = None,
    verbose: bool = False,
    *,
    init_params: str = "kmeans",
    reg_covar: float = 1e-6,
    chunk_size_N: int = 32768,
    chunk_size_K: int = 1024,
    kmeans_init_iters: int = 10,
    kmeans_init_tol: float = 1e-4,
    use_triton: bool = True,
    min_weight: float = 1e-8,
    compute_labels: bool = True,
    approx_top_k: Optional[int] = None,
):
    """Tied-covariance soft EM (reference: torch_fallback.py:3471-3512, loop 2732-3244)."""
    return _fit("tied", x, n_components, max_iters, tol, init_means, init_variances, init_weights, verbose,
                init_params, reg_covar, chunk_size_N, chunk_size_K, min_weight, compute_labels, approx_top_k,
                (kmeans_init_iters, kmeans_init_tol))


batch_gmm_spherical = batch_gmm_Spherical
batch_gmm_diagonal = batch_gmm_Diagonal
batch_gmm_diag = batch_gmm_Diagonal
batch_gmm_full = batch_gmm_Full
batch_gmm_tied = batch_gmm_Tied


# --- the reference's *_torch_native names (torch_fallback.py:1897-3336) -------
# Same parameters as the reference's loops; the Triton and k-means switches
# steer only the reference's own kernels and are validated, not needed.  They
# run on this engine (CUDA tensors), not on torch.


def _check_switch(name, value):
    if not isinstance(value, bool) and value != "auto":
        raise ValueError(f"{name} must be a bool or 'auto'")


def batch_gmm_Spherical_torch_native(
    x: torch.Tensor,
    n_components: int,
    max_iters: int = 100,
    tol: float = 1e-4,
    init_means: Optional[torch.Tensor] = None,
    init_variances: Optional[torch.Tensor] = None,
    init_weights: Optional[torch.Tensor] = None,
    verbose: bool = False,
    *,
    init_params: str = "kmeans",
    reg_covar: float = 1e-6,
    chunk_size_N: int = 32768,
    chunk_size_K: int = 1024,
    kmeans_init_iters: int = 10,
    kmeans_init_tol: float = 1e-4,
    kmeans_use_triton: bool = True,
    gmm_use_triton_estep="auto",
    gmm_use_triton_streaming_update="auto",
    min_weight: float = 1e-8,
    compute_labels: bool = True,
    approx_top_k: Optional[int] = None,
):
    """Spherical soft EM with the reference loop's parameters
    (torch_fallback.py:1897-2397)."""
    _check_switch("gmm_use_triton_estep", gmm_use_triton_estep)
    _check_switch("gmm_use_triton_streaming_update", gmm_use_triton_streaming_update)
    return _fit("spherical", x, n_components, max_iters, tol, init_means, init_variances, init_weights, verbose,
                init_params, reg_covar, chunk_size_N, chunk_size_K, min_weight, compute_labels, approx_top_k,
                (kmeans_init_iters, kmeans_init_tol))


def _matrix_native(cov_type, doc):
    def fit(
        x: torch.Tensor,
        n_components: int,
        max_iters: int = 100,
        tol: float = 1e-4,
        init_means: Optional[torch.Tensor] = None,
        init_variances: Optional[torch.Tensor] = None,
        init_weights: Optional[torch.Tensor] = None,
        verbose: bool = False,
        *,
        init_params: str = "kmeans",
        reg_covar: float = 1e-6,
        chunk_size_N: int = 32768,
        chunk_size_K: int = 1024,
        kmeans_init_iters: int = 10,
        kmeans_init_tol: float = 1e-4,
        kmeans_use_triton: bool = True,
        gmm_use_triton="auto",
        min_weight: float = 1e-8,
        compute_labels: bool = True,
        approx_top_k: Optional[int] = None,
    ):
        _check_switch("gmm_use_triton", gmm_use_triton)
        return _fit(cov_type, x, n_components, max_iters, tol, init_means, init_variances, init_weights, verbose,
                    init_params, reg_covar, chunk_size_N, chunk_size_K, min_weight, compute_labels, approx_top_k,
                (kmeans_init_iters, kmeans_init_tol))

    fit.__doc__ = doc
    return fit


batch_gmm_Diagonal_torch_native = _matrix_native(
    "diag", "Diagonal soft EM with the reference loop's parameters (torch_fallback.py:2401-2728).")
batch_gmm_Diagonal_torch_native.__name__ = "batch_gmm_Diagonal_torch_native"
batch_gmm_Full_torch_native = _matrix_native(
    "full", "Full-covariance soft EM with the reference loop's parameters (torch_fallback.py:3247-3290).")
batch_gmm_Full_torch_native.__name__ = "batch_gmm_Full_torch_native"
batch_gmm_Tied_torch_native = _matrix_native(
    "tied", "Tied-covariance soft EM with the reference loop's parameters (torch_fallback.py:3293-3336).")
batch_gmm_Tied_torch_native.__name__ = "batch_gmm_Tied_torch_native"


# --- inference (torch_fallback.py:780-1345) ----------------------------------


def _inf(fn, cov_type):
    """The inference call with the reference's parameter names: ``variances``
    (spherical, diag), ``covariance`` (tied), ``covariances`` (full)."""
    def call(x, means, params, weights, chunk_size_N, chunk_size_K):
        if chunk_size_N <= 0 or chunk_size_K <= 0:
            raise ValueError("chunk_size_N and chunk_size_K must be positive")
        return fn(cov_type, x, means, params, weights)

    if cov_type in ("spherical", "diag"):
        def run(x, means, variances, weights, *, chunk_size_N: int = 32768, chunk_size_K: int = 1024):
            return call(x, means, variances, weights, chunk_size_N, chunk_size_K)
    elif cov_type == "tied":
        def run(x, means, covariance, weights, *, chunk_size_N: int = 32768, chunk_size_K: int = 1024):
            return call(x, means, covariance, weights, chunk_size_N, chunk_size_K)
    else:
        def run(x, means, covariances, weights, *, chunk_size_N: int = 32768, chunk_size_K: int = 1024):
            return call(x, means, covariances, weights, chunk_size_N, chunk_size_K)

    run.__name__ = f"{cov_type}_{fn.__name__}"
    run.__doc__ = f"{fn.__doc__} ({cov_type} covariance)"
    return run


spherical_assign = _inf(engine.assign, "spherical")
spherical_score_samples = _inf(engine.score_samples, "spherical")
spherical_predict_proba = _inf(engine.predict_proba, "spherical")
diagonal_assign = _inf(engine.assign, "diag")
diagonal_score_samples = _inf(engine.score_samples, "diag")
diagonal_predict_proba = _inf(engine.predict_proba, "diag")
tied_assign = _inf(engine.assign, "tied")
tied_score_samples = _inf(engine.score_samples, "tied")
tied_predict_proba = _inf(engine.predict_proba, "tied")
full_assign = _inf(engine.assign, "full")
full_score_samples = _inf(engine.score_samples, "full")
full_predict_proba = _inf(engine.predict_proba, "full")


# the reference's inference names (torch_fallback.py:780-1345)
spherical_assign_torch_native_chunked = spherical_assign
spherical_score_samples_torch_native_chunked = spherical_score_samples
spherical_predict_proba_torch_native_chunked = spherical_predict_proba
diagonal_assign_torch_native_chunked = diagonal_assign
diagonal_score_samples_torch_native_chunked = diagonal_score_samples
diagonal_predict_proba_torch_native_chunked = diagonal_predict_proba
tied_assign_torch_native_chunked = tied_assign
tied_score_samples_torch_native_chunked = tied_score_samples
tied_predict_proba_torch_native_chunked = tied_predict_proba
full_assign_torch_native_chunked = full_assign
full_score_samples_torch_native_chunked = full_score_samples
full_predict_proba_torch_native_chunked = full_predict_proba
