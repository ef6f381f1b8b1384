"""k-means initialisation of a fit (``init_params="kmeans"``) on the GPU.

The reference's k-means initialisation (gmmxx/torch_fallback.py:1571-1623,
``_kmeans_initialize``) seeds centroids with greedy k-means++
(``_kmeans_plus_plus_init_means``, 1390-1451), refines them with Lloyd
iterations from its optional dependency flash-kmeans (``flash-kmeans>=0.2``,
``pyproject.toml`` extra "kmeans"; not vendored with the reference), and
derives the initial weights and covariances from the resulting hard labels
(``_hard_label_init_stats*``, 1454-1569).  Without flash-kmeans the reference
falls back to random rows (1580-1582, 1706).

Here every step runs on the device:

* k-means++ -- ``gmmxx_kmeans_pp`` (csrc/kmeans.cu).  The random numbers are
  drawn from torch's CPU generator in the reference's order (the row sample's
  ``randperm``, the first centre's ``randint``, then ``L`` uniforms per further
  centre), so a seeded call picks the same rows as the reference's CPU run.
  Same sample size, trial count (2 + floor(log K)), inverse-CDF candidate rule
  and smallest-potential choice; ``None`` where the reference returns None
  (K > 256 or K > sample size).
* Lloyd -- the published algorithm flash-kmeans implements: assign every
  row to its nearest centroid (first on ties; the engine's spherical
  ``gmmxx_assign`` with unit variances and equal weights is exactly that
  argmin), move each centroid to the mean of its rows (``gmmxx_label_stats``,
  an empty centroid stays), stop after ``max_iters`` or once no centroid moves
  by more than ``tol``.
* hard-label statistics -- the reference's four ``_hard_label_init_stats*``
  formulas over ``gmmxx_label_stats`` sums (and X^T X for tied).
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import _native as nat
from . import engine

# the reference's k-means++ limits (torch_fallback.py:65-69)
KMEANS_PLUS_PLUS_MAX_COMPONENTS = 256
KMEANS_PLUS_PLUS_MAX_SAMPLES = 65536
KMEANS_PLUS_PLUS_MIN_SAMPLES = 4096
KMEANS_PLUS_PLUS_SAMPLES_PER_COMPONENT = 64


def kmeans_plus_plus_init_means(x: torch.Tensor, n_components: int,
                                generator: Optional[torch.Generator] = None) -> Optional[torch.Tensor]:
    """Greedy k-means++ centroids (B, K, D) in x's dtype, or None where the
    reference's ``_kmeans_plus_plus_init_means`` returns None.  ``x`` (B, N, D)
    on a CUDA device; the random draws come from ``generator`` (torch's default
    CPU generator when None) exactly as the reference draws them on the CPU."""
    x = engine.check_x(x)
    b, n, d = x.shape
    k = int(n_components)
    target = max(KMEANS_PLUS_PLUS_MIN_SAMPLES, KMEANS_PLUS_PLUS_SAMPLES_PER_COMPONENT * k)
    sample_n = min(n, KMEANS_PLUS_PLUS_MAX_SAMPLES, target)
    if k <= 0 or k > sample_n or k > KMEANS_PLUS_PLUS_MAX_COMPONENTS:
        return None
    g = generator if generator is not None else torch.default_generator
    if sample_n == n:
        sample = x
    else:
        idx = torch.randperm(n, generator=g)[:sample_n]
        sample = x.index_select(1, idx.to(x.device))
    sample_f = sample.to(torch.float32).contiguous()
    first = torch.randint(0, sample_n, (b,), generator=g)
    trials = 2 + int(math.log(float(k)))
    draws = [torch.rand((b, trials), generator=g, dtype=torch.float32) for _ in range(k - 1)]
    dev = x.device
    u = (torch.stack(draws) if draws else torch.zeros((1, b, trials))).to(dev).contiguous()
    first = first.to(dev)
    centers = torch.empty((b, k, d), dtype=torch.float32, device=dev)
    ws = torch.empty(max(1, nat.kmeans_pp_workspace_bytes(b, sample_n, trials)), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        nat.call("gmmxx_kmeans_pp", sample_f.data_ptr(), b, sample_n, d, k, trials, first.data_ptr(), u.data_ptr(),
                 centers.data_ptr(), ws.data_ptr(), ws.numel(), engine._stream_ptr(dev))
    return centers.to(x.dtype)


def label_stats(x: torch.Tensor, labels: torch.Tensor, k: int, mode: int,
                means: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-label sums (B, K, F) over the rows of x (gmmxx_label_stats):
    mode 0 [count, sum x], 1 [count, sum x, sum (x - mu_label)^2],
    2 [count, sum x, sum x_i x_j (i <= j)]."""
    b, n, d = x.shape
    dev = x.device
    f = nat.label_stats_width(mode, d)
    out = torch.empty((b, k, f), dtype=torch.float32, device=dev)
    ws = torch.empty(max(256, nat.label_stats_workspace_bytes(mode, b, n, d, k)), dtype=torch.uint8, device=dev)
    m = means.to(device=dev, dtype=torch.float32).contiguous() if means is not None else None
    with torch.cuda.device(dev):
        nat.call("gmmxx_label_stats", engine._X_DTYPES[x.dtype], x.data_ptr(), b, n, d, k,
                 labels.to(device=dev, dtype=torch.int64).contiguous().data_ptr(), engine._p(m), mode, out.data_ptr(),
                 ws.data_ptr(), ws.numel(), engine._stream_ptr(dev))
    return out


def nearest(x: torch.Tensor, means: torch.Tensor) -> torch.Tensor:
    """Index of each row's nearest centroid (first on ties): the spherical
    argmax with unit variances and equal weights."""
    b, k = means.shape[0], means.shape[1]
    ones = torch.ones((b, k), dtype=torch.float32, device=x.device)
    return engine.assign("spherical", x, means, ones, ones / float(k))


def lloyd(x: torch.Tensor, means: torch.Tensor, max_iters: int, tol: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """Lloyd iterations from ``means``: returns (labels of the final means,
    final means fp32).  An empty centroid keeps its position; the loop stops
    early once no centroid moves by more than ``tol``."""
    k, d = means.shape[1], means.shape[2]
    means = means.to(torch.float32).contiguous()
    for _ in range(max(0, int(max_iters))):
        st = label_stats(x, nearest(x, means), k, 0)
        cnt = st[..., :1]
        new = torch.where(cnt > 0, st[..., 1:1 + d] / cnt.clamp_min(1.0), means)
        shift = float((new - means).norm(dim=-1).max())
        means = new.contiguous()
        if shift <= tol:
            break
    return nearest(x, means), means


def hard_label_init(cov_type: str, x: torch.Tensor, means: torch.Tensor, labels: torch.Tensor,
                    reg_covar: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """(weights, covariances) from hard labels: the reference's
    _hard_label_init_stats (spherical), _diag, _full and _tied
    (torch_fallback.py:1454-1569), over device-side label sums."""
    b, n, d = x.shape
    k = means.shape[1]
    mu = means.to(torch.float32)
    mode = {"spherical": 1, "diag": 1, "full": 2, "tied": 0}[cov_type]
    st = label_stats(x, labels, k, mode, mu)
    counts = st[..., 0]
    sum_x = st[..., 1:1 + d]
    counts_safe = counts.clamp_min(1.0)
    weights = counts_safe / counts_safe.sum(dim=-1, keepdim=True)
    eye = torch.eye(d, device=x.device, dtype=torch.float32)
    if cov_type in ("spherical", "diag"):
        sq = st[..., 1 + d:]
        gv = engine.global_covariance(cov_type, x, k, reg_covar)
        if cov_type == "spherical":
            var = sq.sum(dim=-1) / counts_safe / float(d)
            cov = torch.where(counts > 0, var, gv)
        else:
            var = sq / counts_safe.unsqueeze(-1)
            cov = torch.where(counts.unsqueeze(-1) > 0, var, gv)
        return weights, cov.clamp_min(reg_covar)
    if cov_type == "tied":
        xx = torch.zeros((b, d, d), dtype=torch.float32, device=x.device)
        ws = engine._WS.get(x.device, nat.workspace_bytes(nat.TIED, b, n, d, 1))
        with torch.cuda.device(x.device):
            nat.call("gmmxx_xx_total", engine._X_DTYPES[x.dtype], x.data_ptr(), b, n, d, xx.data_ptr(), ws.data_ptr(),
                     ws.numel(), engine._stream_ptr(x.device))
        cross = torch.einsum("bkd,bke->bde", sum_x, mu)
        scatter = xx - cross - cross.transpose(1, 2) + torch.einsum("bk,bkd,bke->bde", counts, mu, mu)
        cov = scatter / float(n) + reg_covar * eye
        return weights, engine._sym(cov)
    # full: unpack sum x_i x_j (i <= j)
    iu = torch.triu_indices(d, d, device=x.device)
    sxx = torch.zeros((b, k, d, d), dtype=torch.float32, device=x.device)
    sxx[..., iu[0], iu[1]] = st[..., 1 + d:]
    sxx[..., iu[1], iu[0]] = st[..., 1 + d:]
    mc, mr = mu.unsqueeze(-1), mu.unsqueeze(-2)
    scatter = sxx - mc * sum_x.unsqueeze(-2) - sum_x.unsqueeze(-1) * mr + counts[..., None, None] * (mc * mr)
    cov = scatter / counts_safe[..., None, None] + reg_covar * eye
    gc = engine.global_covariance("full", x, k, reg_covar)
    cov = torch.where(counts[..., None, None] > 0, cov, gc)
    return weights, engine._sym(cov)


def kmeans_initialize(cov_type: str, x: torch.Tensor, k: int, *, max_iters: int, tol: float, reg_covar: float,
                      generator: Optional[torch.Generator] = None):
    """(means fp32, covariances, weights) of init_params="kmeans", or None
    where the reference's k-means++ returns None (the caller then draws random
    rows, as the reference does)."""
    seeds = kmeans_plus_plus_init_means(x, k, generator)
    if seeds is None:
        return None
    labels, means = lloyd(x, seeds, max_iters, tol)
    weights, cov = hard_label_init(cov_type, x, means, labels, reg_covar)
    return means, cov.contiguous(), weights.contiguous()
