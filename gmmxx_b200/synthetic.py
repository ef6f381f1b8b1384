"""Seeded synthetic mixtures with the benchmark configurations' distributions.

No public dataset backs the reference's benchmark; the configurations name
their generating distributions, which these generators reproduce (rows are
generated on the device in chunks, bf16 rounding after generation):

  0  spherical fp32  N=100k  D=32  K=64   mu~U(-10,10), sigma~U(0.5,2), Dir(1)
  1  diag      bf16  N=50M   D=64  K=512  mu~N(0,25 I), var_d~LogU(0.1,4), Dir(0.5)
  2  tied      fp32  N=20M   D=64  K=256  Sigma=A A^T/D+0.1 I, mu~N(0,16 I), uniform
  3  full      fp32  B=64 x N=262144, D=16, K=32  Sigma_k~Wishart(D+2, I), mu~U(-5,5), Dir(1)
  4  spherical bf16  N=200M  D=128 K=8192 mu~N(0,4 I), sigma~U(0.3,1.5), Zipf(1.1)
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch


@dataclass(frozen=True)
class Config:
    index: int
    cov_type: str
    dtype: torch.dtype
    B: int
    N: int
    D: int
    K: int
    iters: int


CONFIGS = {
    0: Config(0, "spherical", torch.float32, 1, 100_000, 32, 64, 20),
    1: Config(1, "diag", torch.bfloat16, 1, 50_000_000, 64, 512, 10),
    2: Config(2, "tied", torch.float32, 1, 20_000_000, 64, 256, 10),
    3: Config(3, "full", torch.float32, 64, 262_144, 16, 32, 15),
    4: Config(4, "spherical", torch.bfloat16, 1, 200_000_000, 128, 8192, 5),
}


@dataclass
class Mixture:
    means: np.ndarray      # (B, K, D)
    cov: np.ndarray        # per-type covariance parameters (B, ...)
    weights: np.ndarray    # (B, K)


def mixture_params(cfg: Config, seed: int = 0) -> Mixture:
    """The generating mixture (host, float64 -> float32)."""
    rng = np.random.default_rng(seed)
    B, D, K = cfg.B, cfg.D, cfg.K
    if cfg.index == 0:
        means = rng.uniform(-10, 10, (B, K, D))
        cov = rng.uniform(0.5, 2.0, (B, K)) ** 2
        w = rng.dirichlet(np.ones(K), size=B)
    elif cfg.index == 1:
        means = rng.normal(0, 5.0, (B, K, D))
        cov = np.exp(rng.uniform(np.log(0.1), np.log(4.0), (B, K, D)))
        w = rng.dirichlet(np.full(K, 0.5), size=B)
    elif cfg.index == 2:
        a = rng.normal(0, 1, (B, D, D))
        cov = a @ np.swapaxes(a, 1, 2) / D + 0.1 * np.eye(D)
        means = rng.normal(0, 4.0, (B, K, D))
        w = np.full((B, K), 1.0 / K)
    elif cfg.index == 3:
        g = rng.normal(0, 1, (B, K, D + 2, D))
        cov = np.swapaxes(g, 2, 3) @ g  # Wishart(D+2, I)
        means = rng.uniform(-5, 5, (B, K, D))
        w = rng.dirichlet(np.ones(K), size=B)
    else:
        means = rng.normal(0, 2.0, (B, K, D))
        cov = rng.uniform(0.3, 1.5, (B, K)) ** 2
        z = 1.0 / np.arange(1, K + 1) ** 1.1
        w = np.repeat((z / z.sum())[None], B, 0)
        rng.shuffle(w.T)  # spread the heavy components over the index range
    w = w / w.sum(-1, keepdims=True)
    return Mixture(means.astype(np.float32), cov.astype(np.float32), w.astype(np.float32))


def sample_rows(cfg: Config, mix: Mixture, n: int, device: torch.device, seed: int,
                out: Optional[torch.Tensor] = None, chunk: int = 1 << 22) -> torch.Tensor:
    """Draw n rows per problem on `device` into out (B, n, D) of cfg.dtype."""
    B, D, K = cfg.B, cfg.D, cfg.K
    if out is None:
        out = torch.empty((B, n, D), dtype=cfg.dtype, device=device)
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    means = torch.from_numpy(mix.means).to(device)
    cdf = torch.from_numpy(np.cumsum(mix.weights, -1)).to(device)
    cdf[:, -1] = 1.0
    if cfg.cov_type in ("spherical", "diag"):
        scale = torch.from_numpy(np.sqrt(mix.cov)).to(device)
    else:
        chol = torch.linalg.cholesky(torch.from_numpy(mix.cov).to(device=device, dtype=torch.float64)).float()
    for b in range(B):
        for n0 in range(0, n, chunk):
            m = min(chunk, n - n0)
            u = torch.rand((m,), generator=g, device=device)
            z = torch.searchsorted(cdf[b], u).clamp_max(K - 1)
            eps = torch.randn((m, D), generator=g, device=device)
            if cfg.cov_type == "spherical":
                xb = means[b, z] + scale[b, z, None] * eps
            elif cfg.cov_type == "diag":
                xb = means[b, z] + scale[b, z] * eps
            elif cfg.cov_type == "tied":
                xb = means[b, z] + eps @ chol[b].T
            else:
                xb = means[b, z] + torch.einsum("nde,ne->nd", chol[b, z], eps)
            out[b, n0:n0 + m] = xb.to(cfg.dtype)
    return out


def initial_params(cfg: Config, mix: Mixture, seed: int = 1):
    """Identical seeded initial parameters for every implementation / rank:
    the generating means perturbed by N(0, 0.25) noise, unit (co)variances,
    uniform weights (host float32 arrays)."""
    rng = np.random.default_rng(seed)
    B, D, K = cfg.B, cfg.D, cfg.K
    means = (mix.means + 0.5 * rng.standard_normal(mix.means.shape)).astype(np.float32)
    if cfg.cov_type == "spherical":
        cov = np.ones((B, K), np.float32)
    elif cfg.cov_type == "diag":
        cov = np.ones((B, K, D), np.float32)
    elif cfg.cov_type == "tied":
        cov = np.repeat(np.eye(D, dtype=np.float32)[None], B, 0)
    else:
        cov = np.tile(np.eye(D, dtype=np.float32), (B, K, 1, 1))
    w = np.full((B, K), 1.0 / K, np.float32)
    return means, cov, w
