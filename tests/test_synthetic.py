"""The synthetic stand-ins for the benchmark configurations (no public
dataset backs them): shapes, dtypes and generating distributions as
BASELINE.json's configs name them, seeded and reproducible."""

import numpy as np
import pytest
import torch

from gmmxx_b200 import synthetic

# (covariance type, x dtype, B, N, D, K, EM iterations) of configs[0..4]
EXPECTED = {
    0: ("spherical", torch.float32, 1, 100_000, 32, 64, 20),
    1: ("diag", torch.bfloat16, 1, 50_000_000, 64, 512, 10),
    2: ("tied", torch.float32, 1, 20_000_000, 64, 256, 10),
    3: ("full", torch.float32, 64, 262_144, 16, 32, 15),
    4: ("spherical", torch.bfloat16, 1, 200_000_000, 128, 8192, 5),
}


@pytest.mark.parametrize("index", sorted(EXPECTED))
def test_config_shapes(index):
    c = synthetic.CONFIGS[index]
    assert (c.cov_type, c.dtype, c.B, c.N, c.D, c.K, c.iters) == EXPECTED[index]


@pytest.mark.parametrize("index", sorted(EXPECTED))
def test_mixture_distributions(index):
    cfg = synthetic.CONFIGS[index]
    m = synthetic.mixture_params(cfg)
    B, K, D = cfg.B, cfg.K, cfg.D
    assert m.means.shape == (B, K, D) and m.weights.shape == (B, K)
    np.testing.assert_allclose(m.weights.sum(-1), 1.0, rtol=1e-5)
    assert (m.weights > 0).all()
    if index == 0:
        assert np.abs(m.means).max() <= 10 and 0.25 <= m.cov.min() and m.cov.max() <= 4.0
    elif index == 1:
        assert m.cov.shape == (B, K, D) and 0.1 <= m.cov.min() and m.cov.max() <= 4.0
        assert abs(m.means.std() - 5.0) < 0.2
    elif index == 2:
        assert m.cov.shape == (B, D, D)
        assert np.linalg.eigvalsh(m.cov).min() >= 0.1 - 1e-4  # A A^T / D + 0.1 I
        np.testing.assert_allclose(m.weights, 1.0 / K)
    elif index == 3:
        assert m.cov.shape == (B, K, D, D)
        assert np.linalg.eigvalsh(m.cov).min() > 0  # Wishart(D + 2, I) is positive definite
        assert np.abs(m.means).max() <= 5
    else:
        assert 0.09 <= m.cov.min() and m.cov.max() <= 2.25
        ranks = np.sort(m.weights[0])[::-1]
        np.testing.assert_allclose(ranks[0] / ranks[1], 2.0 ** 1.1, rtol=1e-4)  # Zipf(1.1)


@pytest.mark.parametrize("index", [0, 1, 2, 3])
def test_sampled_rows_are_seeded(index):
    cfg = synthetic.CONFIGS[index]
    mix = synthetic.mixture_params(cfg)
    a = synthetic.sample_rows(cfg, mix, 1000, torch.device("cpu"), seed=5, chunk=300)
    b = synthetic.sample_rows(cfg, mix, 1000, torch.device("cpu"), seed=5, chunk=300)
    c = synthetic.sample_rows(cfg, mix, 1000, torch.device("cpu"), seed=6, chunk=300)
    assert a.shape == (cfg.B, 1000, cfg.D) and a.dtype == cfg.dtype
    assert torch.equal(a, b) and not torch.equal(a, c)
    assert torch.isfinite(a.float()).all()


def test_initial_parameters_are_shared_and_seeded():
    cfg = synthetic.CONFIGS[1]
    mix = synthetic.mixture_params(cfg)
    m1, c1, w1 = synthetic.initial_params(cfg, mix)
    m2, c2, w2 = synthetic.initial_params(cfg, mix)
    assert np.array_equal(m1, m2) and np.array_equal(c1, c2) and np.array_equal(w1, w2)
    assert c1.shape == (1, 512, 64) and (c1 == 1).all() and np.allclose(w1, 1 / 512)
    assert abs((m1 - mix.means).std() - 0.5) < 0.01  # the generating means perturbed by N(0, 0.5^2)


def test_bench_launch_count_matches_the_kernel_sequence(monkeypatch):
    """bench.py's gpu_launches claim per EM iteration: prep (2, +2 Cholesky
    kernels for tied / full), the statistics kernels, finalize (2).  Config
    4 (spherical D = 128, K = 8192) on the diag-kernel layout: pack, 32
    row-statistics launches (groups of 2 chunks), combine, log-likelihood
    sum, 16 x (second pass + reduce); on em_tc_kernel (the legacy layout)
    the first pass has 16 groups of 4 chunks."""
    import bench

    monkeypatch.delenv("GMMXX_B200_SPH_KERNEL", raising=False)
    cfg = synthetic.CONFIGS
    assert bench.launches_per_iteration(cfg[4], True) == 2 + (1 + 32 + 2 + 2 * 16) + 2
    assert bench.launches_per_iteration(cfg[1], True) == 2 + 3 + 2
    assert bench.launches_per_iteration(cfg[2], True) == 4 + 3 + 2
    assert bench.launches_per_iteration(cfg[3], False) == 4 + 2 + 2
    assert bench.launches_per_iteration(cfg[0], False) == 2 + 2 + 2
    monkeypatch.setenv("GMMXX_B200_SPH_KERNEL", "legacy")
    assert bench.launches_per_iteration(cfg[4], True) == 2 + (1 + 16 + 2 + 2 * 16) + 2
