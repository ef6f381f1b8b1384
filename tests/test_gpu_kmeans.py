"""k-means initialisation on the GPU (init_params="kmeans").

* k-means++ seeds (gmmxx_kmeans_pp) after torch.manual_seed(seed) equal the
  centroids the reference's own _kmeans_plus_plus_init_means picked on the CPU
  (tests/golden/init_kmeanspp_*.npz, make_kmeans_golden.py) -- exactly, since
  centroids are data rows; and None where the reference declines.
* Lloyd iterations and the hard-label initial parameters equal the oracle's
  (oracle.lloyd, oracle.hard_label_init) from the same seeds, for every
  covariance type.
* The per-label sums of gmmxx_label_stats equal numpy's for every mode and
  x dtype.
* The estimator and the large-N entry point report the k-means source."""

import numpy as np
import pytest
import torch

import oracle
from conftest import golden_cases, kmeans_pp_reference_draws, load_golden

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", golden_cases("init_kmeanspp_"))
def test_kmeans_pp_matches_reference_golden(cuda_device, case):
    from gmmxx_b200 import kmeans

    g = load_golden(case)
    x = torch.from_numpy(g["x"]).to(cuda_device)
    torch.manual_seed(int(g["seed"]))
    got = kmeans.kmeans_plus_plus_init_means(x, int(g["k"]))
    np.testing.assert_array_equal(got.cpu().numpy(), g["centers"])


def test_kmeans_pp_declines_like_the_reference(cuda_device):
    from gmmxx_b200 import kmeans

    x = torch.randn(1, 20_000, 3, device=cuda_device)
    assert kmeans.kmeans_plus_plus_init_means(x, 257) is None     # K above 256
    assert kmeans.kmeans_plus_plus_init_means(x[:, :100], 120) is None  # K above the sample
    assert kmeans.kmeans_plus_plus_init_means(x, 3).shape == (1, 3, 3)


def _blobs(seed, b, n, d, k):
    rng = np.random.default_rng(seed)
    mu = rng.uniform(-8, 8, (b, k, d))
    z = rng.integers(0, k, (b, n))
    x = np.take_along_axis(mu, z[..., None], 1) + rng.uniform(0.4, 1.2, (b, k))[np.arange(b)[:, None], z][..., None] \
        * rng.standard_normal((b, n, d))
    return x.astype(np.float32)


@pytest.mark.parametrize("cov", ["spherical", "diag", "tied", "full"])
def test_kmeans_init_matches_oracle(cuda_device, cov):
    from gmmxx_b200 import kmeans

    x = _blobs(3, 2, 5000, 5, 7)
    seed = 21
    torch.manual_seed(seed)
    means, c, w = kmeans.kmeans_initialize(cov, torch.from_numpy(x).to(cuda_device), 7, max_iters=6, tol=1e-4,
                                           reg_covar=1e-6)
    sample, first, u = kmeans_pp_reference_draws(torch.from_numpy(x), 7, seed)
    seeds = oracle.kmeans_plus_plus(sample.numpy(), 7, first.numpy(), u.numpy())
    lab, m = oracle.lloyd(x, seeds, 6, 1e-4)
    w_o, c_o = oracle.hard_label_init(cov, x, m, lab, 1e-6)
    np.testing.assert_allclose(means.cpu().numpy(), m, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(w.cpu().numpy(), w_o, rtol=1e-6)
    np.testing.assert_allclose(c.cpu().numpy(), c_o, rtol=1e-4, atol=1e-4)  # fp32 cancellation in the scatter


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_label_stats_match_numpy(cuda_device, mode, dtype):
    from gmmxx_b200 import kmeans

    rng = np.random.default_rng(mode)
    b, n, d, k = 2, 9000, 6, 11
    xt = torch.from_numpy(rng.standard_normal((b, n, d)).astype(np.float32)).to(dtype)
    x = xt.float().numpy().astype(np.float64)
    lab = rng.integers(0, k, (b, n))
    lab[:, :3] = 0  # label k-1 may stay empty
    lab[lab == k - 1] = 1
    mu = rng.standard_normal((b, k, d)).astype(np.float32)
    got = kmeans.label_stats(xt.to(cuda_device), torch.from_numpy(lab).to(cuda_device), k, mode,
                             torch.from_numpy(mu).to(cuda_device)).cpu().numpy()
    for bi in range(b):
        for l in range(k):
            rows = x[bi, lab[bi] == l]
            want = [np.array([len(rows)], np.float64), rows.sum(0)]
            if mode == 1:
                want.append(np.square(rows - mu[bi, l]).sum(0))
            elif mode == 2:
                iu = np.triu_indices(d)
                want.append((rows.T @ rows)[iu])
            np.testing.assert_allclose(got[bi, l], np.concatenate(want), rtol=2e-5, atol=2e-4)


def test_estimator_and_large_n_report_the_kmeans_source(cuda_device):
    import gmmxx_b200 as G

    x = torch.from_numpy(_blobs(5, 1, 8000, 4, 6)[0])
    g = G.GMMXX(k=6, niter=3, covariance_type="diag", init_params="kmeans", seed=3, backend="cuda").fit(
        x.to(cuda_device))
    assert g.init_source_ == "kmeans"
    g = G.GMMXX(k=300, niter=1, covariance_type="diag", init_params="kmeans", seed=3, backend="cuda").fit(
        x.to(cuda_device))
    assert g.init_source_ == "random"  # the reference's k-means++ declines K > 256
    out = G.batch_gmm_largeN_cpu(x[None], 6, covariance_type="spherical", device=cuda_device, dtype=torch.float32,
                                 max_iters=2, tol=0.0, chunk_size_N=3000, seed=1, init_params="kmeans")
    assert out[4]["init_source"] == "kmeans_sampled"  # a 4096-row sample of the 8000 rows
