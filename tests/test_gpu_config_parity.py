"""GPU parity on the shapes the benchmark runs, against the numpy oracle
(float32 and float64 runs of the reference's algorithm from the same initial
parameters), plus the estimator and the large-N entry point through the calls
a user makes.

* configs[1..4] at their own D, K (and B = 64 for config 3), with the
  configuration's generating distribution, on a row cut the oracle finishes in
  seconds: diag bf16 K = 512 (tensor cores), tied fp32 K = 256 (the route
  config 2 takes), full fp32 B = 64 D = 16 K = 32, spherical bf16 D = 128
  K = 8192 with Zipf(1.1) weights, whose smallest components hold well under
  one row (the inactive-component keep rule, torch_fallback.py:2293-2301);
* ``GMMXX.train(init_means=...)`` for every covariance type, unbatched and
  batched, fp32 and bf16 input (upcast semantics, interface.py:426-433), and a
  host input larger than ``chunk_size_data_cpu`` (the streamed route);
* ``batch_gmm_largeN_cpu`` from its documented seeded initialisation.

Tolerances: parameters within 1e-4 relative / 1e-4
absolute of the float32 oracle, or no further from the float64 answer than
that plus twice the float32 oracle's own error; mean log-likelihood within
1e-4 relative (fp32 X) or 1e-3 (bf16 X); labels >= 99.9 % identical."""

import dataclasses

import numpy as np
import pytest
import torch

import oracle
from test_gpu_parity import _init_cov, _mixture, assert_bound_parity, assert_parity

pytestmark = pytest.mark.gpu

CPU = torch.device("cpu")


def _config_case(index, n, seed=77):
    from gmmxx_b200 import synthetic

    cfg = dataclasses.replace(synthetic.CONFIGS[index], N=n)
    mix = synthetic.mixture_params(cfg)
    means, cov, w = synthetic.initial_params(cfg, mix)
    x = synthetic.sample_rows(cfg, mix, n, CPU, seed=seed)
    return cfg, x, means, cov, w


def _check(got, ref32, ref64, lb_rtol, labels_min=0.999, ref32_alt=None):
    labels, means, cov, w, info = got
    alt = (lambda i: None) if ref32_alt is None else (lambda i: ref32_alt[i])
    assert_parity(means.cpu().numpy(), ref32[1], ref64[1], name="means", ref32_alt=alt(1))
    assert_parity(cov.cpu().numpy(), ref32[2], ref64[2], name="covariances", ref32_alt=alt(2))
    assert_parity(w.cpu().numpy(), ref32[3], ref64[3], name="weights", ref32_alt=alt(3))
    assert_bound_parity(info["lower_bound"], ref32[4]["lower_bound"], ref64[4]["lower_bound"], lb_rtol,
                        None if ref32_alt is None else ref32_alt[4]["lower_bound"])
    if labels is not None:
        assert (labels.cpu().numpy() == ref32[0]).mean() >= labels_min


@pytest.mark.parametrize("index,n,iters,path", [
    (1, 131_072, 2, "tensor-core"),    # diag bf16, D=64, K=512
    (2, 200_000, 3, "tensor-core"),    # tied fp32, D=64, K=256
    (3, 4_096, 3, "cuda-core"),        # full fp32, B=64, D=16, K=32
    (4, 65_536, 2, "tensor-core"),     # spherical bf16, D=128, K=8192, Zipf(1.1)
])
def test_config_shape_matches_oracle(cuda_device, index, n, iters, path):
    """Config 3's Wishart(D + 2, I) components overlap heavily, so its EM
    amplifies rounding; a second fp32 oracle run with another row chunking
    measures how far the reference's own fp32 answer moves with summation
    order."""
    from gmmxx_b200 import engine

    cfg, x, m, c, w = _config_case(index, n)
    xf = x.float().numpy()
    ref32 = oracle.fit(cfg.cov_type, xf, cfg.K, iters, 0.0, m, c, w)
    ref64 = oracle.fit(cfg.cov_type, xf, cfg.K, iters, 0.0, m, c, w, dtype=np.float64)
    alt = oracle.fit(cfg.cov_type, xf, cfg.K, iters, 0.0, m, c, w, chunk_size_N=1000) if index == 3 else None
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)
    got = engine.em_fit(cfg.cov_type, x.to(cuda_device), cfg.K, max_iters=iters, tol=0.0, init_means=t(m),
                        init_variances=t(c), init_weights=t(w))
    if path is not None:
        assert got[4]["kernel_path"] == path
    _check(got, ref32, ref64, 1e-4 if cfg.dtype == torch.float32 else 1e-3, ref32_alt=alt)
    if index == 4:  # the case exercises components that end up (nearly) empty
        assert float(got[3].min()) < 1.0 / n


@pytest.mark.parametrize("cov", ["spherical", "diag", "tied", "full"])
def test_estimator_train_matches_oracle(cuda_device, cov):
    """GMMXX.train with injected initial parameters: unbatched (N, D) data with
    unbatched init tensors, then bf16 data of the same values (upcast)."""
    from gmmxx_b200 import GMMXX

    d, k = (8, 6) if cov != "full" else (5, 4)
    x, init = _mixture(31 + d, 1, 5000, d, k)
    icov = _init_cov(cov, x, k)
    w = np.full((1, k), 1.0 / k, np.float32)
    ref32 = oracle.fit(cov, x, k, 4, 0.0, init, icov, w)
    ref64 = oracle.fit(cov, x, k, 4, 0.0, init, icov, w, dtype=np.float64)
    g = GMMXX(k=k, niter=4, tol=0.0, covariance_type=cov, backend="cuda", device=cuda_device)
    g.train(torch.from_numpy(x[0]).to(cuda_device), init_means=torch.from_numpy(init[0]),
            init_covariances=torch.from_numpy(icov[0]), init_weights=torch.from_numpy(w[0]))
    assert g.means_.shape == (k, d) and g.labels_.shape == (5000,)
    got = (g.labels_[None], g.means_[None], g.covariances_[None], g.weights_[None], g.fit_info_)
    _check(got, ref32, ref64, 1e-4)
    assert g.lower_bound_ == pytest.approx(g.fit_info_["lower_bound"])
    # bf16 data: the estimator reads the rounded values in fp32
    xb = torch.from_numpy(x[0]).to(torch.bfloat16)
    xbf = xb.float().numpy()[None]
    rb32 = oracle.fit(cov, xbf, k, 4, 0.0, init, icov, w)
    rb64 = oracle.fit(cov, xbf, k, 4, 0.0, init, icov, w, dtype=np.float64)
    g.train(xb.to(cuda_device), init_means=torch.from_numpy(init), init_covariances=torch.from_numpy(icov),
            init_weights=torch.from_numpy(w))
    assert g.means_.dtype == torch.float32
    _check((g.labels_[None], g.means_[None], g.covariances_[None], g.weights_[None], g.fit_info_), rb32, rb64, 1e-3)


def test_estimator_batched_and_streamed_match_oracle(cuda_device):
    """Batched (B, N, D) input keeps B in the fitted attributes; a host input
    larger than chunk_size_data_cpu goes through the streamed driver; both
    equal the oracle."""
    from gmmxx_b200 import GMMXX

    x, init = _mixture(41, 3, 3000, 6, 5)
    icov = _init_cov("diag", x, 5)
    w = np.full((3, 5), 0.2, np.float32)
    ref32 = oracle.fit("diag", x, 5, 4, 0.0, init, icov, w)
    ref64 = oracle.fit("diag", x, 5, 4, 0.0, init, icov, w, dtype=np.float64)
    g = GMMXX(k=5, niter=4, tol=0.0, covariance_type="diag", backend="cuda", device=cuda_device)
    t = torch.from_numpy
    g.train(t(x).to(cuda_device), init_means=t(init), init_covariances=t(icov), init_weights=t(w))
    assert g.means_.shape == (3, 5, 6)
    _check((g.labels_, g.means_, g.covariances_, g.weights_, g.fit_info_), ref32, ref64, 1e-4)

    xs, init1 = _mixture(42, 1, 9000, 6, 5)
    icov1 = _init_cov("spherical", xs, 5)
    w1 = np.full((1, 5), 0.2, np.float32)
    r32 = oracle.fit("spherical", xs, 5, 4, 0.0, init1, icov1, w1)
    r64 = oracle.fit("spherical", xs, 5, 4, 0.0, init1, icov1, w1, dtype=np.float64)
    g = GMMXX(k=5, niter=4, tol=0.0, covariance_type="spherical", backend="cuda", device=cuda_device,
              chunk_size_data_cpu=2000)
    g.train(t(xs[0]), init_means=t(init1[0]), init_covariances=t(icov1[0]), init_weights=t(w1[0]))
    assert g.large_n_streaming_enabled_
    _check((g.labels_[None], g.means_[None], g.covariances_[None], g.weights_[None], g.fit_info_), r32, r64, 1e-4)


@pytest.mark.parametrize("cov", ["spherical", "diag", "tied", "full"])
def test_largeN_entry_point_matches_oracle(cuda_device, cov):
    """batch_gmm_largeN_cpu (host rows, chunk_size_N-row chunks) from its
    documented initialisation -- the reference's large-N sample
    (large_n.py:630-645: torch.manual_seed(seed), then min(N, max(K, min(65536,
    max(4096, 64 K, K)))) rows drawn with torch.randint), random rows of that
    sample moved to the device (torch_fallback.py:1384-1387), its global
    covariance, uniform weights -- equals the oracle started from the same
    parameters."""
    import gmmxx_b200 as G

    d, k, n, seed = (7, 5, 12_000, 11) if cov != "full" else (4, 3, 12_000, 11)
    x, _ = _mixture(51 + d, 1, n, d, k)
    xt = torch.from_numpy(x)
    out = G.batch_gmm_largeN_cpu(xt, k, covariance_type=cov, device=cuda_device, dtype=torch.float32, max_iters=4,
                                 tol=0.0, chunk_size_N=3000, seed=seed, init_params="random")
    assert out[4]["init_source"] == "random_sampled"
    torch.manual_seed(seed)
    s = min(n, max(k, min(65536, max(4096, 64 * k, k))))
    sample = x[:, torch.randint(0, n, (s,)).numpy()]
    ridx = torch.randint(0, s, (1, k), device=cuda_device)
    m0 = sample[:, ridx[0].cpu().numpy()]
    c0 = _init_cov(cov, sample, k)
    w0 = np.full((1, k), 1.0 / k, np.float32)
    ref32 = oracle.fit(cov, x, k, 4, 0.0, m0, c0, w0)
    ref64 = oracle.fit(cov, x, k, 4, 0.0, m0, c0, w0, dtype=np.float64)
    assert out[0].device.type == "cpu"
    _check(out, ref32, ref64, 1e-4)
