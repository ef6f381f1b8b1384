"""Host-resident X on the GPU: the reference's large-N entry points
(gmmxx/large_n.py:866-1594, 1907-2502) and the estimator's streaming of host
inputs larger than ``chunk_size_data_cpu`` (interface.py:435-491) give the
results of the device-resident calls on the same rows: per-row inference is
identical whatever the chunking, and a streamed fit is the streamed driver's
fit for the same seed."""

import numpy as np
import pytest
import torch

import gmmxx_b200 as G

pytestmark = pytest.mark.gpu


def _mixture(seed, n=5000, d=8, k=6):
    rng = np.random.default_rng(seed)
    centers = rng.uniform(-6, 6, size=(k, d))
    z = rng.integers(0, k, n)
    x = centers[z] + rng.normal(size=(n, d))
    return torch.from_numpy(x.astype(np.float32))[None]


@pytest.mark.parametrize("cov", ["spherical", "diag", "tied", "full"])
def test_largeN_fit_is_the_streamed_fit(cuda_device, cov):
    from gmmxx_b200 import large_n

    x = _mixture(1)
    out = G.batch_gmm_largeN_cpu(x, 6, covariance_type=cov, device=cuda_device, dtype=torch.float32, max_iters=4,
                                 tol=0.0, chunk_size_N=1500, seed=7)
    torch.manual_seed(7)
    ref = large_n.em_fit_streamed(cov, x, 6, device=cuda_device, chunk_rows=1500, max_iters=4, tol=0.0)
    labels, info = out[0], out[4]
    assert labels.device.type == "cpu" and labels.dtype == torch.int64 and labels.shape == (1, 5000)
    assert torch.equal(labels, ref[0].cpu())
    for a, b in zip(out[1:4], ref[1:4]):
        assert torch.equal(a, b)
    assert info["large_n_streaming_enabled"] and info["fallback_reason"] is None
    assert not info["approximate_em_enabled"]


def test_largeN_compute_dtype(cuda_device):
    """dtype=bfloat16 on fp32 host rows computes on the rounded rows, as the
    reference's per-chunk conversion does."""
    x = _mixture(2)
    kw = dict(covariance_type="diag", device=cuda_device, max_iters=3, tol=0.0, chunk_size_N=2000, seed=3)
    a = G.batch_gmm_largeN_cpu(x, 6, dtype=torch.bfloat16, **kw)
    b = G.batch_gmm_largeN_cpu(x.to(torch.bfloat16), 6, dtype=torch.bfloat16, **kw)
    for u, v in zip(a[:4], b[:4]):
        assert torch.equal(u, v)


def test_largeN_inference_matches_device_inference(cuda_device):
    from gmmxx_b200 import engine

    x = _mixture(3)
    xd = x.to(cuda_device)
    _, means, cov, w, _ = engine.em_fit("diag", xd, 6, max_iters=3, tol=0.0)
    kw = dict(covariance_type="diag", device=cuda_device, dtype=torch.float32, chunk_size_N=1300, chunk_size_K=1024)
    lab = G.large_n_predict_cpu(x, means, cov, w, **kw)
    assert lab.device.type == "cpu" and lab.dtype == torch.int64
    assert torch.equal(lab, engine.assign("diag", xd, means, cov, w).cpu())
    score = G.large_n_score_samples_cpu(x, means, cov, w, **kw)
    assert score.device.type == "cpu" and score.shape == (1, 5000)
    np.testing.assert_allclose(score.numpy(), engine.score_samples("diag", xd, means, cov, w).cpu().numpy(),
                               rtol=1e-6, atol=1e-6)
    proba = G.large_n_predict_proba_cpu(x, means, cov, w, **kw)
    assert proba.shape == (1, 5000, 6)
    np.testing.assert_allclose(proba.numpy(), engine.predict_proba("diag", xd, means, cov, w).cpu().numpy(),
                               rtol=1e-6, atol=1e-7)
    assert G.large_n_predict_cpu(x, means, cov, w, return_backend_used=True, **kw)[1] == "cuda"
    assert G.large_n_predict_cpu(x, means, cov, w, return_triton_used=True, **kw)[1] is False


def test_estimator_streams_host_inputs_larger_than_a_chunk(cuda_device):
    """fit / predict / score_samples / predict_proba on host rows beyond
    chunk_size_data_cpu stream them through the GPU (interface.py:435-491)."""
    x = _mixture(4, n=6000)[0]
    g = G.GMMXX(k=6, niter=3, tol=0.0, covariance_type="diag", backend="cuda", seed=1, chunk_size_data_cpu=2000)
    g.fit(x)
    assert g.large_n_streaming_enabled_
    xd = x.to(cuda_device)
    assert torch.equal(g.predict(x).cpu(), g.predict(xd).cpu())
    np.testing.assert_allclose(g.score_samples(x).cpu().numpy(), g.score_samples(xd).cpu().numpy(), rtol=1e-6,
                               atol=1e-6)
    np.testing.assert_allclose(g.predict_proba(x).cpu().numpy(), g.predict_proba(xd).cpu().numpy(), rtol=1e-6,
                               atol=1e-7)
