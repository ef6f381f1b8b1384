"""Inference on the tensor-core kernels (bf16 X): the diag kernel (D = 64,
K <= 512, one pass per call; also spherical D = 128 with K <= 512 or in
groups of 512 components) and em_tc_kernel (spherical D = 64, and D = 128
with 512 < K <= 1024: per-row passes per group of 1024 components): labels, score_samples and
predict_proba against the numpy oracle of the reference's chunked torch
functions (torch_fallback.py:780-821, 824-871, 983-1056, 1133-1237) and
against the exact-fp32 CUDA-core kernels on the same inputs.

Tolerances (bf16 X is exact; the logits carry fp32-equivalent weights and
fp32 tensor-core accumulation): log-sum-exp within 2e-4 relative + 2e-3
absolute of the oracle, responsibilities within 1e-4 absolute, labels equal
on at least 99.9 % of rows (rows whose two best components tie to fp32
rounding may flip)."""

import os

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _case(seed, n, d, k, cov_type="diag"):
    rng = np.random.default_rng(seed)
    mu = rng.normal(0, 3.0 if cov_type == "diag" else 2.0, (k, d))
    if cov_type == "diag":
        var = np.exp(rng.uniform(np.log(0.1), np.log(4.0), (k, d)))
    else:
        var = np.repeat(rng.uniform(0.3, 1.5, (k, 1)) ** 2, d, 1)
    w = rng.dirichlet(np.full(k, 0.5))
    z = rng.choice(k, n, p=w)
    x = (mu[z] + np.sqrt(var[z]) * rng.standard_normal((n, d))).astype(np.float32)
    xb = torch.from_numpy(x).to(torch.bfloat16)[None]
    means = (mu + 0.2 * rng.standard_normal(mu.shape)).astype(np.float32)[None]
    if cov_type == "diag":
        cov = (var * rng.uniform(0.8, 1.25, var.shape)).astype(np.float32)[None]
    else:
        cov = (var[:, 0] * rng.uniform(0.8, 1.25, k)).astype(np.float32)[None]
    wts = (w / w.sum()).astype(np.float32)[None]
    return xb, means, cov, wts


def _infer(dev, xb, means, cov, wts, kernel, cov_type="diag"):
    from gmmxx_b200 import _native as nat
    from gmmxx_b200 import engine

    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    os.environ["GMMXX_B200_KERNEL"] = kernel
    try:
        x = xb.to(dev)
        b, n, d = x.shape
        code = nat.DIAG if cov_type == "diag" else nat.SPHERICAL
        path = nat.accumulate_path(code, nat.BFLOAT16, b, n, d, means.shape[1])
        args = (cov_type, x, t(means), t(cov), t(wts))
        out = (engine.assign(*args).cpu().numpy(), engine.score_samples(*args).cpu().numpy(),
               engine.predict_proba(*args).cpu().numpy())
        torch.cuda.synchronize()
        return path, out
    finally:
        os.environ.pop("GMMXX_B200_KERNEL", None)


@pytest.mark.parametrize("n,k", [
    (200_000, 512),   # config-1 shape, cluster of 4
    (70_001, 300),    # ragged N, padded components, cluster of 3
    (66_000, 333),    # K % 4 != 0: scalar stores of responsibilities
    (65_536, 40),     # single-CTA cluster
])
def test_tc_inference_matches_oracle(cuda_device, n, k):
    xb, means, cov, wts = _case(11 + k, n, 64, k)
    path, (lab, lse, proba) = _infer(cuda_device, xb, means, cov, wts, "tc")
    assert path == 1
    x = xb.float().numpy()
    ref_lab = oracle.assign("diag", x, means, cov, wts)
    ref_lse = oracle.score_samples("diag", x, means, cov, wts)
    assert lab.shape == ref_lab.shape and lab.dtype == np.int64
    assert (lab == ref_lab).mean() >= 0.999
    np.testing.assert_allclose(lse, ref_lse, rtol=2e-4, atol=2e-3)
    assert proba.shape == (1, n, k)
    # row sums are 1 and rows agree with the oracle's exp(logit - lse)
    np.testing.assert_allclose(proba.sum(-1), 1.0, atol=1e-4)
    sl = slice(0, 4096)
    ref_p = oracle.predict_proba("diag", x[:, sl], means, cov, wts)
    np.testing.assert_allclose(proba[:, sl], ref_p, atol=1e-4)


def test_tc_inference_matches_cuda_cores(cuda_device):
    xb, means, cov, wts = _case(5, 131_072, 64, 512)
    p_tc, (lab_tc, lse_tc, pr_tc) = _infer(cuda_device, xb, means, cov, wts, "tc")
    p_simt, (lab_s, lse_s, pr_s) = _infer(cuda_device, xb, means, cov, wts, "simt")
    assert p_tc == 1 and p_simt == 0
    assert (lab_tc == lab_s).mean() >= 0.999
    np.testing.assert_allclose(lse_tc, lse_s, rtol=2e-4, atol=2e-3)
    np.testing.assert_allclose(pr_tc, pr_s, atol=1e-4)


def test_tc_inference_labels_first_of_equal_components(cuda_device):
    """Two identical components: the argmax keeps the first (the reference's
    strict '>' merge, torch_fallback.py:814-817) within a row part, across
    parts of one CTA and across cluster ranks."""
    xb, means, cov, wts = _case(3, 65_536, 64, 256)
    pairs = ((5, 6), (40, 40 + 64), (20, 20 + 128))
    for a, b in pairs:
        means[0, b] = means[0, a]
        cov[0, b] = cov[0, a]
        wts[0, a] = wts[0, b] = 0.1
    _, (lab, _, _) = _infer(cuda_device, xb, means, cov, wts, "tc")
    for a, b in pairs:
        assert (lab == a).any()
        assert not (lab == b).any()


@pytest.mark.parametrize("n,d,k", [
    (100_000, 128, 256),   # one group of 2 chunks
    (65_536, 64, 64),      # one CTA
    (70_001, 128, 1024),   # one group of 8 chunks, ragged N
    (66_000, 128, 2304),   # three groups (8, 8, 2 chunks): combine kernels
    (65_536, 64, 1100),    # two groups, K % 4 == 0 but the last chunk padded
])
def test_tc_spherical_inference_matches_oracle(cuda_device, n, d, k):
    xb, means, cov, wts = _case(21 + k + d, n, d, k, "spherical")
    path, (lab, lse, proba) = _infer(cuda_device, xb, means, cov, wts, "tc", "spherical")
    assert path == 1
    x = xb.float().numpy()
    ref_lab = oracle.assign("spherical", x, means, cov, wts)
    ref_lse = oracle.score_samples("spherical", x, means, cov, wts)
    assert lab.dtype == np.int64 and (lab == ref_lab).mean() >= 0.999
    np.testing.assert_allclose(lse, ref_lse, rtol=2e-4, atol=2e-3)
    assert proba.shape == (1, n, k)
    np.testing.assert_allclose(proba.sum(-1), 1.0, atol=1e-4)
    sl = slice(0, 2048)
    np.testing.assert_allclose(proba[:, sl], oracle.predict_proba("spherical", x[:, sl], means, cov, wts), atol=1e-4)


def test_tc_spherical_inference_matches_cuda_cores(cuda_device):
    xb, means, cov, wts = _case(8, 65_536, 128, 2304, "spherical")
    p_tc, (lab_tc, lse_tc, pr_tc) = _infer(cuda_device, xb, means, cov, wts, "tc", "spherical")
    p_s, (lab_s, lse_s, pr_s) = _infer(cuda_device, xb, means, cov, wts, "simt", "spherical")
    assert p_tc == 1 and p_s == 0
    assert (lab_tc == lab_s).mean() >= 0.999
    np.testing.assert_allclose(lse_tc, lse_s, rtol=2e-4, atol=2e-3)
    np.testing.assert_allclose(pr_tc, pr_s, atol=1e-4)


@pytest.mark.parametrize("d", [64, 128])
def test_tc_spherical_labels_first_of_equal_components(cuda_device, d):
    """Identical components across halves, cluster ranks and groups: the
    first one wins (torch_fallback.py:814-817)."""
    xb, means, cov, wts = _case(4, 65_536, d, 2304, "spherical")
    counts = np.bincount(oracle.assign("spherical", xb.float().numpy(), means, cov, wts)[0], minlength=2304)
    # the most populated component of a range, duplicated `offset` later
    spans = ((0, 64, 64), (128, 256, 128), (256, 512, 1024), (1024, 1280, 512))
    pairs = []
    for lo, hi, offset in spans:
        a = lo + int(np.argmax(counts[lo:hi]))
        pairs.append((a, a + offset))
    for a, b in pairs:
        means[0, b] = means[0, a]
        cov[0, b] = cov[0, a]
        wts[0, b] = wts[0, a]
    _, (lab, _, _) = _infer(cuda_device, xb, means, cov, wts, "tc", "spherical")
    for a, b in pairs:
        assert (lab == a).any()
        assert not (lab == b).any()


@pytest.mark.parametrize("n,k", [
    (80_000, 256),    # one pass, cluster of 2
    (70_001, 512),    # one pass, cluster of 4, ragged N
    (66_000, 2304),   # grouped: 5 groups of 4 chunks, the last of 2
    (65_536, 1030),   # grouped, K % 4 != 0: per-element stores of responsibilities
])
def test_tc_sph128_inference_layouts_agree(cuda_device, n, k):
    """Spherical D = 128 inference on the diag kernel's layout (one pass for
    K <= 512; per-group row statistics or labels, their combination, and for
    predict_proba a pass per group from the combined log-sum-exp) agrees with
    em_tc_kernel (GMMXX_B200_SPH_KERNEL=legacy) and with the oracle."""
    xb, means, cov, wts = _case(51 + k, n, 128, k, "spherical")
    path, (lab, lse, proba) = _infer(cuda_device, xb, means, cov, wts, "tc", "spherical")
    os.environ["GMMXX_B200_SPH_KERNEL"] = "legacy"
    try:
        p_old, (lab_o, lse_o, pr_o) = _infer(cuda_device, xb, means, cov, wts, "tc", "spherical")
    finally:
        os.environ.pop("GMMXX_B200_SPH_KERNEL", None)
    assert path == 1 and p_old == 1
    # the two layouts form |x|^2 differently (fp32 in the prep warps against
    # three bf16 terms through the tensor cores): agreement to the path's
    # tolerance against the oracle
    assert (lab == lab_o).mean() >= 0.999
    np.testing.assert_allclose(lse, lse_o, rtol=2e-4, atol=2e-3)
    np.testing.assert_allclose(proba, pr_o, atol=1e-4)
    x = xb.float().numpy()
    assert (lab == oracle.assign("spherical", x, means, cov, wts)).mean() >= 0.999
    np.testing.assert_allclose(lse, oracle.score_samples("spherical", x, means, cov, wts), rtol=2e-4, atol=2e-3)
    np.testing.assert_allclose(proba.sum(-1), 1.0, atol=1e-4)
    sl = slice(0, 2048)
    np.testing.assert_allclose(proba[:, sl], oracle.predict_proba("spherical", x[:, sl], means, cov, wts), atol=1e-4)


@pytest.mark.parametrize("cov_type,d,k", [("diag", 64, 512), ("spherical", 128, 1100), ("spherical", 128, 256)])
def test_tc_predict_proba_unaligned_output(cuda_device, cov_type, d, k):
    """predict_proba into a caller buffer that starts 4 bytes off a 16-byte
    boundary: the kernels take their per-element store path (the host checks
    the alignment before allowing 16-byte stores) and agree with an aligned
    call bit for bit."""
    from gmmxx_b200 import engine

    xb, means, cov, wts = _case(31, 65_536, d, k, cov_type)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)
    x = xb.to(cuda_device)
    args = (cov_type, x, t(means), t(cov), t(wts))
    n = x.shape[1]
    buf = torch.full((n * k + 1,), -1.0, dtype=torch.float32, device=cuda_device)
    out = buf[1:].view(1, n, k)
    assert out.data_ptr() % 16 != 0
    got = engine.predict_proba(*args, out=out)
    ref = engine.predict_proba(*args)
    torch.cuda.synchronize()
    assert buf[0].item() == -1.0  # nothing written before the view
    assert torch.equal(got, ref)
