"""The numpy oracle reproduces the reference's own outputs (golden vectors
recorded from gmmxx/torch_fallback.py by tests/golden/make_golden.py)."""

import numpy as np
import pytest

import oracle
from conftest import golden_cases, load_golden


@pytest.mark.parametrize("case", golden_cases())
def test_oracle_fit_matches_reference(case):
    g = load_golden(case)
    cov = str(g["cov_type"])
    labels, means, c, w, info = oracle.fit(
        cov, g["x"], int(g["n_components"]), int(g["iters"]), 0.0, g["init_means"], g["init_var"],
        g["init_weights"], reg_covar=float(g["reg_covar"]), chunk_size_N=int(g["chunk_size_N"]),
        chunk_size_K=int(g["chunk_size_K"]), approx_top_k=int(g["approx_top_k"]) if "approx_top_k" in g else None)
    assert info["approximate_em_enabled"] == ("approx_top_k" in g)
    np.testing.assert_allclose(means, g["means"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(c, g["cov"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(w, g["weights"], rtol=1e-4, atol=1e-4)
    hist = np.array(info["lower_bound_history"])
    ref = g["lower_bound_history"]
    assert hist.shape == ref.shape
    np.testing.assert_allclose(hist, ref, rtol=1e-4, atol=1e-5)
    assert (labels == g["labels"]).mean() == 1.0


@pytest.mark.parametrize("case", golden_cases())
def test_oracle_inference_matches_reference(case):
    g = load_golden(case)
    cov = str(g["cov_type"])
    kw = dict(chunk_size_N=int(g["chunk_size_N"]), chunk_size_K=int(g["chunk_size_K"]))
    args = (cov, g["x"], g["means"], g["cov"], g["weights"])
    assert (oracle.assign(*args, **kw) == g["assign"]).all()
    np.testing.assert_allclose(oracle.score_samples(*args, **kw), g["score_samples"], rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(oracle.predict_proba(*args, **kw), g["predict_proba"], rtol=1e-4, atol=1e-5)


def test_oracle_float32_noise_floor_is_small():
    """fp32 oracle vs the same algorithm in fp64 on a golden case: the fp32
    arithmetic of the reference is far inside the parity tolerances."""
    g = load_golden("diag_basic")
    a = oracle.fit("diag", g["x"], 4, 8, 0.0, g["init_means"], g["init_var"], g["init_weights"])
    b = oracle.fit("diag", g["x"], 4, 8, 0.0, g["init_means"], g["init_var"], g["init_weights"], dtype=np.float64)
    np.testing.assert_allclose(a[1], b[1], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(a[2], b[2], rtol=1e-4, atol=1e-5)


def test_oracle_jitter_ladder_engages_on_singular_covariance():
    cov = np.zeros((1, 3, 3), np.float32)
    cov[0, 0, 0] = cov[0, 1, 1] = 1.0  # third direction singular
    prec, logdet = oracle.precision_and_logdet(cov)
    assert np.isfinite(prec).all()
    # first working jitter is 1e-6 -> log det = log(1e-6)
    assert abs(float(logdet[0]) - np.log(1e-6)) < 1e-3


def test_oracle_approx_top_k_edges():
    """approx_top_k >= K is exact EM (torch_fallback.py:605-606); <= 0 is an
    error; top_k = 1 gives hard responsibilities (each row's whole weight on
    its best component)."""
    g = load_golden("diag_basic")
    args = ("diag", g["x"], 4, 3, 0.0, g["init_means"], g["init_var"], g["init_weights"])
    exact = oracle.fit(*args)
    same = oracle.fit(*args, approx_top_k=4)
    assert not same[4]["approximate_em_enabled"] and same[4]["approx_top_k"] is None
    for a, b in zip(exact[1:4], same[1:4]):
        np.testing.assert_array_equal(a, b)
    with pytest.raises(ValueError):
        oracle.fit(*args, approx_top_k=0)
    hard = oracle.fit("diag", g["x"], 4, 1, 0.0, g["init_means"], g["init_var"], g["init_weights"],
                      approx_top_k=1)
    lab = oracle.assign("diag", g["x"], *_first_step_params(g))
    counts = np.bincount(lab[0], minlength=4).astype(np.float32) / lab.shape[1]
    np.testing.assert_allclose(hard[3][0], np.maximum(counts, 1e-8) / np.maximum(counts, 1e-8).sum(), rtol=1e-5)


def _first_step_params(g):
    """The parameters the first iteration's E-step uses (weights renormalised,
    variances clamped as the loop's prologue does)."""
    w = np.maximum(g["init_weights"], np.float32(1e-8))
    w = (w / w.sum(-1, keepdims=True)).astype(np.float32)
    return g["init_means"], np.maximum(g["init_var"], np.float32(1e-6)), w
