"""The functional API's names and parameters are the reference's
(gmmxx/__init__.py:11-34, torch_fallback.py:780-1345, 1897-3513), and its
argument checks run on the host before any kernel."""

import inspect

import pytest
import torch

import gmmxx_b200 as G

FIT_COMMON = ["x", "n_components", "max_iters", "tol", "init_means", "init_variances", "init_weights", "verbose",
              "init_params", "reg_covar", "chunk_size_N", "chunk_size_K", "kmeans_init_iters", "kmeans_init_tol"]
TAIL = ["min_weight", "compute_labels", "approx_top_k"]


@pytest.mark.parametrize("name,switches", [
    ("batch_gmm_Spherical", ["use_triton"]),
    ("batch_gmm_Diagonal", ["use_triton"]),
    ("batch_gmm_Full", ["use_triton"]),
    ("batch_gmm_Tied", ["use_triton"]),
    ("batch_gmm_Spherical_torch_native",
     ["kmeans_use_triton", "gmm_use_triton_estep", "gmm_use_triton_streaming_update"]),
    ("batch_gmm_Diagonal_torch_native", ["kmeans_use_triton", "gmm_use_triton"]),
    ("batch_gmm_Full_torch_native", ["kmeans_use_triton", "gmm_use_triton"]),
    ("batch_gmm_Tied_torch_native", ["kmeans_use_triton", "gmm_use_triton"]),
])
def test_fit_signatures(name, switches):
    params = list(inspect.signature(getattr(G, name)).parameters)
    assert params == FIT_COMMON + switches + TAIL


@pytest.mark.parametrize("cov,third", [("spherical", "variances"), ("diagonal", "variances"),
                                       ("tied", "covariance"), ("full", "covariances")])
@pytest.mark.parametrize("kind", ["assign", "score_samples", "predict_proba"])
def test_inference_signatures(cov, third, kind):
    for name in (f"{cov}_{kind}", f"{cov}_{kind}_torch_native_chunked"):
        fn = getattr(G, name)
        assert list(inspect.signature(fn).parameters) == ["x", "means", third, "weights", "chunk_size_N",
                                                          "chunk_size_K"], name


def test_lowercase_aliases():
    assert G.batch_gmm_spherical is G.batch_gmm_Spherical
    assert G.batch_gmm_diag is G.batch_gmm_Diagonal and G.batch_gmm_diagonal is G.batch_gmm_Diagonal
    assert G.batch_gmm_full is G.batch_gmm_Full and G.batch_gmm_tied is G.batch_gmm_Tied


@pytest.mark.parametrize("call,exc", [
    (lambda x: G.batch_gmm_Diagonal_torch_native(x, 3, gmm_use_triton="sometimes"), ValueError),
    (lambda x: G.batch_gmm_Spherical_torch_native(x, 3, gmm_use_triton_estep="x"), ValueError),
    (lambda x: G.batch_gmm_Spherical(x, 3, approx_top_k=0), ValueError),
    (lambda x: G.batch_gmm_Spherical(x, 0), ValueError),
    (lambda x: G.batch_gmm_Tied(x, 3, chunk_size_N=0), ValueError),
    (lambda x: G.batch_gmm_Full(x, 3, min_weight=0.0), ValueError),
    (lambda x: G.batch_gmm_Spherical(x[0], 3), ValueError),          # not (B, N, D)
    (lambda x: G.batch_gmm_Spherical(x, 3), ValueError),             # host tensor: the engine needs CUDA
    (lambda x: G.spherical_assign(x, x[:, :2], torch.ones(1, 2), torch.ones(1, 2), chunk_size_N=0), ValueError),
])
def test_argument_checks(call, exc):
    with pytest.raises(exc):
        call(torch.zeros(1, 8, 2))


REFERENCE_EXPORTS = [
    "batch_gmm_Spherical", "batch_gmm_Spherical_torch_native", "batch_gmm_Diagonal",
    "batch_gmm_Diagonal_torch_native", "batch_gmm_Full", "batch_gmm_Full_torch_native", "batch_gmm_Tied",
    "batch_gmm_Tied_torch_native", "batch_gmm_spherical", "batch_gmm_diagonal", "batch_gmm_diag", "batch_gmm_full",
    "batch_gmm_tied", "diagonal_assign_torch_native_chunked", "diagonal_predict_proba_torch_native_chunked",
    "diagonal_score_samples_torch_native_chunked", "full_assign_torch_native_chunked",
    "full_predict_proba_torch_native_chunked", "full_score_samples_torch_native_chunked",
    "tied_assign_torch_native_chunked", "tied_predict_proba_torch_native_chunked",
    "tied_score_samples_torch_native_chunked", "GMMXX", "batch_gmm_largeN_cpu", "large_n_predict_cpu",
    "large_n_predict_proba_cpu", "large_n_score_samples_cpu", "spherical_assign_triton", "spherical_logsumexp_triton",
    "spherical_resp_triton", "diag_assign_triton", "diag_logsumexp_triton", "diag_resp_triton", "full_assign_triton",
    "full_logsumexp_triton", "full_resp_triton", "triton_blocked_update_diag", "triton_blocked_update_full",
    "triton_blocked_update_spherical", "triton_blocked_update_tied_projected", "triton_streaming_update_spherical",
    "triton_weighted_update_spherical", "fused_single_tile_update_config", "triton_fused_single_tile_update_diag",
    "triton_fused_single_tile_update_spherical", "triton_fused_single_tile_update_tied_native",
    "approx_topk_update_spherical_config", "triton_approx_topk_update_spherical", "cuda_ops",
]


def test_every_reference_export_is_importable():
    """Every name the reference package exports (gmmxx/__init__.py:104-154)
    imports from gmmxx_b200; the Triton kernels are None, as they are in the
    reference when Triton is unavailable."""
    for name in REFERENCE_EXPORTS:
        assert hasattr(G, name), name
        if "triton" in name or name.endswith("_config"):
            assert getattr(G, name) is None, name
