"""gmmxx_b200 -- a B200-native (sm_100a) soft-EM engine for Gaussian mixtures.

Drop-in for the hot path of OpsiClear/GMMXX: the ``GMMXX`` estimator and the
``batch_gmm_*`` functional API with the reference's signatures, served by
hand-written CUDA kernels behind a C ABI (``include/gmmxx_b200.h``).
"""

from ._native import CudaBackendUnavailable, GmmxxError, UnsupportedShape
from .api import (
    batch_gmm_diag,
    batch_gmm_Diagonal,
    batch_gmm_Diagonal_torch_native,
    batch_gmm_diagonal,
    batch_gmm_Full,
    batch_gmm_Full_torch_native,
    batch_gmm_full,
    batch_gmm_Spherical,
    batch_gmm_Spherical_torch_native,
    batch_gmm_spherical,
    batch_gmm_Tied,
    batch_gmm_Tied_torch_native,
    batch_gmm_tied,
    diagonal_assign,
    diagonal_assign_torch_native_chunked,
    diagonal_predict_proba,
    diagonal_predict_proba_torch_native_chunked,
    diagonal_score_samples,
    diagonal_score_samples_torch_native_chunked,
    full_assign,
    full_assign_torch_native_chunked,
    full_predict_proba,
    full_predict_proba_torch_native_chunked,
    full_score_samples,
    full_score_samples_torch_native_chunked,
    spherical_assign,
    spherical_assign_torch_native_chunked,
    spherical_predict_proba,
    spherical_predict_proba_torch_native_chunked,
    spherical_score_samples,
    spherical_score_samples_torch_native_chunked,
    tied_assign,
    tied_assign_torch_native_chunked,
    tied_predict_proba,
    tied_predict_proba_torch_native_chunked,
    tied_score_samples,
    tied_score_samples_torch_native_chunked,
)
from . import cuda_ops  # noqa: F401  (the reference's operator-level surface, gmmxx.cuda_ops)
from .interface import GMMXX
from .large_n import (
    batch_gmm_largeN_cpu,
    em_fit_streamed,
    large_n_predict_cpu,
    large_n_predict_proba_cpu,
    large_n_score_samples_cpu,
)

__all__ = [
    "GMMXX",
    "CudaBackendUnavailable",
    "GmmxxError",
    "UnsupportedShape",
    "batch_gmm_Spherical",
    "batch_gmm_Diagonal",
    "batch_gmm_Full",
    "batch_gmm_Tied",
    "batch_gmm_spherical",
    "batch_gmm_diagonal",
    "batch_gmm_diag",
    "batch_gmm_full",
    "batch_gmm_tied",
    "batch_gmm_Spherical_torch_native",
    "batch_gmm_Diagonal_torch_native",
    "batch_gmm_Full_torch_native",
    "batch_gmm_Tied_torch_native",
    "spherical_assign_torch_native_chunked",
    "spherical_score_samples_torch_native_chunked",
    "spherical_predict_proba_torch_native_chunked",
    "diagonal_assign_torch_native_chunked",
    "diagonal_score_samples_torch_native_chunked",
    "diagonal_predict_proba_torch_native_chunked",
    "tied_assign_torch_native_chunked",
    "tied_score_samples_torch_native_chunked",
    "tied_predict_proba_torch_native_chunked",
    "full_assign_torch_native_chunked",
    "full_score_samples_torch_native_chunked",
    "full_predict_proba_torch_native_chunked",
    "spherical_assign",
    "spherical_score_samples",
    "spherical_predict_proba",
    "diagonal_assign",
    "diagonal_score_samples",
    "diagonal_predict_proba",
    "tied_assign",
    "tied_score_samples",
    "tied_predict_proba",
    "full_assign",
    "full_score_samples",
    "full_predict_proba",
    "em_fit_streamed",
    "batch_gmm_largeN_cpu",
    "large_n_predict_cpu",
    "large_n_predict_proba_cpu",
    "large_n_score_samples_cpu",
    "cuda_ops",
]

# The reference exports its Triton kernels under these names and sets each to
# None when Triton is unavailable (gmmxx/__init__.py:35-101).  This engine has
# no Triton kernels, so they are None here too: code that imports them, or
# tests them against None before use, runs unchanged.
approx_topk_update_spherical_config = None
triton_approx_topk_update_spherical = None
spherical_assign_triton = None
spherical_logsumexp_triton = None
spherical_resp_triton = None
diag_assign_triton = None
diag_logsumexp_triton = None
diag_resp_triton = None
full_assign_triton = None
full_logsumexp_triton = None
full_resp_triton = None
triton_blocked_update_diag = None
triton_blocked_update_full = None
triton_blocked_update_spherical = None
triton_blocked_update_tied_projected = None
triton_streaming_update_spherical = None
triton_weighted_update_spherical = None
fused_single_tile_update_config = None
triton_fused_single_tile_update_diag = None
triton_fused_single_tile_update_spherical = None
triton_fused_single_tile_update_tied_native = None

__version__ = "0.1.0"
