"""gmmxx_b200 -- a B200-native (sm_100a) soft-EM engine for Gaussian mixtures.

Drop-in for the hot path of OpsiClear/GMMXX: the ``GMMXX`` estimator and the
``batch_gmm_*`` functional API with the reference's signatures, served by
hand-written CUDA kernels behind a C ABI (``include/gmmxx_b200.h``).
"""

from ._native import CudaBackendUnavailable, GmmxxError, UnsupportedShape
from .api import (
    batch_gmm_diag,
    batch_gmm_Diagonal,
    batch_gmm_diagonal,
    batch_gmm_Full,
    batch_gmm_full,
    batch_gmm_Spherical,
    batch_gmm_spherical,
    batch_gmm_Tied,
    batch_gmm_tied,
    diagonal_assign,
    diagonal_predict_proba,
    diagonal_score_samples,
    full_assign,
    full_predict_proba,
    full_score_samples,
    spherical_assign,
    spherical_predict_proba,
    spherical_score_samples,
    tied_assign,
    tied_predict_proba,
    tied_score_samples,
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

__version__ = "0.1.0"
