"""``GMMXX`` estimator backed by the B200 engine.

Same constructor, attributes and methods as the reference estimator
(gmmxx/interface.py:125-2558): fit / train / fit_predict / predict /
predict_proba / score_samples / score / aic / bic / get_params / set_params,
(N, D) or batched (B, N, D) input, spherical / diag / tied / full covariance.
Every fit and inference call runs on the CUDA engine; there is no Triton or
torch fallback, so ``backend="cuda"`` or ``"auto"`` on a machine without the
engine raises :class:`CudaBackendUnavailable` instead of silently degrading.
Host-resident inputs larger than ``chunk_size_data_cpu`` rows are streamed
through the GPU each iteration (gmmxx_b200.large_n), as in the reference
(interface.py:435-491).
"""

from __future__ import annotations

import math
import os
import warnings
from typing import Any, Optional

import torch

from . import _native as nat
from . import engine, large_n

_VALID_COVARIANCE_TYPES = {"spherical", "diag", "tied", "full"}
_VALID_BACKENDS = {"auto", "cuda", "triton", "torch"}
_COVARIANCE_ALIASES = {"diagonal": "diag"}
_SKLEARN_PARAM_ALIASES = {"n_components": "k", "max_iter": "niter", "random_state": "seed", "n_features": "d"}


def _normalize_covariance_type(covariance_type: str) -> str:
    covariance_type = _COVARIANCE_ALIASES.get(covariance_type, covariance_type)
    if covariance_type not in _VALID_COVARIANCE_TYPES:
        raise ValueError("covariance_type must be 'spherical', 'diag', 'diagonal', 'tied', or 'full'")
    return covariance_type


def _optional_positive_int(value, name):
    if value is None:
        return None
    value = int(value)
    if value <= 0:
        raise ValueError(f"{name} must be positive")
    return value


def _positive_int(value, name):
    value = int(value)
    if value <= 0:
        raise ValueError(f"{name} must be positive")
    return value


def _resolve_alias(primary, alias, *, primary_name, alias_name):
    if primary is not None and alias is not None and int(primary) != int(alias):
        raise ValueError(f"Received conflicting {primary_name}={primary} and {alias_name}={alias}")
    return primary if primary is not None else alias


class GMMXX:
    """Gaussian mixture model fitted by soft EM on the B200 engine
    (reference: gmmxx/interface.py:125)."""

    def __init__(
        self,
        d: Optional[int] = None,
        k: Optional[int] = None,
        niter: Optional[int] = None,
        tol: float = 1e-4,
        use_triton: Optional[bool] = None,
        seed: Optional[int] = None,
        chunk_size_data: int = 32768,
        chunk_size_centroids: int = 1024,
        chunk_size_data_cpu: int = 1048576,
        verbose: bool = False,
        dtype: Optional[torch.dtype] = None,
        device: Optional[torch.device] = None,
        init_params: str = "kmeans",
        reg_covar: float = 1e-6,
        init_kmeans_iters: int = 10,
        init_kmeans_tol: float = 1e-4,
        covariance_type: str = "spherical",
        matmul_precision: Optional[str] = None,
        compute_labels_on_fit: bool = True,
        approx_top_k: Optional[int] = None,
        n_components: Optional[int] = None,
        max_iter: Optional[int] = None,
        random_state: Optional[int] = None,
        n_features: Optional[int] = None,
        backend: str = "auto",
    ):
        d = _resolve_alias(d, n_features, primary_name="d", alias_name="n_features")
        k = _resolve_alias(k, n_components, primary_name="k", alias_name="n_components")
        niter = _resolve_alias(niter, max_iter, primary_name="niter", alias_name="max_iter")
        seed = _resolve_alias(seed, random_state, primary_name="seed", alias_name="random_state")
        if backend not in _VALID_BACKENDS:
            raise ValueError(f"backend must be one of {_VALID_BACKENDS}, got {backend!r}")
        if use_triton is not None:
            if backend != "auto":
                raise ValueError(
                    "Cannot pass both backend= and use_triton= to GMMXX. Drop use_triton; backend= is the canonical kwarg.")
            warnings.warn("use_triton is deprecated; use backend=... instead.", DeprecationWarning, stacklevel=2)
            self._legacy_no_triton = use_triton is False
        else:
            self._legacy_no_triton = False
        self.backend = backend
        if k is None:
            raise ValueError("k or n_components is required")
        self.d = _optional_positive_int(d, "d")
        self.k = _positive_int(k, "k")
        self.niter = _positive_int(100 if niter is None else niter, "niter")
        self.tol = float(tol)
        if self.tol < 0.0:
            raise ValueError("tol must be non-negative")
        self.seed = int(0 if seed is None else seed)
        self.chunk_size_data = _positive_int(chunk_size_data, "chunk_size_data")
        self.chunk_size_centroids = _positive_int(chunk_size_centroids, "chunk_size_centroids")
        self.chunk_size_data_cpu = _positive_int(chunk_size_data_cpu, "chunk_size_data_cpu")
        self.verbose = bool(verbose)
        self.dtype = dtype
        self.init_params = init_params
        self.reg_covar = float(reg_covar)
        if self.reg_covar < 0.0:
            raise ValueError("reg_covar must be non-negative")
        self.init_kmeans_iters = _positive_int(init_kmeans_iters, "init_kmeans_iters")
        self.init_kmeans_tol = float(init_kmeans_tol)
        if self.init_kmeans_tol < 0.0:
            raise ValueError("init_kmeans_tol must be non-negative")
        self.covariance_type = _normalize_covariance_type(covariance_type)
        if matmul_precision is not None and matmul_precision not in {"highest", "high", "medium"}:
            raise ValueError("matmul_precision must be None, 'highest', 'high', or 'medium'")
        self.matmul_precision = matmul_precision
        self.compute_labels_on_fit = bool(compute_labels_on_fit)
        self.approx_top_k = _optional_positive_int(approx_top_k, "approx_top_k")
        self._raw_device = device
        if device is None:
            self.device = torch.device("cuda:0" if torch.cuda.is_available() else "cpu")
        else:
            self.device = torch.device(device)
        self._reset_fit_state()

    # --- state ---------------------------------------------------------------

    @property
    def use_triton(self) -> bool:
        return False

    def _reset_fit_state(self) -> None:
        self.means_b = self.variances_b = self.covariances_b = self.weights_b = None
        self.cluster_ids_b = None
        self.means_ = self.weights_ = self.covariances_ = self.labels_ = None
        self.lower_bound_ = None
        self.lower_bound_history_ = None
        self.n_iter_ = None
        self.init_source_ = None
        self.fit_info_ = None
        self.triton_estep_enabled_ = None
        self.triton_fused_update_enabled_ = None
        self.triton_approx_topk_enabled_ = None
        self.triton_streaming_update_enabled_ = None
        self.triton_labels_enabled_ = None
        self.approximate_em_enabled_ = None
        self.approx_top_k_ = None
        self.large_n_streaming_enabled_ = None
        self.copy_stream_prefetch_enabled_ = None
        self.last_fallback_reason_ = None
        self.last_backend_used_ = None
        self.cuda_estep_enabled_ = None
        self.cuda_fused_update_enabled_ = None
        self.cuda_approx_topk_enabled_ = None
        self._batch_size = None

    def _squeeze_if_unbatched(self, value):
        if value is None:
            return None
        return value.squeeze(0) if self._batch_size is None else value

    def _set_fit_result(self, *, labels_b, means_b, variances_b, weights_b, info, batch_size) -> None:
        self.cluster_ids_b = labels_b
        self.means_b = means_b
        self.variances_b = variances_b
        self.covariances_b = variances_b
        self.weights_b = weights_b
        self._batch_size = batch_size
        self.means_ = self._squeeze_if_unbatched(means_b)
        self.weights_ = self._squeeze_if_unbatched(weights_b)
        self.covariances_ = self._squeeze_if_unbatched(variances_b)
        self.labels_ = self._squeeze_if_unbatched(labels_b)
        self.lower_bound_ = float(info["lower_bound"])
        self.lower_bound_history_ = list(info["lower_bound_history"])
        self.n_iter_ = int(info["n_iter"])
        self.init_source_ = str(info["init_source"])
        self.fit_info_ = dict(info)
        self.triton_estep_enabled_ = False
        self.triton_fused_update_enabled_ = False
        self.triton_approx_topk_enabled_ = False
        self.triton_streaming_update_enabled_ = False
        self.triton_labels_enabled_ = False
        self.approximate_em_enabled_ = bool(info.get("approximate_em_enabled", False))
        self.approx_top_k_ = info.get("approx_top_k")
        self.large_n_streaming_enabled_ = bool(info.get("large_n_streaming_enabled", False))
        self.copy_stream_prefetch_enabled_ = bool(info.get("copy_stream_prefetch_enabled", False))
        self.last_fallback_reason_ = None
        self.last_backend_used_ = "cuda"
        self.cuda_estep_enabled_ = True
        self.cuda_fused_update_enabled_ = True
        self.cuda_approx_topk_enabled_ = bool(info.get("cuda_approx_topk_enabled", False))

    # --- input handling --------------------------------------------------------

    def _normalize_input(self, data):
        if not torch.is_tensor(data):
            raise TypeError("data must be a torch.Tensor")
        if not data.dtype.is_floating_point:
            raise TypeError("data must be a floating point tensor")
        if data.ndim == 2:
            n, d = data.shape
            if n == 0:
                raise ValueError("data must contain at least one sample")
            if self.d is None:
                self.d = int(d)
            elif d != self.d:
                raise ValueError(f"Expected d={self.d}, got d={d}")
            return data.unsqueeze(0), None
        if data.ndim == 3:
            bsz, _, d = data.shape
            if bsz == 0 or data.shape[1] == 0:
                raise ValueError("data must contain at least one sample")
            if self.d is None:
                self.d = int(d)
            elif d != self.d:
                raise ValueError(f"Expected d={self.d}, got d={d}")
            return data, bsz
        raise ValueError("data must have shape (N, D) or (B, N, D)")

    def _effective_backend(self) -> str:
        """``backend``, with the GMMXX_BACKEND environment variable consulted
        when it is "auto" and ignored when not a valid name (the reference's
        resolve_backend_with_env, _dispatch.py:128-144)."""
        if self.backend == "auto":
            env = os.environ.get("GMMXX_BACKEND")
            if env in _VALID_BACKENDS:
                return env
        return self.backend

    def _require_engine(self) -> None:
        backend = self._effective_backend()
        if backend in {"triton", "torch"}:
            raise ValueError(
                f"backend={backend!r} is not provided by gmmxx_b200; this engine implements the CUDA backend "
                "(use backend='cuda' or 'auto')")
        if self.device.type != "cuda":
            raise nat.CudaBackendUnavailable("the gmmxx_b200 engine needs a CUDA device")
        nat.load()

    def _engine_dtype(self, x_b):
        """Input dtype the engine reads.  bf16/fp16 inputs are read as stored and
        computed in fp32 -- identical to the reference's upcast
        (interface.py:426-433) because the conversion is exact."""
        if self.dtype is not None and self.dtype != x_b.dtype:
            return self.dtype
        return x_b.dtype

    def _is_large_cpu_stream_input(self, x_b) -> bool:
        return x_b.device.type == "cpu" and self.device.type == "cuda" and x_b.shape[1] > self.chunk_size_data_cpu

    def _prepare_compute_tensor(self, x_b):
        return x_b.to(device=self.device, dtype=self._engine_dtype(x_b), copy=False).contiguous()

    # --- fitting -----------------------------------------------------------------

    def train(self, data, init_means=None, init_covariances=None, init_weights=None):
        """Fit.  ``init_*`` inject initial parameters (the parity seam of the
        reference's functional API, torch_fallback.py:1646-1682); they are
        optional extras over the reference estimator."""
        self._reset_fit_state()
        x_b, batch_size = self._normalize_input(data)
        if batch_size is None:  # unbatched (N, D) data: init tensors may come without the batch axis
            init_means, init_covariances, init_weights = self._batched_init(init_means, init_covariances,
                                                                            init_weights)
        self._require_engine()
        torch.manual_seed(self.seed)
        torch.cuda.manual_seed_all(self.seed)
        kw = dict(max_iters=self.niter, tol=self.tol, init_means=init_means, init_variances=init_covariances,
                  init_weights=init_weights, init_params=self.init_params, reg_covar=self.reg_covar,
                  compute_labels=self.compute_labels_on_fit, verbose=self.verbose, approx_top_k=self.approx_top_k,
                  kmeans_init_iters=self.init_kmeans_iters, kmeans_init_tol=self.init_kmeans_tol)
        if self._is_large_cpu_stream_input(x_b):
            if batch_size is not None and x_b.shape[0] != 1:
                raise ValueError("large-N CPU streaming supports batch size 1")
            xs = x_b if self.dtype is None else x_b.to(self.dtype)
            labels_b, means_b, cov_b, w_b, info = large_n.em_fit_streamed(
                self.covariance_type, xs, self.k, device=self.device, chunk_rows=self.chunk_size_data_cpu, **kw)
        else:
            x_dev = self._prepare_compute_tensor(x_b)
            labels_b, means_b, cov_b, w_b, info = engine.em_fit(self.covariance_type, x_dev, self.k, **kw)
        self._set_fit_result(labels_b=labels_b, means_b=means_b, variances_b=cov_b, weights_b=w_b, info=info,
                             batch_size=batch_size)
        return self

    def _batched_init(self, init_means, init_covariances, init_weights):
        """Initial parameters of an unbatched fit in the engine's (1, ...) shapes:
        means (K, D), covariances (K,) / (K, D) / (D, D) / (K, D, D) by type and
        weights (K,) gain the batch axis; tensors that already have it pass."""
        cov_ndim = {"spherical": 1, "diag": 2, "tied": 2, "full": 3}[self.covariance_type]

        def add(t, ndim):
            return t.unsqueeze(0) if torch.is_tensor(t) and t.ndim == ndim else t

        return add(init_means, 2), add(init_covariances, cov_ndim), add(init_weights, 1)

    def fit(self, data, y: Any = None, **init):
        del y
        return self.train(data, **init)

    def fit_predict(self, data, y: Any = None):
        del y
        self.train(data)
        if self.cluster_ids_b is None:
            labels = self.predict(data)
            self.cluster_ids_b = labels.unsqueeze(0) if self._batch_size is None else labels
            self.labels_ = labels
            return labels
        return self.cluster_ids_b.squeeze(0) if self._batch_size is None else self.cluster_ids_b

    # --- inference -------------------------------------------------------------

    def _require_trained(self) -> None:
        if self.means_b is None or self.variances_b is None or self.weights_b is None:
            raise RuntimeError("Model not trained. Call train() or fit() first.")

    def _infer(self, kind, data):
        self._require_trained()
        x_b, batch_size = self._normalize_input(data)
        if batch_size != self._batch_size:
            raise ValueError(f"Model was trained with batch size B={self._batch_size}, but received B={batch_size}.")
        self._require_engine()
        if self._is_large_cpu_stream_input(x_b):
            out = large_n.predict_streamed(kind, self.covariance_type, x_b, self.means_b, self.variances_b,
                                           self.weights_b, device=self.device, chunk_rows=self.chunk_size_data_cpu)
        else:
            fn = {"assign": engine.assign, "score_samples": engine.score_samples,
                  "predict_proba": engine.predict_proba}[kind]
            out = fn(self.covariance_type, self._prepare_compute_tensor(x_b), self.means_b, self.variances_b,
                     self.weights_b)
        self.last_backend_used_ = "cuda"
        return out.squeeze(0) if batch_size is None else out

    def predict(self, data) -> torch.Tensor:
        return self._infer("assign", data)

    def predict_proba(self, data) -> torch.Tensor:
        return self._infer("predict_proba", data)

    def score_samples(self, data) -> torch.Tensor:
        return self._infer("score_samples", data)

    def score(self, data, y: Any = None) -> float:
        del y
        return float(self.score_samples(data).mean().item())

    def _n_parameters(self, batch_size: int = 1) -> int:
        self._require_trained()
        d = int(self.means_b.shape[-1])
        k = int(self.means_b.shape[1])
        covariance_params = {"spherical": k, "diag": k * d, "tied": d * (d + 1) // 2,
                             "full": k * d * (d + 1) // 2}[self.covariance_type]
        return int(batch_size * (k * d + covariance_params + k - 1))

    def bic(self, data) -> float:
        scores = self.score_samples(data)
        n_samples = int(scores.numel())
        batch_size = int(scores.shape[0]) if scores.ndim == 2 else 1
        return float(-2.0 * scores.sum().item() + self._n_parameters(batch_size) * math.log(float(n_samples)))

    def aic(self, data) -> float:
        scores = self.score_samples(data)
        batch_size = int(scores.shape[0]) if scores.ndim == 2 else 1
        return float(-2.0 * scores.sum().item() + 2.0 * self._n_parameters(batch_size))

    # --- sklearn-style params ---------------------------------------------------

    def get_params(self, deep: bool = True) -> dict:
        del deep
        return {
            "d": self.d, "n_components": self.k, "max_iter": self.niter, "tol": self.tol,
            "random_state": self.seed, "chunk_size_data": self.chunk_size_data,
            "chunk_size_centroids": self.chunk_size_centroids, "chunk_size_data_cpu": self.chunk_size_data_cpu,
            "verbose": self.verbose, "dtype": self.dtype, "device": self.device, "init_params": self.init_params,
            "reg_covar": self.reg_covar, "init_kmeans_iters": self.init_kmeans_iters,
            "init_kmeans_tol": self.init_kmeans_tol, "covariance_type": self.covariance_type,
            "matmul_precision": self.matmul_precision, "compute_labels_on_fit": self.compute_labels_on_fit,
            "approx_top_k": self.approx_top_k, "backend": self.backend,
        }

    def set_params(self, **params):
        if not params:
            return self
        valid = set(self.get_params().keys()) | {"k", "niter", "seed", "n_features", "n_components", "max_iter",
                                                  "random_state", "use_triton", "backend"}
        for raw_name, value in params.items():
            if raw_name not in valid:
                raise ValueError(f"Invalid parameter {raw_name!r} for GMMXX")
            name = _SKLEARN_PARAM_ALIASES.get(raw_name, raw_name)
            if name == "d":
                value = _optional_positive_int(value, "d")
            elif name in {"k", "niter", "chunk_size_data", "chunk_size_centroids", "chunk_size_data_cpu",
                          "init_kmeans_iters"}:
                value = _positive_int(value, name)
            elif name in {"tol", "reg_covar", "init_kmeans_tol"}:
                value = float(value)
                if value < 0.0:
                    raise ValueError(f"{name} must be non-negative")
            elif name == "seed":
                value = int(value)
            elif name == "use_triton":
                if value is not None:
                    if self.backend != "auto":
                        raise ValueError("Cannot set use_triton when backend is already explicit")
                    warnings.warn("use_triton is deprecated", DeprecationWarning, stacklevel=2)
                    self._legacy_no_triton = not bool(value)
                continue
            elif name == "backend":
                if value not in _VALID_BACKENDS:
                    raise ValueError(f"backend must be one of {_VALID_BACKENDS}, got {value!r}")
                self.backend = value
                continue
            elif name in {"verbose", "compute_labels_on_fit"}:
                value = bool(value)
            elif name == "covariance_type":
                value = _normalize_covariance_type(value)
            elif name == "matmul_precision" and value is not None and value not in {"highest", "high", "medium"}:
                raise ValueError("matmul_precision must be None, 'highest', 'high', or 'medium'")
            elif name == "approx_top_k":
                value = _optional_positive_int(value, "approx_top_k")
            elif name == "device":
                value = torch.device(value)
                self._raw_device = value
            setattr(self, name, value)
        self._reset_fit_state()
        return self

    # --- save / load ------------------------------------------------------------

    _STATE_FORMAT = "gmmxx_b200.GMMXX"
    _STATE_VERSION = 1

    def state_dict(self) -> dict:
        """The fitted model as plain Python values and CPU tensors.

        The reference keeps a fit only in memory (its fitted attributes are
        set in gmmxx/interface.py:369-396 and nothing writes them out); this is
        an addition.  The dict holds the constructor parameters, the batched
        parameters (``means`` (B, K, D), ``covariances`` in the layout of the
        covariance type, ``weights`` (B, K)), the fit labels when they were
        computed and the fit record (``lower_bound``, history, iteration
        count, init source).  ``torch.save`` writes it and
        ``torch.load(..., weights_only=True)`` reads it back.
        """
        self._require_trained()
        params = self.get_params()
        params["dtype"] = None if self.dtype is None else str(self.dtype).split(".")[-1]
        params["device"] = str(self.device)
        cpu = lambda t: None if t is None else t.detach().to("cpu").clone()
        return {
            "format": self._STATE_FORMAT,
            "version": self._STATE_VERSION,
            "params": params,
            "batch_size": self._batch_size,
            "means": cpu(self.means_b),
            "covariances": cpu(self.variances_b),
            "weights": cpu(self.weights_b),
            "labels": cpu(self.cluster_ids_b),
            "fit_info": dict(self.fit_info_ or {}),
        }

    def load_state_dict(self, state: dict) -> "GMMXX":
        """Restore a model written by :meth:`state_dict`.  The constructor
        parameters are taken from the state except ``device``, which stays the
        one this estimator was built with; the parameter tensors move there.
        Raises ``ValueError`` on a state of another format or version, or whose
        tensors do not have the shapes its covariance type needs."""
        if not isinstance(state, dict) or state.get("format") != self._STATE_FORMAT:
            raise ValueError("not a gmmxx_b200.GMMXX state")
        if state.get("version") != self._STATE_VERSION:
            raise ValueError(f"unsupported GMMXX state version {state.get('version')!r}")
        params = dict(state["params"])
        params.pop("device", None)
        if params.get("dtype") is not None:
            params["dtype"] = getattr(torch, params["dtype"])
        backend = params.pop("backend", "auto")
        means, cov, weights, labels = state["means"], state["covariances"], state["weights"], state["labels"]
        batch_size = state["batch_size"]
        for name, t in (("means", means), ("covariances", cov), ("weights", weights)):
            if not torch.is_tensor(t) or not t.dtype.is_floating_point:
                raise ValueError(f"state entry {name!r} must be a floating point tensor")
        if means.ndim != 3:
            raise ValueError("state means must have shape (B, K, D)")
        b, k, d = means.shape
        if (batch_size is None and b != 1) or (batch_size is not None and batch_size != b):
            raise ValueError("state batch_size does not match the parameter tensors")
        cov_type = _normalize_covariance_type(params["covariance_type"])
        shapes = {"spherical": (b, k), "diag": (b, k, d), "tied": (b, d, d), "full": (b, k, d, d)}
        if tuple(cov.shape) != shapes[cov_type]:
            raise ValueError(f"state covariances must have shape {shapes[cov_type]} for {cov_type} covariance")
        if tuple(weights.shape) != (b, k):
            raise ValueError(f"state weights must have shape {(b, k)}")
        if labels is not None and (not torch.is_tensor(labels) or labels.ndim != 2 or labels.shape[0] != b):
            raise ValueError("state labels must have shape (B, N)")
        if params.get("n_components") != k or params.get("d") not in (None, d):
            raise ValueError("state parameters do not match the parameter tensors")
        self.set_params(backend=backend, **params)
        info = dict(state.get("fit_info") or {})
        for key in ("lower_bound", "lower_bound_history", "n_iter", "init_source"):
            if key not in info:
                raise ValueError(f"state fit_info lacks {key!r}")
        dev = lambda t: t.to(device=self.device, dtype=torch.float32).contiguous()
        self._set_fit_result(labels_b=None if labels is None else labels.to(self.device, torch.int64),
                             means_b=dev(means), variances_b=dev(cov), weights_b=dev(weights), info=info,
                             batch_size=batch_size)
        self.d = d
        return self

    def save(self, path) -> None:
        """Write :meth:`state_dict` to ``path`` with ``torch.save``."""
        torch.save(self.state_dict(), path)

    @classmethod
    def load(cls, path, device: Optional[torch.device] = None) -> "GMMXX":
        """Read a model written by :meth:`save`; ``device`` (default: the one it
        was fitted on) is where its parameters are placed."""
        state = torch.load(path, map_location="cpu", weights_only=True)
        if not isinstance(state, dict) or "params" not in state:
            raise ValueError("not a gmmxx_b200.GMMXX state")
        params = state["params"]
        model = cls(k=params["n_components"], device=params["device"] if device is None else device)
        return model.load_state_dict(state)
