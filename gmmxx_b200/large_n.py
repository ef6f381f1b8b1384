"""Host-resident X streamed through the GPU every EM iteration.

Rebuild of the reference's large-N driver (gmmxx/large_n.py:866-1594,
prefetcher 502-627): X stays in (pinned) host memory; each iteration streams
it through two device chunk buffers on a copy stream while the compute stream
runs ``gmmxx_em_accumulate`` on the previous chunk.  Statistics accumulate on
the device across chunks, so the host never synchronises inside an iteration
(the reference syncs once per chunk, large_n.py:313).  Like the reference it
handles B == 1.
"""

from __future__ import annotations

import os
import time
from typing import Optional

import torch

from . import _native as nat
from . import engine


class ChunkStreamer:
    """Double-buffered host -> device row chunks (copy stream + events)."""

    def __init__(self, x_host: torch.Tensor, chunk_rows: int, device: torch.device):
        if x_host.ndim != 3 or x_host.shape[0] != 1:
            raise ValueError("host streaming takes x of shape (1, N, D)")
        if x_host.is_cuda:
            raise ValueError("x_host must be in host memory")
        self.x = x_host.contiguous()
        if not self.x.is_pinned():
            self.x = self.x.pin_memory()
        self.n, self.d = self.x.shape[1], self.x.shape[2]
        self.chunk = max(1, min(int(chunk_rows), self.n))
        self.device = device
        self.bufs = [torch.empty((1, self.chunk, self.d), dtype=self.x.dtype, device=device) for _ in range(2)]
        self.copy_stream = torch.cuda.Stream(device=device)
        self.copied = [torch.cuda.Event() for _ in range(2)]
        self.free = [torch.cuda.Event() for _ in range(2)]
        self.h2d_bytes = 0

    def chunks(self):
        """Yield (device view (1, rows, D), row offset); the caller's compute
        stream must not outrun the yielded chunk's copy (handled here)."""
        compute = torch.cuda.current_stream(self.device)
        starts = list(range(0, self.n, self.chunk))
        for ci, n0 in enumerate(starts):
            slot = ci & 1
            n1 = min(n0 + self.chunk, self.n)
            with torch.cuda.stream(self.copy_stream):
                if ci >= 2:
                    self.copy_stream.wait_event(self.free[slot])
                dst = self.bufs[slot][:, : n1 - n0]
                dst.copy_(self.x[:, n0:n1], non_blocking=True)
                self.h2d_bytes += dst.numel() * dst.element_size()
                self.copied[slot].record(self.copy_stream)
            compute.wait_event(self.copied[slot])
            yield dst, n0
            self.free[slot].record(compute)


def em_fit_streamed(
    cov_type: str,
    x_host: torch.Tensor,
    n_components: int,
    *,
    device: torch.device,
    chunk_rows: int = 1 << 20,
    max_iters: int = 100,
    tol: float = 1e-4,
    init_means: Optional[torch.Tensor] = None,
    init_variances: Optional[torch.Tensor] = None,
    init_weights: Optional[torch.Tensor] = None,
    init_params: str = "kmeans",
    reg_covar: float = 1e-6,
    min_weight: float = engine.MIN_WEIGHT_DEFAULT,
    compute_labels: bool = True,
    verbose: bool = False,
    streamer: Optional[ChunkStreamer] = None,
    approx_top_k: Optional[int] = None,
):
    """Soft EM over host-resident X (B == 1), streamed chunk by chunk;
    ``approx_top_k`` as in engine.em_fit (the reference's large-N driver takes
    the same option, large_n.py:887-1005)."""
    covc = engine.cov_code(cov_type)
    device = torch.device(device)
    if x_host.dtype not in engine._X_DTYPES:
        raise TypeError(f"x dtype {x_host.dtype} not supported")
    b, n, d = x_host.shape
    engine.check_window(cov_type, d)
    if n == 0:
        raise ValueError("x must contain at least one sample")
    with torch.cuda.device(device):
        st = streamer or ChunkStreamer(x_host, chunk_rows, device)
        if init_means is None:
            if init_params not in {"kmeans", "random"}:
                raise ValueError("init_params must be 'kmeans' or 'random'")
            idx = torch.randint(0, n, (1, n_components))
            init_means = torch.gather(st.x, 1, idx[..., None].expand(-1, -1, d)).float()
        # initial covariance from the full data when not given
        if init_variances is None:
            sample = st.x[:, :: max(1, n // (1 << 20))].to(device)
            init_variances = engine.global_covariance(cov_type, sample, init_means.shape[1], reg_covar)
        probe = st.bufs[0][:, :1]
        means, cov, weights, source = engine.initial_parameters(
            cov_type, probe, n_components, init_means, init_variances, init_weights, reg_covar, init_params)
        k = means.shape[1]
        top_k = engine.resolve_approx_top_k(approx_top_k, k)
        scratch = None
        if top_k is not None:
            scratch = torch.empty(nat.topk_scratch_bytes(1, st.chunk, top_k), dtype=torch.uint8, device=device)
        stream = engine._stream_ptr(device)
        f = nat.stat_width(covc, d)
        ws = engine._WS.get(device, nat.workspace_bytes(covc, 1, st.chunk, d, k))
        stats = torch.zeros((1, k, f), dtype=torch.float32, device=device)
        ll = torch.zeros((1,), dtype=torch.float64, device=device)
        lb_hist = torch.zeros((max_iters,), dtype=torch.float32, device=device)
        xdt = engine._X_DTYPES[x_host.dtype]
        xx = None
        if covc == nat.TIED:
            xx = torch.zeros((1, d, d), dtype=torch.float32, device=device)
            for xc, _ in st.chunks():
                nat.call("gmmxx_xx_total", xdt, xc.data_ptr(), 1, xc.shape[1], d, xx.data_ptr(), ws.data_ptr(),
                         ws.numel(), stream)
        prev = None
        it = 0
        t0 = time.perf_counter()
        for it in range(max_iters):
            nat.call("gmmxx_em_prepare", covc, 1, d, k, means.data_ptr(), cov.data_ptr(), weights.data_ptr(),
                     float(reg_covar), float(min_weight), ws.data_ptr(), ws.numel(), stream)
            stats.zero_()
            ll.zero_()
            for xc, _ in st.chunks():
                if top_k is not None:
                    nat.call("gmmxx_em_accumulate_topk", covc, xdt, xc.data_ptr(), 1, xc.shape[1], d, k, top_k,
                             ws.data_ptr(), ws.numel(), scratch.data_ptr(), scratch.numel(), stats.data_ptr(),
                             ll.data_ptr(), stream)
                    continue
                nat.call("gmmxx_em_accumulate", covc, xdt, xc.data_ptr(), 1, xc.shape[1], d, k, ws.data_ptr(),
                         ws.numel(), stats.data_ptr(), ll.data_ptr(), stream)
            if verbose:
                prev_means = means.clone()
            nat.call("gmmxx_em_finalize", covc, 1, d, k, n, stats.data_ptr(), ll.data_ptr(), engine._p(xx),
                     float(reg_covar), float(min_weight), means.data_ptr(), cov.data_ptr(), weights.data_ptr(),
                     lb_hist[it:].data_ptr(), stream)
            if verbose or tol > 0.0:
                lb = float(lb_hist[it].item())
                if verbose:
                    print(engine.verbose_line(cov_type, it, lb, means, prev_means))
                if tol > 0.0 and prev is not None and it + 1 < max_iters and abs(lb - prev) < tol:
                    break
                prev = lb
        elapsed = time.perf_counter() - t0
        n_iter = it + 1
        hist = lb_hist[:n_iter].tolist()
        if cov_type != "spherical" and not (tol > 0.0 or verbose):
            hist = [0.0] * (n_iter - 1) + [hist[-1]]
        labels = None
        if compute_labels:
            labels = torch.empty((1, n), dtype=torch.int64, device=device)
            for xc, n0 in st.chunks():
                labels[:, n0:n0 + xc.shape[1]] = engine.assign(cov_type, xc, means, cov, weights)
    info = {
        "n_iter": n_iter,
        "lower_bound": hist[-1],
        "lower_bound_history": hist,
        "init_source": source,
        "triton_estep_enabled": False,
        "triton_fused_update_enabled": False,
        "triton_streaming_update_enabled": False,
        "approximate_em_enabled": top_k is not None,
        "approx_top_k": top_k,
        "cuda_approx_topk_enabled": top_k is not None,
        "large_n_streaming_enabled": True,
        "copy_stream_prefetch_enabled": True,
        "cuda_engine": "gmmxx_b200",
        "backend_breakdown": {"cuda": n_iter},
        "ms_per_iter": 1e3 * elapsed / n_iter,
    }
    return labels, means, cov, weights, info


def predict_streamed(kind: str, cov_type: str, x_host: torch.Tensor, means, cov, weights, *, device,
                     chunk_rows: int = 1 << 20):
    """Chunked inference over host-resident X (reference: large_n.py:1907-2502).
    ``kind`` is "assign", "score_samples" or "predict_proba"; results are
    returned on the device."""
    device = torch.device(device)
    fn = {"assign": engine.assign, "score_samples": engine.score_samples,
          "predict_proba": engine.predict_proba}[kind]
    with torch.cuda.device(device):
        st = ChunkStreamer(x_host, chunk_rows, device)
        outs = []
        for xc, _ in st.chunks():
            outs.append(fn(cov_type, xc, means, cov, weights))
        return torch.cat(outs, dim=1)


# ---------------------------------------------------------------------------
# the reference's large-N entry points (gmmxx/large_n.py:866-1594, 1907-2502)
# ---------------------------------------------------------------------------

_COV_TYPES = ("spherical", "diag", "tied", "full")


def _validate_large_n_input(x_cpu: torch.Tensor, device) -> torch.device:
    """The reference's input contract (large_n.py:468-478): (1, N, D) floating
    point in host memory, a CUDA target device."""
    device = torch.device(device)
    if x_cpu.ndim != 3:
        raise ValueError("x must have shape (B, N, D)")
    if x_cpu.shape[0] != 1:
        raise NotImplementedError("Large-N CPU streaming currently supports only B=1")
    if x_cpu.device.type != "cpu":
        raise ValueError("Large-N streaming expects a CPU input tensor")
    if device.type != "cuda":
        raise ValueError("Large-N streaming expects a CUDA target device")
    if not x_cpu.dtype.is_floating_point:
        raise TypeError("GMM input must be a floating point tensor")
    return device


def _check_backend(backend: str) -> None:
    """backend (with GMMXX_BACKEND consulted for "auto") must resolve to this
    engine; the reference's torch and Triton backends are not provided."""
    valid = ("auto", "cuda", "triton", "torch")
    if backend not in valid:
        raise ValueError(f"backend must be one of {valid}, got {backend!r}")
    effective = backend
    if backend == "auto" and os.environ.get("GMMXX_BACKEND") in valid:
        effective = os.environ["GMMXX_BACKEND"]
    if effective in ("torch", "triton"):
        raise ValueError(f"backend={effective!r} is not provided by gmmxx_b200; this engine implements the CUDA "
                         "backend (use backend='cuda' or 'auto')")


def _compute_input(x_cpu: torch.Tensor, dtype: Optional[torch.dtype]) -> torch.Tensor:
    """X in the dtype the reference computes in (its chunks are converted to
    ``dtype`` on the device).  bf16 / fp16 X with an fp32 compute dtype is read
    as stored (the conversion is exact); a conversion that rounds (fp32 to a
    16-bit type, between the 16-bit types, float64 to fp32) is applied once on
    the host."""
    target = x_cpu.dtype if dtype is None else dtype
    if target not in engine._X_DTYPES:
        raise TypeError(f"compute dtype {target} not supported (float32, bfloat16, float16)")
    if target == x_cpu.dtype or (target == torch.float32 and x_cpu.dtype in (torch.bfloat16, torch.float16)):
        return x_cpu
    return x_cpu.to(target)


def batch_gmm_largeN_cpu(
    x_cpu: torch.Tensor,
    n_components: int,
    *,
    covariance_type: str,
    device: torch.device,
    dtype: torch.dtype,
    max_iters: int = 100,
    tol: float = 1e-4,
    verbose: bool = False,
    init_params: str = "kmeans",
    reg_covar: float = 1e-6,
    chunk_size_N: int = 32768,
    chunk_size_K: int = 1024,
    kmeans_init_iters: int = 10,
    kmeans_init_tol: float = 1e-4,
    kmeans_use_triton: bool = True,
    gmm_use_triton="auto",
    min_weight: float = 1e-8,
    compute_labels: bool = True,
    max_init_samples: int = 65536,
    approx_top_k: Optional[int] = None,
    backend: str = "auto",
    legacy_no_triton: bool = False,
    seed: int = 0,
):
    """Soft EM over host-resident X with the reference's signature and return
    value (large_n.py:866-1594): ``(labels (1, N) int64 on the host or None,
    means, covariances, weights, info)``.  Rows stream through the GPU in
    ``chunk_size_N``-row chunks (em_fit_streamed).  ``chunk_size_K``, the
    k-means and Triton arguments and ``max_init_samples`` steer only the
    reference's own kernels and initialisation and are validated, not needed;
    initial means are ``n_components`` rows drawn with ``seed`` (the
    reference's fallback when flash_kmeans is absent)."""
    del kmeans_init_iters, kmeans_init_tol, kmeans_use_triton, gmm_use_triton, max_init_samples, legacy_no_triton
    device = _validate_large_n_input(x_cpu, device)
    if covariance_type not in _COV_TYPES:
        raise ValueError("covariance_type must be 'spherical', 'diag', 'tied', or 'full'")
    if n_components <= 0:
        raise ValueError("n_components must be positive")
    if max_iters <= 0:
        raise ValueError("max_iters must be positive")
    if chunk_size_N <= 0 or chunk_size_K <= 0:
        raise ValueError("chunk_size_N and chunk_size_K must be positive")
    if min_weight <= 0.0:
        raise ValueError("min_weight must be positive")
    _check_backend(backend)
    x = _compute_input(x_cpu, dtype)
    torch.manual_seed(seed)
    labels, means, cov, weights, info = em_fit_streamed(
        covariance_type, x, int(n_components), device=device, chunk_rows=int(chunk_size_N), max_iters=max_iters,
        tol=tol, init_params=init_params, reg_covar=reg_covar, min_weight=min_weight,
        compute_labels=compute_labels, verbose=verbose, approx_top_k=approx_top_k)
    info = dict(info, fallback_reason=None)
    return (None if labels is None else labels.cpu()), means, cov, weights, info


def _predict_to_host(kind: str, x_cpu, means, variances, weights, covariance_type, device, dtype, chunk_size_N,
                     chunk_size_K, backend):
    device = _validate_large_n_input(x_cpu, device)
    if covariance_type not in _COV_TYPES:
        raise ValueError("covariance_type must be 'spherical', 'diag', 'tied', or 'full'")
    if chunk_size_N <= 0 or chunk_size_K <= 0:
        raise ValueError("chunk_size_N and chunk_size_K must be positive")
    _check_backend(backend)
    x = _compute_input(x_cpu, dtype)
    n, k = x.shape[1], means.shape[1]
    fn = {"assign": engine.assign, "score_samples": engine.score_samples,
          "predict_proba": engine.predict_proba}[kind]
    shape, out_dtype = {"assign": ((1, n), torch.int64), "score_samples": ((1, n), torch.float32),
                        "predict_proba": ((1, n, k), torch.float32)}[kind]
    out = torch.empty(shape, dtype=out_dtype)
    with torch.cuda.device(device):
        st = ChunkStreamer(x, int(chunk_size_N), device)
        for xc, n0 in st.chunks():
            out[:, n0:n0 + xc.shape[1]] = fn(covariance_type, xc, means, variances, weights).cpu()
    return out


def large_n_predict_cpu(x_cpu, means, variances, weights, *, covariance_type: str, device, dtype, chunk_size_N: int,
                        chunk_size_K: int, use_triton: bool = True, return_triton_used: bool = False,
                        return_backend_used: bool = False, backend: str = "auto", legacy_no_triton: bool = False):
    """Labels (1, N) int64 on the host for host-resident X (the reference's
    large_n.py:1907-2075); with ``return_backend_used`` also "cuda", with
    ``return_triton_used`` also False."""
    del use_triton, legacy_no_triton
    labels = _predict_to_host("assign", x_cpu, means, variances, weights, covariance_type, device, dtype,
                              chunk_size_N, chunk_size_K, backend)
    if return_backend_used:
        return labels, "cuda"
    if return_triton_used:
        return labels, False
    return labels


def large_n_score_samples_cpu(x_cpu, means, variances, weights, *, covariance_type: str, device, dtype,
                              chunk_size_N: int, chunk_size_K: int, use_triton: bool = True, backend: str = "auto",
                              legacy_no_triton: bool = False, return_backend_used: bool = False):
    """Per-row log-likelihood (1, N) fp32 on the host (the reference's
    large_n.py:2078-2256)."""
    del use_triton, legacy_no_triton
    scores = _predict_to_host("score_samples", x_cpu, means, variances, weights, covariance_type, device, dtype,
                              chunk_size_N, chunk_size_K, backend)
    return (scores, "cuda") if return_backend_used else scores


def large_n_predict_proba_cpu(x_cpu, means, variances, weights, *, covariance_type: str, device, dtype,
                              chunk_size_N: int, chunk_size_K: int, use_triton: bool = True, backend: str = "auto",
                              legacy_no_triton: bool = False, return_backend_used: bool = False):
    """Responsibilities (1, N, K) fp32 on the host (the reference's
    large_n.py:2259-2502)."""
    del use_triton, legacy_no_triton
    probs = _predict_to_host("predict_proba", x_cpu, means, variances, weights, covariance_type, device, dtype,
                             chunk_size_N, chunk_size_K, backend)
    return (probs, "cuda") if return_backend_used else probs
