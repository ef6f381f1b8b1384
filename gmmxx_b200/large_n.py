"""Host-resident X streamed through the GPU every EM iteration.

Rebuild of the reference's large-N driver (gmmxx/large_n.py:866-1594,
prefetcher 502-627): X stays in host memory; each iteration streams it
through two device chunk buffers on a copy stream while the compute stream
runs ``gmmxx_em_accumulate`` on the previous chunk.  Statistics accumulate on
the device across chunks, so the host never synchronises inside an iteration
(the reference syncs once per chunk, large_n.py:313).  Pinned X is copied to
the device straight from its rows; pageable X goes through two pinned staging
chunks, so the extra host memory is two chunks, not a second copy of X (the
reference's prefetcher stages the same way, large_n.py:502-573).

With ``comm`` every rank streams its own row shard and the iteration's
statistics are sum-allreduced, exactly as ``engine.em_fit`` does for
device-resident shards (one collective per iteration).  Like the reference it
handles B == 1.
"""

from __future__ import annotations

import contextlib
import os
from typing import Optional

import torch

from . import _native as nat
from . import engine


class ChunkStreamer:
    """Double-buffered host -> device row chunks (copy stream + events).

    Every device buffer is refilled only after the compute stream has
    finished with the chunk it last held, including a chunk yielded by an
    earlier ``chunks()`` pass (the 'free' events carry over between passes).
    For pageable X the rows are first copied on the host into one of two
    pinned staging chunks; a staging chunk is refilled only after its previous
    host -> device copy has completed (the host waits on that copy's event),
    so the host copy of one chunk overlaps the device work of the other."""

    def __init__(self, x_host: torch.Tensor, chunk_rows: int, device: torch.device):
        if x_host.ndim != 3 or x_host.shape[0] != 1:
            raise ValueError("host streaming takes x of shape (1, N, D)")
        if x_host.is_cuda:
            raise ValueError("x_host must be in host memory")
        self.x = x_host.contiguous()
        self.pinned = self.x.is_pinned()
        self.n, self.d = self.x.shape[1], self.x.shape[2]
        self.chunk = max(1, min(int(chunk_rows), self.n))
        self.device = device
        self.bufs = [torch.empty((1, self.chunk, self.d), dtype=self.x.dtype, device=device) for _ in range(2)]
        self.stage = None
        if not self.pinned:
            self.stage = [torch.empty((1, self.chunk, self.d), dtype=self.x.dtype, pin_memory=True) for _ in range(2)]
        self.copy_stream = torch.cuda.Stream(device=device)
        self.copied = [torch.cuda.Event() for _ in range(2)]
        self.free = [torch.cuda.Event() for _ in range(2)]
        self.free_recorded = [False, False]  # free[slot] was recorded at least once (any pass)
        self.h2d_pending = [False, False]    # staging chunk slot has a copy that may be in flight
        self.h2d_bytes = 0

    def chunks(self):
        """Yield (device view (1, rows, D), row offset).  The compute stream
        waits for each chunk's copy before the caller's work on it; the chunk's
        buffer is released when the caller asks for the next one (or leaves
        the loop)."""
        compute = torch.cuda.current_stream(self.device)
        for ci, n0 in enumerate(range(0, self.n, self.chunk)):
            slot = ci & 1
            n1 = min(n0 + self.chunk, self.n)
            src = self.x[:, n0:n1]
            if self.stage is not None:
                if self.h2d_pending[slot]:
                    self.copied[slot].synchronize()  # the staging chunk's previous copy has landed
                staged = self.stage[slot][:, : n1 - n0]
                staged.copy_(src)
                src = staged
            with torch.cuda.stream(self.copy_stream):
                if self.free_recorded[slot]:
                    self.copy_stream.wait_event(self.free[slot])
                dst = self.bufs[slot][:, : n1 - n0]
                dst.copy_(src, non_blocking=True)
                self.h2d_bytes += dst.numel() * dst.element_size()
                self.copied[slot].record(self.copy_stream)
            self.h2d_pending[slot] = True
            compute.wait_event(self.copied[slot])
            try:
                yield dst, n0
            finally:
                self.free[slot].record(compute)
                self.free_recorded[slot] = True


class StreamedOps(engine.CudaOps):
    """The four per-iteration kernels of ``engine.em_loop`` over host-resident
    rows: ``xx_total`` and ``accumulate`` stream this rank's rows chunk by
    chunk; ``prepare``, ``finalize`` and the status check are those of
    device-resident X (``engine.CudaOps``)."""

    def __init__(self, cov_type: str, streamer: ChunkStreamer, k: int, top_k: Optional[int] = None):
        self.cov_type = cov_type
        self.covc = engine.cov_code(cov_type)
        self.st = streamer
        self.b, self.n, self.d = 1, streamer.n, streamer.d
        self.k = k
        self.xdt = engine._X_DTYPES[streamer.x.dtype]
        self.device = streamer.device
        self.stream = engine._stream_ptr(streamer.device)
        self.stat_width = nat.stat_width(self.covc, self.d)
        self.ws = engine._WS.get(streamer.device, nat.workspace_bytes(self.covc, 1, streamer.chunk, self.d, k))
        self.top_k = top_k
        self.paths = set()
        self.scratch = None
        if top_k is not None:
            self.scratch = torch.empty(nat.topk_scratch_bytes(1, streamer.chunk, top_k), dtype=torch.uint8,
                                       device=streamer.device)

    def xx_total(self, xx: torch.Tensor) -> None:
        for xc, _ in self.st.chunks():
            nat.call("gmmxx_xx_total", self.xdt, xc.data_ptr(), 1, xc.shape[1], self.d, xx.data_ptr(),
                     self.ws.data_ptr(), self.ws.numel(), self.stream)

    def accumulate(self, stats, ll) -> None:
        for xc, _ in self.st.chunks():
            n = xc.shape[1]
            if self.top_k is not None:
                nat.call("gmmxx_em_accumulate_topk", self.covc, self.xdt, xc.data_ptr(), 1, n, self.d, self.k,
                         self.top_k, self.ws.data_ptr(), self.ws.numel(), self.scratch.data_ptr(),
                         self.scratch.numel(), stats.data_ptr(), ll.data_ptr(), self.stream)
                continue
            nat.call("gmmxx_em_accumulate", self.covc, self.xdt, xc.data_ptr(), 1, n, self.d, self.k,
                     self.ws.data_ptr(), self.ws.numel(), stats.data_ptr(), ll.data_ptr(), self.stream)
            self.paths.add(nat.last_accumulate_path())


def select_init_sample(x_host: torch.Tensor, n_components: int, max_init_samples: int, device: torch.device):
    """The reference's initialisation sample of host rows (large_n.py:630-645):
    ``min(N, max(K, min(max_init_samples, max(4096, 64 K, K))))`` rows drawn with
    ``torch.randint`` (all rows when that is N), moved to ``device``.  Returns
    (sample (1, S, D), whether it is a strict subset)."""
    n = x_host.shape[1]
    target = max(4096, n_components * 64, n_components)
    sample_n = min(n, max(n_components, min(max_init_samples, target)))
    if sample_n == n:
        return x_host.to(device), False
    idx = torch.randint(0, n, (sample_n,), device=x_host.device)
    return x_host.index_select(1, idx).to(device), True


def _device_ctx(device: torch.device):
    return torch.cuda.device(device) if device.type == "cuda" else contextlib.nullcontext()


def _from_rank0(comm, make, shape, dtype, device) -> torch.Tensor:
    """``make()`` evaluated on rank 0 and broadcast (every rank the same
    initial parameter); without ``comm`` just ``make()``."""
    if comm is None:
        return make()
    t = make().to(device=device, dtype=dtype).contiguous() if comm.rank == 0 else \
        torch.zeros(shape, dtype=dtype, device=device)
    return comm.broadcast_(t, 0)


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
    comm: Optional[engine.Comm] = None,
    kmeans_init_iters: int = 10,
    kmeans_init_tol: float = 1e-4,
    max_init_samples: int = 65536,
):
    """Soft EM over host-resident X (B == 1), streamed chunk by chunk;
    ``approx_top_k`` as in engine.em_fit (the reference's large-N driver takes
    the same option, large_n.py:887-1005).

    Without ``init_means`` the initial parameters come from a random row sample
    moved to the device, as the reference's large-N driver draws them
    (large_n.py:630-725): ``sample_n = min(N, max(K, min(max_init_samples,
    max(4096, 64 K, K))))`` rows chosen with ``torch.randint``, then k-means or
    random initialisation on the sample (``init_source`` gets "_sampled" when
    the sample is a strict subset).

    With ``comm``, ``x_host`` is this rank's row shard: the fit is over the
    union of the shards (statistics allreduced once per iteration, the
    finalize replicated), initial parameters that are not given are drawn
    from rank 0's shard and broadcast, and the returned labels are the
    shard's."""
    engine.cov_code(cov_type)
    device = torch.device(device)
    if x_host.dtype not in engine._X_DTYPES:
        raise TypeError(f"x dtype {x_host.dtype} not supported")
    b, n, d = x_host.shape
    engine.check_window(cov_type, d)
    if max_iters <= 0:
        raise ValueError("max_iters must be positive")
    with _device_ctx(device):
        n_total = n
        if comm is not None:
            nt = torch.tensor([n], dtype=torch.int64, device=device)
            comm.allreduce_(nt)
            n_total = int(nt.item())
        if n_total == 0:
            raise ValueError("x must contain at least one sample")
        st = streamer or ChunkStreamer(x_host, chunk_rows, device)
        shape = lambda k: {"spherical": (1, k), "diag": (1, k, d), "tied": (1, d, d), "full": (1, k, d, d)}[cov_type]
        source = "user"
        if init_means is None:
            if init_params not in {"kmeans", "random"}:
                raise ValueError("init_params must be 'kmeans' or 'random'")
            sample, sampled = select_init_sample(st.x, n_components, max_init_samples, device)
            k = int(n_components)
            m0, c0, w0, source = engine.initial_parameters(
                cov_type, sample, k, None, init_variances, init_weights, reg_covar, init_params, kmeans_init_iters,
                kmeans_init_tol)
            source = source + ("_sampled" if sampled else "")
            init_means = _from_rank0(comm, lambda: m0, (1, k, d), torch.float32, device)
            init_variances = _from_rank0(comm, lambda: c0, shape(k), torch.float32, device)
            init_weights = _from_rank0(comm, lambda: w0, (1, k), torch.float32, device)
        k = init_means.shape[1]
        if init_variances is None:  # from a row sample of the (rank-0) data
            def gcov():
                sample = st.x[:, :: max(1, n // (1 << 20))].to(device)
                return engine.global_covariance(cov_type, sample, k, reg_covar)

            init_variances = _from_rank0(comm, gcov, shape(k), torch.float32, device)
        probe = st.bufs[0][:, :1]
        means, cov, weights, user = engine.initial_parameters(
            cov_type, probe, n_components, init_means, init_variances, init_weights, reg_covar, init_params)
        source = source if source != "user" else user
        top_k = engine.resolve_approx_top_k(approx_top_k, k)
        ops = StreamedOps(cov_type, st, k, top_k)
        n_iter, hist, elapsed = engine.em_loop(ops, cov_type, means, cov, weights, n_total=n_total,
                                               max_iters=max_iters, tol=tol, reg_covar=reg_covar,
                                               min_weight=min_weight, verbose=verbose, comm=comm)
        labels = None
        if compute_labels:
            labels = torch.empty((1, n), dtype=torch.int64, device=device)
            for xc, n0 in st.chunks():
                labels[:, n0:n0 + xc.shape[1]] = engine.assign(cov_type, xc, means, cov, weights)
    info = engine.fit_info(n_iter, hist, source, elapsed, gpus=1 if comm is None else comm.world_size,
                           approximate_em_enabled=top_k is not None, approx_top_k=top_k,
                           cuda_approx_topk_enabled=top_k is not None, large_n_streaming_enabled=True,
                           copy_stream_prefetch_enabled=True, kernel_path=ops.kernel_path())
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
    del kmeans_use_triton, gmm_use_triton, legacy_no_triton
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
        compute_labels=compute_labels, verbose=verbose, approx_top_k=approx_top_k,
        kmeans_init_iters=kmeans_init_iters, kmeans_init_tol=kmeans_init_tol, max_init_samples=max_init_samples)
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
