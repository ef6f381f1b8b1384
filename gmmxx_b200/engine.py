"""EM driver over the C ABI: parameter state, per-iteration orchestration,
optional N-sharding across ranks, and the inference entry points.

One soft-EM iteration is three C ABI calls on the current CUDA stream:

    gmmxx_em_prepare     prologue (clamp / renormalise) + component table
    gmmxx_em_accumulate  fused E-step + M-step statistics over the local rows
    [allreduce]          one collective of stats (B, K, F) and the
                         log-likelihood packed into one fp32 buffer, only
                         when the rows are sharded over several ranks
    gmmxx_em_finalize    M-step finalize, identical on every rank

so parameters stay bit-identical across ranks without a broadcast.  With
``approx_top_k`` the statistics call is ``gmmxx_em_accumulate_topk`` (each
row's responsibilities over its top_k components).  The loop never
synchronises the host unless ``tol > 0`` or ``verbose`` (as in the reference,
gmmxx/torch_fallback.py:2060-2330).

Semantics follow the reference's torch loops; see ``batch_gmm_*`` in
``gmmxx_b200.api`` for the public signatures.
"""

from __future__ import annotations

import math
import time
from typing import Dict, Optional, Tuple

import torch

from . import _native as nat

_X_DTYPES = {torch.float32: nat.FLOAT32, torch.bfloat16: nat.BFLOAT16, torch.float16: nat.FLOAT16}

MIN_WEIGHT_DEFAULT = 1e-8

# largest approx_top_k the engine's selection kernel keeps per row
MAX_APPROX_TOP_K = 64


def resolve_approx_top_k(approx_top_k: Optional[int], n_components: int) -> Optional[int]:
    """``approx_top_k`` as the EM loops use it (the reference's
    _resolve_approx_top_k, torch_fallback.py:599-607): None or >= K means exact
    EM, <= 0 is an error.  Values above MAX_APPROX_TOP_K (below K) are outside
    the engine's window."""
    if approx_top_k is None:
        return None
    top_k = int(approx_top_k)
    if top_k <= 0:
        raise ValueError("approx_top_k must be positive or None")
    if top_k >= n_components:
        return None
    if top_k > MAX_APPROX_TOP_K:
        raise nat.UnsupportedShape(nat.ERR_UNSUPPORTED,
                                   f"approx_top_k={top_k} exceeds the engine window (<= {MAX_APPROX_TOP_K})")
    return top_k


def cov_code(cov_type: str) -> int:
    try:
        return nat.COV_TYPES[cov_type]
    except KeyError:
        raise ValueError("covariance_type must be 'spherical', 'diag', 'tied' or 'full'") from None


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _p(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def check_x(x: torch.Tensor) -> torch.Tensor:
    if not torch.is_tensor(x):
        raise TypeError("x must be a torch.Tensor")
    if x.ndim != 3:
        raise ValueError("x must have shape (B, N, D)")
    if not x.is_cuda:
        raise ValueError(f"x must be on a CUDA device for the cuda engine, got {x.device}")
    if x.dtype not in _X_DTYPES:
        raise TypeError(f"x dtype {x.dtype} not supported (float32, bfloat16, float16)")
    return x.contiguous()


def check_window(cov_type: str, d: int) -> None:
    lim = nat.MAX_D_FULL if cov_type == "full" else nat.MAX_D
    if d > lim:
        raise nat.UnsupportedShape(nat.ERR_UNSUPPORTED, f"D={d} exceeds the engine window (D <= {lim} for {cov_type})")


class Workspace:
    """Per-device scratch buffer, grown on demand and reused across calls."""

    def __init__(self):
        self._buf: Dict[torch.device, torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        buf = self._buf.get(device)
        if buf is None or buf.numel() < nbytes:
            # zero-filled: the first word is the C ABI's sticky status word
            buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
            self._buf[device] = buf
        return buf


_WS = Workspace()


# ---------------------------------------------------------------------------
# initial parameters (reference: torch_fallback.py:1348-1894)
# ---------------------------------------------------------------------------


def _sym(m: torch.Tensor) -> torch.Tensor:
    return 0.5 * (m + m.transpose(-1, -2))


def global_covariance(cov_type: str, x: torch.Tensor, k: int, reg_covar: float) -> torch.Tensor:
    """torch_fallback.py:1348-1381 (_global_*_variance / covariance)."""
    xf = x.to(torch.float32)
    b, n, d = x.shape
    if cov_type == "spherical":
        mean = xf.mean(dim=1)
        second = xf.square().sum(dim=-1).mean(dim=1)
        gv = (second - mean.square().sum(dim=-1)).clamp_min(0.0) / float(d)
        return gv.clamp_min(reg_covar).unsqueeze(-1).expand(-1, k).clone()
    c = xf - xf.mean(dim=1, keepdim=True)
    if cov_type == "diag":
        return c.square().mean(dim=1).clamp_min(reg_covar).unsqueeze(1).expand(-1, k, -1).clone()
    cov = torch.bmm(c.transpose(1, 2), c) / float(n)
    cov = _sym(cov) + reg_covar * torch.eye(d, device=x.device, dtype=torch.float32)
    if cov_type == "tied":
        return cov
    return cov.unsqueeze(1).expand(-1, k, -1, -1).clone()


def initial_parameters(
    cov_type: str,
    x: torch.Tensor,
    k: int,
    init_means: Optional[torch.Tensor],
    init_cov: Optional[torch.Tensor],
    init_weights: Optional[torch.Tensor],
    reg_covar: float,
    init_params: str = "kmeans",
    kmeans_iters: int = 10,
    kmeans_tol: float = 1e-4,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, str]:
    """User init (clamp / renormalise as the reference does), k-means or
    random init (torch_fallback.py:1646-1894).

    ``init_params="kmeans"``: k-means++ seeds, ``kmeans_iters`` Lloyd
    iterations and the hard-label weights and covariances, all on the device
    (``gmmxx_b200.kmeans``; the reference's path with its flash-kmeans
    dependency, torch_fallback.py:1571-1623).  Where the reference's k-means++
    declines (K > 256 or K > its row sample) both draw random rows instead
    (_random_init_means, torch_fallback.py:1384-1387).
    """
    b, n, d = x.shape
    dev = x.device
    if init_means is not None:
        means = init_means.detach().to(device=dev, dtype=torch.float32).clone().contiguous()
        if means.ndim != 3:
            raise ValueError("init_means must have shape (B, K, D)")
        if means.shape[0] != b or means.shape[2] != d:
            raise ValueError("init_means must have shape (B, K, D) matching x")
        k = means.shape[1]
        source = "user"
    else:
        if init_params not in {"kmeans", "random"}:
            raise ValueError("init_params must be 'kmeans' or 'random'")
        km = None
        if init_params == "kmeans" and x.is_cuda:  # host rows (CPU test doubles) take the random draw
            from . import kmeans

            km = kmeans.kmeans_initialize(cov_type, x, k, max_iters=kmeans_iters, tol=kmeans_tol,
                                          reg_covar=reg_covar)
        if km is not None:
            means, init_cov, init_weights = km
            source = "kmeans"
        else:
            # _random_init_means (torch_fallback.py:1384-1387)
            idx = torch.randint(0, n, (b, k), device=dev)
            means = torch.gather(x, 1, idx[..., None].expand(-1, -1, d)).to(torch.float32).contiguous()
            source = "random"
            init_cov = None
            init_weights = None
    if init_weights is None:
        weights = torch.full((b, k), 1.0 / float(k), device=dev, dtype=torch.float32)
    else:
        weights = init_weights.detach().to(device=dev, dtype=torch.float32).clone()
        if weights.shape != (b, k):
            raise ValueError("init_weights must have shape (B, K)")
    if source == "user":
        weights = weights.clamp_min(1e-8)
        weights = weights / weights.sum(dim=-1, keepdim=True)
    if init_cov is None:
        cov = global_covariance(cov_type, x, k, reg_covar)
    else:
        cov = init_cov.detach().to(device=dev, dtype=torch.float32).clone()
    shapes = {"spherical": (b, k), "diag": (b, k, d), "tied": (b, d, d), "full": (b, k, d, d)}
    if tuple(cov.shape) != shapes[cov_type]:
        raise ValueError(f"init_variances must have shape {shapes[cov_type]} for {cov_type} covariance")
    if cov_type in ("spherical", "diag"):
        if source == "user":
            cov = cov.clamp_min(reg_covar)
    else:
        cov = _sym(cov)
    return means.contiguous(), cov.contiguous(), weights.contiguous(), source


# ---------------------------------------------------------------------------
# EM loop
# ---------------------------------------------------------------------------


class Comm:
    """Sum-allreduce over the ranks that share one fit (one per GPU)."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def allreduce_(self, t: torch.Tensor) -> torch.Tensor:
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM, group=self.group)
        return t

    def broadcast_(self, t: torch.Tensor, src: int = 0) -> torch.Tensor:
        """Rank ``src``'s tensor on every rank (``src`` is a rank of the group)."""
        self.dist.broadcast(t, src=self.dist.get_global_rank(self.group, src) if self.group is not None else src,
                            group=self.group)
        return t


def kernel_path_name(paths) -> str:
    """The statistics kernels a fit ran, from the gmmxx_last_accumulate_path
    values its accumulate calls reported (several when chunks differed)."""
    names = [nat.PATH_NAMES.get(p) for p in sorted(paths) if nat.PATH_NAMES.get(p)]
    return " + ".join(names) if names else "none"


class CudaOps:
    """The four per-iteration kernels of one fit, bound to one device buffer
    of rows.  ``em_loop`` drives any object with this interface."""

    def __init__(self, cov_type: str, x: torch.Tensor, k: int, top_k: Optional[int] = None):
        self.cov_type = cov_type
        self.covc = cov_code(cov_type)
        self.x = x
        self.b, self.n, self.d = x.shape
        self.k = k
        self.xdt = _X_DTYPES[x.dtype]
        self.device = x.device
        self.stream = _stream_ptr(x.device)
        self.stat_width = nat.stat_width(self.covc, self.d)
        self.ws = _WS.get(x.device, nat.workspace_bytes(self.covc, self.b, self.n, self.d, k))
        # approximate top-k EM: the per-row lists between its two passes
        self.top_k = top_k
        self.paths = set()  # gmmxx_last_accumulate_path after each exact-EM accumulate call
        self.scratch = None
        if top_k is not None:
            self.scratch = torch.empty(nat.topk_scratch_bytes(self.b, self.n, top_k), dtype=torch.uint8,
                                       device=x.device)

    def xx_total(self, xx: torch.Tensor) -> None:
        nat.call("gmmxx_xx_total", self.xdt, self.x.data_ptr(), self.b, self.n, self.d, xx.data_ptr(),
                 self.ws.data_ptr(), self.ws.numel(), self.stream)

    def prepare(self, means, cov, weights, reg_covar, min_weight) -> None:
        nat.call("gmmxx_em_prepare", self.covc, self.b, self.d, self.k, means.data_ptr(), cov.data_ptr(),
                 weights.data_ptr(), float(reg_covar), float(min_weight), self.ws.data_ptr(), self.ws.numel(),
                 self.stream)

    def accumulate(self, stats, ll) -> None:
        if self.top_k is not None:
            nat.call("gmmxx_em_accumulate_topk", self.covc, self.xdt, self.x.data_ptr(), self.b, self.n, self.d,
                     self.k, self.top_k, self.ws.data_ptr(), self.ws.numel(), self.scratch.data_ptr(),
                     self.scratch.numel(), stats.data_ptr(), ll.data_ptr(), self.stream)
            return
        nat.call("gmmxx_em_accumulate", self.covc, self.xdt, self.x.data_ptr(), self.b, self.n, self.d, self.k,
                 self.ws.data_ptr(), self.ws.numel(), stats.data_ptr(), ll.data_ptr(), self.stream)
        self.paths.add(nat.last_accumulate_path())

    def kernel_path(self) -> str:
        """Which statistics kernels this fit launched (fit_info's kernel_path)."""
        if self.top_k is not None:
            return "cuda-core (approximate top-k)"
        return kernel_path_name(self.paths)

    def finalize(self, n_total, stats, ll, xx, reg_covar, min_weight, means, cov, weights, lb_slot) -> None:
        nat.call("gmmxx_em_finalize", self.covc, self.b, self.d, self.k, n_total, stats.data_ptr(), ll.data_ptr(),
                 _p(xx), float(reg_covar), float(min_weight), means.data_ptr(), cov.data_ptr(), weights.data_ptr(),
                 lb_slot.data_ptr(), self.stream)

    def check_status(self) -> None:
        status = ctypes_int()
        nat.call("gmmxx_workspace_status", self.ws.data_ptr(), status.ref(), self.stream)
        if status.value == nat.ERR_TIMEOUT:
            raise nat.GmmxxError(status.value, "a bounded device-side wait expired in the EM kernel")
        if status.value == nat.ERR_UNSUPPORTED:
            raise nat.GmmxxError(status.value, "an EM kernel rejected its launch configuration on the device")
        if status.value != nat.OK:
            raise nat.GmmxxError(status.value, "covariance not positive definite after the jitter ladder")


def em_loop(ops, cov_type, means, cov, weights, *, n_total, max_iters, tol, reg_covar, min_weight, verbose,
            comm=None):
    """The soft-EM iteration loop (reference loops: torch_fallback.py:2060-2330,
    2486-2696, 2864-3200) over kernel ops ``ops``; with ``comm`` the local
    statistics are sum-allreduced before the (replicated) finalize.

    Returns (n_iter, lower_bound_history list, seconds)."""
    dev = means.device
    b, k = weights.shape
    d = means.shape[2]
    nstat = b * k * ops.stat_width
    # one buffer for the collective: the statistics and, in its last slot, the
    # log-likelihood (fp32 there; per-rank sums are exact to ~1e-7 relative)
    pack = torch.zeros((nstat + (1 if comm is not None else 0),), dtype=torch.float32, device=dev)
    stats = pack[:nstat].view(b, k, ops.stat_width)
    ll = torch.zeros((1,), dtype=torch.float64, device=dev)
    lb_hist = torch.zeros((max_iters,), dtype=torch.float32, device=dev)
    xx = None
    if cov_type == "tied":
        xx = torch.zeros((b, d, d), dtype=torch.float32, device=dev)
        ops.xx_total(xx)
        if comm is not None:
            comm.allreduce_(xx)
    prev = None
    it = 0
    t0 = time.perf_counter()
    for it in range(max_iters):
        ops.prepare(means, cov, weights, reg_covar, min_weight)
        stats.zero_()
        ll.zero_()
        ops.accumulate(stats, ll)
        if comm is not None:  # the iteration's one collective
            pack[nstat:].copy_(ll)
            comm.allreduce_(pack)
            ll.copy_(pack[nstat:])
        if verbose:
            prev_means, prev_cov = means.clone(), cov.clone()
        ops.finalize(n_total, stats, ll, xx, reg_covar, min_weight, means, cov, weights, lb_hist[it:])
        if verbose or tol > 0.0:
            lb = float(lb_hist[it].item())
            if verbose:
                print(verbose_line(cov_type, it, lb, means, prev_means, cov, prev_cov))
            if tol > 0.0 and prev is not None and it + 1 < max_iters and abs(lb - prev) < tol:
                break
            prev = lb
    ops.check_status()
    elapsed = time.perf_counter() - t0
    n_iter = it + 1
    hist = lb_hist[:n_iter].tolist()
    if cov_type != "spherical" and not (tol > 0.0 or verbose):
        # torch_fallback.py:2487/2865: the diag / tied / full loops record 0.0
        # for iterations whose bound was not collected.
        hist = [0.0] * (n_iter - 1) + [hist[-1]]
    return n_iter, hist, elapsed


def verbose_line(cov_type, it, lb, means, prev_means, cov=None, prev_cov=None) -> str:
    """The per-iteration line the reference's loops print with verbose=True:
    bound and largest mean shift (torch_fallback.py:2310-2316, large_n.py:
    1542-1547), plus the largest variance change for diag
    (torch_fallback.py:2680-2694) or covariance change for tied / full
    (3180-3194)."""
    shift = (means - prev_means).norm(dim=-1).max().item()
    line = f"Iter {it}, lower_bound: {lb:.6f}, mean_shift: {shift:.6f}"
    if prev_cov is not None and cov_type in ("diag", "tied", "full"):
        name = "variance_shift" if cov_type == "diag" else "covariance_shift"
        line += f", {name}: {(cov.float() - prev_cov.float()).abs().max().item():.6f}"
    return line


def fit_info(n_iter, hist, source, elapsed, gpus=1, **extra):
    info = {
        "n_iter": n_iter,
        "lower_bound": hist[-1],
        "lower_bound_history": hist,
        "init_source": source,
        "triton_estep_enabled": False,
        "triton_fused_update_enabled": False,
        "triton_approx_topk_enabled": False,
        "triton_streaming_update_enabled": False,
        "triton_labels_enabled": False,
        "approximate_em_enabled": False,
        "approx_top_k": None,
        "cuda_engine": "gmmxx_b200",
        "backend_breakdown": {"cuda": n_iter},
        "gpus": gpus,
        "ms_per_iter": 1e3 * elapsed / n_iter,
    }
    info.update(extra)
    return info


def em_fit(
    cov_type: str,
    x: torch.Tensor,
    n_components: int,
    *,
    max_iters: int = 100,
    tol: float = 1e-4,
    init_means: Optional[torch.Tensor] = None,
    init_variances: Optional[torch.Tensor] = None,
    init_weights: Optional[torch.Tensor] = None,
    init_params: str = "kmeans",
    reg_covar: float = 1e-6,
    min_weight: float = MIN_WEIGHT_DEFAULT,
    compute_labels: bool = True,
    verbose: bool = False,
    comm: Optional[Comm] = None,
    approx_top_k: Optional[int] = None,
    kmeans_init_iters: int = 10,
    kmeans_init_tol: float = 1e-4,
):
    """Soft EM on the CUDA engine.  ``x`` (B, N_local, D) is this rank's row
    shard when ``comm`` is given (the fit is over the union of all shards;
    returned labels are the local shard's).  ``approx_top_k`` in [1, K - 1]
    runs approximate top-k EM (each row's responsibilities restricted to its
    top_k components; torch_fallback.py:667-767)."""
    cov_code(cov_type)
    x = check_x(x)
    b, n_local, d = x.shape
    check_window(cov_type, d)
    if n_components <= 0:
        raise ValueError("n_components must be positive")
    if max_iters <= 0:
        raise ValueError("max_iters must be positive")
    if min_weight <= 0.0:
        raise ValueError("min_weight must be positive")
    dev = x.device
    with torch.cuda.device(dev):
        n_total = n_local
        if comm is not None:
            nt = torch.tensor([n_local], dtype=torch.int64, device=dev)
            comm.allreduce_(nt)
            n_total = int(nt.item())
        if n_total == 0:
            raise ValueError("x must contain at least one sample")
        if comm is not None and init_means is None:  # one initialisation for every rank: rank 0's, broadcast
            means, cov, weights, source = initial_parameters(
                cov_type, x, n_components, None, init_variances, init_weights, reg_covar, init_params,
                kmeans_init_iters, kmeans_init_tol)
            for t in (means, cov, weights):
                comm.broadcast_(t, 0)
        else:
            means, cov, weights, source = initial_parameters(
                cov_type, x, n_components, init_means, init_variances, init_weights, reg_covar, init_params,
                kmeans_init_iters, kmeans_init_tol)
        top_k = resolve_approx_top_k(approx_top_k, means.shape[1])
        ops = CudaOps(cov_type, x, means.shape[1], top_k)
        n_iter, hist, elapsed = em_loop(ops, cov_type, means, cov, weights, n_total=n_total, max_iters=max_iters,
                                        tol=tol, reg_covar=reg_covar, min_weight=min_weight, verbose=verbose,
                                        comm=comm)
        labels = assign(cov_type, x, means, cov, weights) if compute_labels else None
    info = fit_info(n_iter, hist, source, elapsed, gpus=1 if comm is None else comm.world_size,
                    approximate_em_enabled=top_k is not None, approx_top_k=top_k,
                    cuda_approx_topk_enabled=top_k is not None, kernel_path=ops.kernel_path())
    return labels, means, cov, weights, info


class ctypes_int:
    """A host int the C ABI can write through (gmmxx_workspace_status)."""

    def __init__(self):
        import ctypes

        self._c = ctypes.c_int(0)

    def ref(self):
        import ctypes

        return ctypes.addressof(self._c)

    @property
    def value(self) -> int:
        return int(self._c.value)


# ---------------------------------------------------------------------------
# inference
# ---------------------------------------------------------------------------


def _infer_args(cov_type, x, means, cov, weights):
    covc = cov_code(cov_type)
    x = check_x(x)
    b, n, d = x.shape
    check_window(cov_type, d)
    dev = x.device
    means = means.to(device=dev, dtype=torch.float32).contiguous()
    cov = cov.to(device=dev, dtype=torch.float32).contiguous()
    weights = weights.to(device=dev, dtype=torch.float32).contiguous()
    if means.ndim != 3 or means.shape[0] != b or means.shape[2] != d:
        raise ValueError("means must have shape (B, K, D) matching x")
    k = means.shape[1]
    if weights.shape != (b, k):
        raise ValueError("weights must have shape (B, K)")
    shapes = {"spherical": (b, k), "diag": (b, k, d), "tied": (b, d, d), "full": (b, k, d, d)}
    if tuple(cov.shape) != shapes[cov_type]:
        raise ValueError(f"covariance must have shape {shapes[cov_type]} for {cov_type}")
    ws = _WS.get(dev, nat.workspace_bytes(covc, b, n, d, k))
    return covc, x, means, cov, weights, ws, (b, n, d, k)


def _check_tc_infer(covc, x, ws, dims) -> None:
    """After an inference call that ran on a tensor-core kernel (diag or
    spherical, bf16 X in its shape window): read the workspace status word
    (one stream sync) so that an expired bounded wait raises instead of
    leaving stale output."""
    b, n, d, k = dims
    if covc not in (nat.DIAG, nat.SPHERICAL) or x.dtype != torch.bfloat16 or \
            nat.accumulate_path(covc, nat.BFLOAT16, b, n, d, k) != 1:
        return
    status = ctypes_int()
    nat.call("gmmxx_workspace_status", ws.data_ptr(), status.ref(), _stream_ptr(x.device))
    if status.value == nat.ERR_TIMEOUT:
        raise nat.GmmxxError(status.value, "a bounded device-side wait expired in the inference kernel")
    if status.value == nat.ERR_UNSUPPORTED:
        raise nat.GmmxxError(status.value, "the inference kernel rejected its launch configuration on the device")


def assign(cov_type, x, means, cov, weights) -> torch.Tensor:
    """(B, N) int64 labels (torch_fallback.py:780-965)."""
    covc, x, means, cov, weights, ws, (b, n, d, k) = _infer_args(cov_type, x, means, cov, weights)
    out = torch.empty((b, n), dtype=torch.int64, device=x.device)
    with torch.cuda.device(x.device):
        nat.call("gmmxx_assign", covc, _X_DTYPES[x.dtype], x.data_ptr(), b, n, d, k, means.data_ptr(),
                 cov.data_ptr(), weights.data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(),
                 _stream_ptr(x.device))
        _check_tc_infer(covc, x, ws, (b, n, d, k))
    return out


def score_samples(cov_type, x, means, cov, weights) -> torch.Tensor:
    """(B, N) float32 per-sample log-likelihood (torch_fallback.py:983-1130)."""
    covc, x, means, cov, weights, ws, (b, n, d, k) = _infer_args(cov_type, x, means, cov, weights)
    out = torch.empty((b, n), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        nat.call("gmmxx_logsumexp", covc, _X_DTYPES[x.dtype], x.data_ptr(), b, n, d, k, means.data_ptr(),
                 cov.data_ptr(), weights.data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(),
                 _stream_ptr(x.device))
        _check_tc_infer(covc, x, ws, (b, n, d, k))
    return out


def resp(cov_type, x, means, cov, weights, log_norm) -> torch.Tensor:
    """(B, N, K) float32 exp(logit - log_norm) for a given log_norm (B, N)."""
    covc, x, means, cov, weights, ws, (b, n, d, k) = _infer_args(cov_type, x, means, cov, weights)
    log_norm = log_norm.to(device=x.device, dtype=torch.float32).contiguous()
    if log_norm.shape != (b, n):
        raise ValueError("log_norm must have shape (B, N)")
    out = torch.empty((b, n, k), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        nat.call("gmmxx_resp", covc, _X_DTYPES[x.dtype], x.data_ptr(), b, n, d, k, means.data_ptr(),
                 cov.data_ptr(), weights.data_ptr(), log_norm.data_ptr(), out.data_ptr(), ws.data_ptr(),
                 ws.numel(), _stream_ptr(x.device))
    return out


def predict_proba(cov_type, x, means, cov, weights, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """(B, N, K) float32 responsibilities (torch_fallback.py:1133-1345)."""
    covc, x, means, cov, weights, ws, (b, n, d, k) = _infer_args(cov_type, x, means, cov, weights)
    if out is None:
        out = torch.empty((b, n, k), dtype=torch.float32, device=x.device)
    elif out.shape != (b, n, k) or out.dtype != torch.float32 or not out.is_contiguous() or out.device != x.device:
        raise ValueError("out must be a contiguous float32 (B, N, K) tensor on x's device")
    with torch.cuda.device(x.device):
        nat.call("gmmxx_predict_proba", covc, _X_DTYPES[x.dtype], x.data_ptr(), b, n, d, k, means.data_ptr(),
                 cov.data_ptr(), weights.data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(),
                 _stream_ptr(x.device))
        _check_tc_infer(covc, x, ws, (b, n, d, k))
    return out


def canary_add_offset(inp: torch.Tensor, offset: int) -> torch.Tensor:
    """Smoke kernel (reference: gmmxx/_cuda.py:77-97)."""
    if not inp.is_cuda or inp.dtype != torch.int32:
        raise ValueError("canary input must be an int32 CUDA tensor")
    inp = inp.contiguous()
    out = torch.empty_like(inp)
    with torch.cuda.device(inp.device):
        nat.call("gmmxx_canary_add_offset", inp.data_ptr(), out.data_ptr(), inp.numel(), int(offset),
                 _stream_ptr(inp.device))
    return out


def log2pi() -> float:
    return math.log(2.0 * math.pi)
