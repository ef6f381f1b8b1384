"""Multi-rank EM on CPU: the N-sharded path of ``engine.em_loop`` with a
``gloo`` process group (world size 2), no GPU.

Each rank holds a contiguous shard of the rows and runs prepare -> accumulate
on it; ``engine.Comm`` sum-allreduces the statistics and the log-likelihood;
every rank finalizes.  The per-rank kernels are replaced by ``OracleOps``, a
CPU implementation of the same four-call interface built on the oracle (the
oracle is the checker here, not the product), so the test exercises the host
logic of the sharded fit: shard bookkeeping, the collective order, the
replicated finalize and the bound over all rows.  The result must match the
single-process oracle fit of the unsharded data, and both ranks must hold
identical parameters.

A second case kills one rank before the collective: the surviving rank must
get an error from its process group within the group timeout, not hang.
"""

from __future__ import annotations

import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from oracle import gmm_oracle as orc  # noqa: E402


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleOps:
    """CPU stand-in for ``engine.CudaOps`` on one shard (float64 arithmetic).

    Statistics layout per component: [n_k | sum r x (D) | second moment],
    the second moment being sum r x^2 (diag, D), sum r |x|^2 (spherical, 1),
    nothing (tied) or sum r x x^T (full, D*D)."""

    def __init__(self, cov_type: str, x_shard: np.ndarray, k: int, top_k=None):
        self.cov_type = cov_type
        self.top_k = top_k  # approximate EM: responsibilities over each row's top_k logits
        self.x = x_shard.astype(np.float64)
        self.b, self.n, self.d = self.x.shape
        self.k = k
        d = self.d
        self.stat_width = 1 + d + {"diag": d, "spherical": 1, "tied": 0, "full": d * d}[cov_type]
        self._model = None

    def xx_total(self, xx: torch.Tensor) -> None:
        xx += torch.from_numpy(np.swapaxes(self.x, 1, 2) @ self.x)

    def prepare(self, means, cov, weights, reg_covar, min_weight) -> None:
        # per-iteration prologue (torch_fallback.py:2062-2064, 2486-2488, 2866-2867)
        if self.cov_type in ("spherical", "diag"):
            cov.clamp_(min=reg_covar)
        weights.clamp_(min=min_weight)
        weights /= weights.sum(dim=-1, keepdim=True)
        self._model = orc._Model(self.cov_type, means.numpy(), cov.numpy(), weights.numpy(), np.float64)

    def accumulate(self, stats: torch.Tensor, ll: torch.Tensor) -> None:
        x = self.x
        xsq = np.square(x).sum(axis=-1)
        lg = self._model.logits(x, xsq, 0, self.k)
        if self.top_k is not None:
            order = np.argsort(-lg, axis=-1, kind="stable")[..., :self.top_k]
            vals = np.take_along_axis(lg, order, axis=-1)
            lse = orc._logsumexp(vals)
            r = np.zeros_like(lg)
            np.put_along_axis(r, order, np.exp(vals - lse[:, :, None]), axis=-1)
        else:
            lse = orc._logsumexp(lg)
            r = np.exp(lg - lse[:, :, None])
        d = self.d
        st = np.zeros((self.b, self.k, self.stat_width))
        st[..., 0] = r.sum(axis=1)
        st[..., 1:1 + d] = np.swapaxes(r, 1, 2) @ x
        if self.cov_type == "diag":
            st[..., 1 + d:] = np.swapaxes(r, 1, 2) @ np.square(x)
        elif self.cov_type == "spherical":
            st[..., 1 + d] = (r * xsq[:, :, None]).sum(axis=1)
        elif self.cov_type == "full":
            st[..., 1 + d:] = np.einsum("bnk,bnd,bne->bkde", r, x, x).reshape(self.b, self.k, d * d)
        stats += torch.from_numpy(st).to(stats.dtype)
        ll += float(lse.sum())

    def finalize(self, n_total, stats, ll, xx, reg_covar, min_weight, means, cov, weights, lb_slot) -> None:
        # finalize rules: torch_fallback.py:2293-2305 (spherical), 2654-2666 (diag), 3141-3167 (tied / full)
        st = stats.double().numpy()
        d = self.d
        nk = st[..., 0]
        active = nk > min_weight
        nk_safe = np.maximum(nk, min_weight)
        old_m = means.double().numpy()
        m = np.where(active[..., None], st[..., 1:1 + d] / nk_safe[..., None], old_m)
        c_old = cov.double().numpy()
        if self.cov_type == "spherical":
            v = np.maximum(st[..., 1 + d] - nk * np.square(m).sum(-1), 0.0) / (nk_safe * d)
            c = np.where(active, np.maximum(v, reg_covar), c_old)
        elif self.cov_type == "diag":
            v = np.maximum(st[..., 1 + d:] / nk_safe[..., None] - np.square(m), reg_covar)
            c = np.where(active[..., None], v, c_old)
        else:
            outer = m[..., :, None] * m[..., None, :]
            eye = np.eye(d)
            if self.cov_type == "full":
                sxx = st[..., 1 + d:].reshape(self.b, self.k, d, d)
                cf = (sxx - nk[..., None, None] * outer) / nk_safe[..., None, None]
                cf = 0.5 * (cf + np.swapaxes(cf, -1, -2)) + reg_covar * eye
                c = np.where(active[..., None, None], cf, c_old)
            else:
                ct = (xx.double().numpy() - (nk[..., None, None] * outer).sum(axis=1)) / n_total
                c = 0.5 * (ct + np.swapaxes(ct, -1, -2)) + reg_covar * eye
        w = np.maximum(nk / n_total, min_weight)
        w = w / w.sum(axis=-1, keepdims=True)
        means.copy_(torch.from_numpy(m))
        cov.copy_(torch.from_numpy(c))
        weights.copy_(torch.from_numpy(w))
        lb_slot[0] = float(ll.double()[0]) / (self.b * n_total)

    def check_status(self) -> None:
        pass


def _problem(cov_type, seed=7, b=2, n=600, d=3, k=4):
    g = np.random.default_rng(seed)
    centers = g.uniform(-6, 6, size=(b, k, d))
    comp = g.integers(0, k, size=(b, n))
    x = np.take_along_axis(centers, comp[..., None].repeat(d, -1), axis=1) + g.normal(size=(b, n, d))
    init_m = x[:, :k].copy()
    if cov_type == "spherical":
        init_c = np.ones((b, k))
    elif cov_type == "diag":
        init_c = np.ones((b, k, d))
    elif cov_type == "tied":
        init_c = np.tile(np.eye(d), (b, 1, 1))
    else:
        init_c = np.tile(np.eye(d), (b, k, 1, 1))
    init_w = np.full((b, k), 1.0 / k)
    return x, init_m, init_c, init_w


def _rank_main(rank, world, port, cov_type, iters, out_dir, fail_rank, top_k=None):
    from gmmxx_b200 import engine

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        x, m0, c0, w0 = _problem(cov_type)
        n = x.shape[1]
        lo, hi = rank * n // world, (rank + 1) * n // world
        ops = OracleOps(cov_type, x[:, lo:hi], m0.shape[1], top_k)
        means = torch.from_numpy(m0.copy())
        cov = torch.from_numpy(c0.copy())
        weights = torch.from_numpy(w0.copy())
        if rank == fail_rank:
            raise SystemExit(3)  # this rank dies before its first collective
        try:
            n_iter, hist, _ = engine.em_loop(ops, cov_type, means, cov, weights, n_total=n, max_iters=iters, tol=0.0,
                                             reg_covar=1e-6, min_weight=1e-8, verbose=True, comm=engine.Comm())
            np.savez(os.path.join(out_dir, f"r{rank}.npz"), means=means.numpy(), cov=cov.numpy(),
                     weights=weights.numpy(), hist=np.array(hist))
        except Exception as exc:  # the surviving rank of the failure case
            with open(os.path.join(out_dir, f"r{rank}.err"), "w") as f:
                f.write(repr(exc))
    finally:
        if dist.is_initialized() and rank != fail_rank:
            dist.destroy_process_group()


def _launch(cov_type, iters, tmp_path, fail_rank=-1, world=2, top_k=None):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, cov_type, iters, str(tmp_path), fail_rank, top_k))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
            pytest.fail("a rank did not finish within 120 s")
    return [p.exitcode for p in procs]


@pytest.mark.parametrize("cov_type", ["spherical", "diag", "tied", "full"])
def test_sharded_fit_matches_single_process(cov_type, tmp_path):
    iters = 4
    codes = _launch(cov_type, iters, tmp_path)
    assert codes == [0, 0]
    r0 = np.load(tmp_path / "r0.npz")
    r1 = np.load(tmp_path / "r1.npz")
    for key in ("means", "cov", "weights", "hist"):
        assert np.array_equal(r0[key], r1[key]), f"ranks disagree on {key}"
    x, m0, c0, w0 = _problem(cov_type)
    _, m, c, w, info = orc.fit(cov_type, x, m0.shape[1], iters, 0.0, m0, c0, w0, compute_labels=False,
                               dtype=np.float64)
    # em_loop keeps the statistics and the bound history in fp32 (the C ABI's
    # types), so the sharded fit agrees with the float64 oracle to fp32 rounding
    np.testing.assert_allclose(r0["means"], m, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(r0["cov"], c, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(r0["weights"], w, rtol=1e-5, atol=1e-7)
    # the last bound is the mean log-likelihood over all rows of both shards
    np.testing.assert_allclose(r0["hist"][-1], info["lower_bound_history"][-1], rtol=1e-6)


def test_sharded_approx_fit_matches_single_process(tmp_path):
    """Approximate top-k EM (each row's responsibilities over its 2 best of 4
    components) sharded over two ranks equals the single-process oracle's
    approximate EM: the top-k lists are per row, so sharding changes only the
    summation order of the statistics."""
    codes = _launch("diag", 4, tmp_path, top_k=2)
    assert codes == [0, 0]
    r0 = np.load(tmp_path / "r0.npz")
    r1 = np.load(tmp_path / "r1.npz")
    for key in ("means", "cov", "weights", "hist"):
        assert np.array_equal(r0[key], r1[key]), f"ranks disagree on {key}"
    x, m0, c0, w0 = _problem("diag")
    _, m, c, w, info = orc.fit("diag", x, m0.shape[1], 4, 0.0, m0, c0, w0, compute_labels=False, dtype=np.float64,
                               approx_top_k=2)
    assert info["approximate_em_enabled"]
    np.testing.assert_allclose(r0["means"], m, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(r0["cov"], c, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(r0["weights"], w, rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(r0["hist"][-1], info["lower_bound_history"][-1], rtol=1e-6)


def test_dead_rank_surfaces_as_error(tmp_path):
    codes = _launch("diag", 3, tmp_path, fail_rank=1)
    assert codes[1] == 3
    assert codes[0] == 0, "the surviving rank must return, not crash or hang"
    err = (tmp_path / "r0.err")
    assert err.exists(), "the surviving rank must see an error from its collective"
    assert not (tmp_path / "r0.npz").exists()


@pytest.mark.parametrize("cov_type,extra", [("spherical", None), ("diag", "variance_shift"),
                                            ("tied", "covariance_shift"), ("full", "covariance_shift")])
def test_verbose_lines_match_the_reference_format(cov_type, extra, capsys):
    """verbose=True prints one line per iteration in the reference's format
    (torch_fallback.py:2310-2316, 2680-2694, 3180-3194): the bound, the
    largest mean shift and, for diag / tied / full, the largest change of the
    variances or covariances."""
    import re

    from gmmxx_b200 import engine

    x, m0, c0, w0 = _problem(cov_type, b=1)
    ops = OracleOps(cov_type, x, m0.shape[1])
    means, cov, weights = (torch.from_numpy(a.copy()) for a in (m0, c0, w0))
    n_iter, hist, _ = engine.em_loop(ops, cov_type, means, cov, weights, n_total=x.shape[1], max_iters=3, tol=0.0,
                                     reg_covar=1e-6, min_weight=1e-8, verbose=True)
    lines = capsys.readouterr().out.strip().splitlines()
    assert len(lines) == n_iter == 3
    pat = r"Iter (\d+), lower_bound: (-?\d+\.\d{6}), mean_shift: (\d+\.\d{6})"
    if extra:
        pat += rf", {extra}: (\d+\.\d{{6}})"
    for it, line in enumerate(lines):
        mt = re.fullmatch(pat, line)
        assert mt, line
        assert int(mt.group(1)) == it
        assert float(mt.group(2)) == pytest.approx(hist[it], abs=1e-6)
    # the first iteration moves the means away from their initial rows
    assert float(re.fullmatch(pat, lines[0]).group(3)) > 0.0


# ---------------------------------------------------------------------------
# the host-streamed driver sharded over ranks (large_n.em_fit_streamed)
# ---------------------------------------------------------------------------


class CpuChunker:
    """CPU stand-in for ``large_n.ChunkStreamer``: the shard's row chunks in
    order (no device buffers or streams)."""

    def __init__(self, x_host, chunk_rows, device):
        self.x = x_host
        self.n, self.d = x_host.shape[1], x_host.shape[2]
        self.chunk = max(1, min(int(chunk_rows), self.n))
        self.device = torch.device(device)
        self.bufs = [x_host[:, :self.chunk]]
        self.passes = 0

    def chunks(self):
        self.passes += 1
        for n0 in range(0, self.n, self.chunk):
            yield self.x[:, n0:n0 + self.chunk], n0


class OracleStreamOps(OracleOps):
    """``large_n.StreamedOps`` on the CPU: OracleOps over each streamed chunk."""

    def __init__(self, cov_type, streamer, k, top_k=None):
        super().__init__(cov_type, streamer.x.numpy(), k, top_k)
        self.st = streamer

    def accumulate(self, stats, ll):
        whole = self.x
        try:
            for xc, _ in self.st.chunks():
                self.x = xc.numpy().astype(np.float64)
                self.n = self.x.shape[1]
                super().accumulate(stats, ll)
        finally:
            self.x, self.n = whole, whole.shape[1]

    def kernel_path(self):
        return "oracle"


def _stream_rank_main(rank, world, port, cov_type, iters, out_dir, given_init):
    from gmmxx_b200 import engine, large_n

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        large_n.ChunkStreamer = CpuChunker
        large_n.StreamedOps = OracleStreamOps
        x, m0, c0, w0 = _problem(cov_type, b=1)
        n = x.shape[1]
        lo, hi = rank * n // world, (rank + 1) * n // world
        shard = torch.from_numpy(np.ascontiguousarray(x[:, lo:hi], dtype=np.float32))
        torch.manual_seed(100 + rank)  # a rank-local draw would differ between ranks
        init = dict(init_means=torch.from_numpy(m0), init_variances=torch.from_numpy(c0),
                    init_weights=torch.from_numpy(w0)) if given_init else dict(init_params="random")
        _, means, cov, weights, info = large_n.em_fit_streamed(
            cov_type, shard, m0.shape[1], device="cpu", chunk_rows=70, max_iters=iters, tol=0.0,
            compute_labels=False, comm=engine.Comm(), **init)
        np.savez(os.path.join(out_dir, f"s{rank}.npz"), means=means.numpy(), cov=cov.numpy(),
                 weights=weights.numpy(), hist=np.array(info["lower_bound_history"]), gpus=info["gpus"])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cov_type,given_init", [("diag", True), ("tied", True), ("spherical", False),
                                                 ("full", False)])
def test_sharded_streamed_fit(cov_type, given_init, tmp_path):
    """Each rank streams its own shard in chunks; one allreduce per iteration
    joins them.  With given initial parameters the fit equals the
    single-process oracle on all rows; with drawn ones, rank 0's draw is
    broadcast, so the ranks still end identical."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_stream_rank_main, args=(r, 2, port, cov_type, 4, str(tmp_path), given_init))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
            pytest.fail("a rank did not finish within 120 s")
    assert [p.exitcode for p in procs] == [0, 0]
    r0, r1 = np.load(tmp_path / "s0.npz"), np.load(tmp_path / "s1.npz")
    for key in ("means", "cov", "weights", "hist"):
        assert np.array_equal(r0[key], r1[key]), f"ranks disagree on {key}"
    assert int(r0["gpus"]) == 2
    if given_init:
        x, m0, c0, w0 = _problem(cov_type, b=1)
        _, m, c, w, info = orc.fit(cov_type, x, m0.shape[1], 4, 0.0, m0, c0, w0, compute_labels=False,
                                   dtype=np.float64)
        np.testing.assert_allclose(r0["means"], m, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(r0["cov"], c, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(r0["weights"], w, rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(r0["hist"][-1], info["lower_bound_history"][-1], rtol=1e-6)
