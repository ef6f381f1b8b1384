"""Host-streamed fits on the GPU: buffer reuse across passes, the pinned
staging path for pageable host rows, the reported kernel path, and a fit
sharded over two ranks.

* Every ``ChunkStreamer.chunks()`` pass (one per EM iteration) refills the two
  device buffers while the previous pass's last chunks may still be in use;
  with tol = 0 nothing on the host waits between iterations, so a missing
  wait shows up as wrong statistics.  An even chunk count lines the buffers
  up with the next pass's first copies.  Resident and streamed fits differ
  only in fp32 summation order.
* ``GMMXX_B200_TEST_NO_CLUSTER=1`` makes the tensor-core launch report no
  co-resident cluster (as a device that cannot co-schedule the cluster
  would); the CUDA-core kernels then run and the fit records it.
* Two processes on one GPU, each streaming half of the rows, joined by a
  ``gloo`` process group, fit the union of their shards: both ranks end with
  the same parameters, equal to the oracle on all rows.  The ranks' kernels
  never wait on each other (the only exchange is the host-side collective)."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from test_gpu_parity import PARAM_TOL, _init_cov, _mixture, assert_parity

pytestmark = pytest.mark.gpu


def _separated(seed, n, d, k):
    """Rows of k well-separated spherical clusters and initial means near the
    true ones, so that the fits compared below are well conditioned (a
    random-row initialisation can put two components on one cluster, whose
    split then amplifies summation-order rounding)."""
    rng = np.random.default_rng(seed)
    mu = rng.uniform(-8, 8, (k, d))
    z = rng.integers(0, k, n)
    x = (mu[z] + rng.uniform(0.5, 1.2, k)[z, None] * rng.standard_normal((n, d))).astype(np.float32)[None]
    init = (mu + 0.3 * rng.standard_normal(mu.shape)).astype(np.float32)[None]
    return x, init


@pytest.mark.parametrize("pinned", [True, False])
@pytest.mark.parametrize("cov", ["spherical", "tied"])
def test_streamed_passes_reuse_buffers_safely(cuda_device, pinned, cov):
    from gmmxx_b200 import engine, large_n

    x, init = _separated(61, 16_000, 32, 48)
    icov = _init_cov(cov, x, 48)
    w = np.full((1, 48), 1 / 48, np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    a = engine.em_fit(cov, t(x).to(cuda_device), 48, max_iters=6, tol=0.0, init_means=t(init),
                      init_variances=t(icov), init_weights=t(w))
    xh = t(x).pin_memory() if pinned else t(x)
    st = large_n.ChunkStreamer(xh, 2000, cuda_device)  # 8 chunks per pass
    assert (st.stage is None) == pinned
    b = large_n.em_fit_streamed(cov, xh, 48, device=cuda_device, chunk_rows=2000, max_iters=6, tol=0.0,
                                init_means=t(init), init_variances=t(icov), init_weights=t(w), streamer=st)
    for u, v in zip(a[1:4], b[1:4]):
        np.testing.assert_allclose(u.cpu().numpy(), v.cpu().numpy(), **PARAM_TOL)
    np.testing.assert_allclose(a[4]["lower_bound"], b[4]["lower_bound"], rtol=1e-5)
    assert (a[0] == b[0]).float().mean().item() >= 0.999
    # 6 iterations + the label pass (+ the X^T X pass for tied) streamed every row
    passes = 7 + (1 if cov == "tied" else 0)
    assert st.h2d_bytes == passes * x.nbytes


def test_no_cluster_fallback_is_reported(cuda_device, monkeypatch):
    from gmmxx_b200 import engine

    rng = np.random.default_rng(5)
    mu = rng.normal(0, 3, (64, 64))
    z = rng.integers(0, 64, 70_000)
    x = torch.from_numpy((mu[z] + rng.standard_normal((70_000, 64))).astype(np.float32)).to(torch.bfloat16)[None]
    init = torch.from_numpy((mu + 0.3 * rng.standard_normal(mu.shape)).astype(np.float32))[None]
    xd = x.to(cuda_device)
    a = engine.em_fit("diag", xd, 64, max_iters=2, tol=0.0, init_means=init)
    assert a[4]["kernel_path"] == "tensor-core"
    monkeypatch.setenv("GMMXX_B200_TEST_NO_CLUSTER", "1")
    b = engine.em_fit("diag", xd, 64, max_iters=2, tol=0.0, init_means=init)
    assert "no co-resident cluster" in b[4]["kernel_path"]
    from gmmxx_b200 import _native as nat

    assert nat.last_accumulate_path() == 2
    for u, v in zip(a[1:4], b[1:4]):
        np.testing.assert_allclose(u.cpu().numpy(), v.cpu().numpy(), rtol=1e-4, atol=1e-4)


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_worker(rank, world, port, cov, x, init, icov, w, out_dir):
    import torch.distributed as dist

    from gmmxx_b200 import engine, large_n

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        n = x.shape[1]
        lo, hi = rank * n // world, (rank + 1) * n // world
        shard = torch.from_numpy(np.ascontiguousarray(x[:, lo:hi]))
        t = torch.from_numpy
        labels, means, c, wt, info = large_n.em_fit_streamed(
            cov, shard, init.shape[1], device=dev, chunk_rows=1500, max_iters=4, tol=0.0, init_means=t(init),
            init_variances=t(icov), init_weights=t(w), comm=engine.Comm())
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), labels=labels.cpu().numpy(), means=means.cpu().numpy(),
                 cov=c.cpu().numpy(), w=wt.cpu().numpy(), lb=info["lower_bound"], gpus=info["gpus"])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cov", ["diag", "tied"])
def test_sharded_streamed_fit_matches_oracle(cuda_device, cov, tmp_path):
    import torch.multiprocessing as mp

    x, init = _mixture(71, 1, 9001, 10, 6)
    icov = _init_cov(cov, x, 6)
    w = np.full((1, 6), 1 / 6, np.float32)
    ref32 = oracle.fit(cov, x, 6, 4, 0.0, init, icov, w)
    ref64 = oracle.fit(cov, x, 6, 4, 0.0, init, icov, w, dtype=np.float64)
    mp.start_processes(_shard_worker, args=(2, _free_port(), cov, x, init, icov, w, str(tmp_path)), nprocs=2,
                       join=True, start_method="spawn")
    r = [np.load(tmp_path / f"rank{i}.npz") for i in range(2)]
    for key in ("means", "cov", "w", "lb"):
        assert np.array_equal(r[0][key], r[1][key]), key  # replicated finalize: identical on every rank
    assert int(r[0]["gpus"]) == 2
    assert_parity(r[0]["means"], ref32[1], ref64[1], name="means")
    assert_parity(r[0]["cov"], ref32[2], ref64[2], name="covariances")
    assert_parity(r[0]["w"], ref32[3], ref64[3], name="weights")
    assert abs(float(r[0]["lb"]) - ref32[4]["lower_bound"]) <= 1e-4 * abs(ref32[4]["lower_bound"])
    labels = np.concatenate([r[0]["labels"], r[1]["labels"]], axis=1)
    assert (labels == ref32[0]).mean() >= 0.999
