"""Full covariance with K <= 32 runs the one-pass CUDA-core kernel on a
128-row x 32-component tile (em_small_narrow_kernel); GMMXX_B200_SMALL_TILE=wide
keeps the 64 x 64 tile.  One accumulate call of the two agrees: statistics
to fp32 summation-order noise (relative 1e-5 of each component's largest
statistic), log-likelihood to 1e-6 relative; the fits of both match the
oracle in test_gpu_parity.py / test_gpu_config_parity.py."""

import os

import numpy as np
import pytest
import torch

from test_gpu_parity import _init_cov, _mixture

pytestmark = pytest.mark.gpu


def _one_step(x, k, init, icov, w, tile):
    from gmmxx_b200 import engine

    means, cov, weights, _ = engine.initial_parameters("full", x, k, torch.from_numpy(init),
                                                       torch.from_numpy(icov), torch.from_numpy(w), 1e-6)
    os.environ["GMMXX_B200_SMALL_TILE"] = tile
    try:
        ops = engine.CudaOps("full", x, k)
        stats = torch.zeros((x.shape[0], k, ops.stat_width), device=x.device)
        ll = torch.zeros(1, dtype=torch.float64, device=x.device)
        ops.prepare(means, cov, weights, 1e-6, 1e-8)
        ops.accumulate(stats, ll)
        ops.check_status()
        return stats.cpu().numpy(), float(ll.item())
    finally:
        os.environ.pop("GMMXX_B200_SMALL_TILE", None)


@pytest.mark.parametrize("b,n,d,k", [
    (3, 70_001, 16, 32),   # config-3 problem shape, ragged N, three 64-feature chunks
    (2, 9_000, 6, 20),     # K % 4 != 0: padded components inside the tile, one chunk
    (1, 300, 12, 32),      # fewer rows than one tile
])
def test_narrow_tile_matches_wide(cuda_device, b, n, d, k):
    x, init = _mixture(5 + d + k, b, n, d, k)
    icov = _init_cov("full", x, k)
    w = np.full((b, k), 1.0 / k, np.float32)
    xt = torch.from_numpy(x).to(cuda_device)
    s_n, ll_n = _one_step(xt, k, init, icov, w, "narrow")
    s_w, ll_w = _one_step(xt, k, init, icov, w, "wide")
    scale = np.abs(s_w).max(axis=2, keepdims=True) + 1e-6
    assert np.max(np.abs(s_n - s_w) / scale) < 1e-5
    assert abs(ll_n - ll_w) <= 1e-6 * abs(ll_w)
