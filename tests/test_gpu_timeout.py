"""Failure detection on the GPU without a fault: a bounded wait in the
tensor-core kernel runs out and surfaces as GMMXX_ERR_TIMEOUT on the host,
and the CUDA context stays usable.

GMMXX_B200_TEST_STALL=1 makes the producer warp of em_tc_diag_kernel issue no
X tile loads and shortens every wait to 100 ms: the prep warps' wait for the
first tile expires, they set the kernel's abort flag, every other role leaves
its loop, the MMA thread still commits its final barrier (tensor memory is
drained before it is freed) and the kernel returns with the sticky status bit
set.  Nothing traps or hangs; the next call on the same stream and workspace
runs normally."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_and_context_survives(cuda_device, monkeypatch):
    from gmmxx_b200 import _native as nat
    from gmmxx_b200 import engine

    n, d, k = 65_536, 64, 128
    assert nat.accumulate_path(nat.DIAG, nat.BFLOAT16, 1, n, d, k) == 1
    g = torch.Generator().manual_seed(3)
    x = (torch.randn((1, n, d), generator=g) * 2.0).to(torch.bfloat16).to(cuda_device)
    init = torch.randn((1, k, d), generator=g) * 2.0
    means, cov, weights, _ = engine.initial_parameters("diag", x, k, init, torch.ones((1, k, d)),
                                                       torch.full((1, k), 1.0 / k), 1e-6)
    ops = engine.CudaOps("diag", x, k)
    stats = torch.zeros((1, k, ops.stat_width), device=cuda_device)
    ll = torch.zeros(1, dtype=torch.float64, device=cuda_device)

    monkeypatch.setenv("GMMXX_B200_TEST_STALL", "1")
    ops.prepare(means, cov, weights, 1e-6, 1e-8)
    ops.accumulate(stats, ll)
    with pytest.raises(nat.GmmxxError) as err:
        ops.check_status()
    assert err.value.status == nat.ERR_TIMEOUT

    monkeypatch.delenv("GMMXX_B200_TEST_STALL")
    stats.zero_()
    ll.zero_()
    ops.prepare(means, cov, weights, 1e-6, 1e-8)
    ops.accumulate(stats, ll)
    ops.check_status()  # the status word was cleared; this run completes
    torch.cuda.synchronize()
    nk = stats[0, :, 0].double().sum().item()
    assert abs(nk - n) <= 1e-3 * n
    assert np.isfinite(ll.item())
