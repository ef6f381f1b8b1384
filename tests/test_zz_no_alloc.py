"""gmmxx_logsumexp_noalloc: the score_samples entry point for callers that
cannot allocate device memory (it takes no workspace; its component table sits
in a built-in 8 MiB device array).  Its per-sample log-likelihoods must equal
those of the regular workspace entry point, over two calls in a row with
different models, and it must refuse shapes whose table does not fit.

This file is collected last on purpose: it exercises the shared built-in
array after every other test has run, and must also pass on its own."""


import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc(cov, x, means, covp, weights):
    from gmmxx_b200 import _native as nat
    from gmmxx_b200 import engine

    b, n, d = x.shape
    out = torch.empty((b, n), dtype=torch.float32, device=x.device)
    lib = nat.load()
    rc = lib.gmmxx_logsumexp_noalloc(engine.cov_code(cov), engine._X_DTYPES[x.dtype], x.data_ptr(), b, n, d,
                                     means.shape[1], means.data_ptr(), covp.data_ptr(), weights.data_ptr(),
                                     out.data_ptr(), engine._stream_ptr(x.device))
    return rc, out, lib.gmmxx_last_error().decode()


def _model(cov, b, k, d, dev, seed):
    g = torch.Generator().manual_seed(seed)
    means = torch.randn(b, k, d, generator=g) * 3
    if cov == "spherical":
        c = torch.rand(b, k, generator=g) + 0.5
    elif cov == "diag":
        c = torch.rand(b, k, d, generator=g) + 0.5
    elif cov == "tied":
        a = torch.randn(b, d, d, generator=g)
        c = a @ a.transpose(1, 2) / d + torch.eye(d)
    else:
        a = torch.randn(b, k, d, d, generator=g)
        c = a @ a.transpose(2, 3) / d + torch.eye(d)
    w = torch.rand(b, k, generator=g) + 0.1
    w = w / w.sum(-1, keepdim=True)
    return [t.to(dev).contiguous() for t in (means, c, w)]


def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    from gmmxx_b200 import engine

    cases = [("diag", 2, 5000, 24, 70, torch.float32, 1), ("full", 3, 3000, 6, 5, torch.bfloat16, 2)]
    for cov, b, n, d, k, dt, seed in cases:  # two calls in a row, different models and shapes
        x = (torch.randn(b, n, d, generator=torch.Generator().manual_seed(seed)) * 4).to(dt).to(cuda_device)
        means, covp, w = _model(cov, b, k, d, cuda_device, seed)
        rc, got, msg = _noalloc(cov, x, means, covp, w)
        assert rc == 0, msg
        want = engine.score_samples(cov, x, means, covp, w)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=1e-5, atol=2e-4)


def test_noalloc_rejects_tables_beyond_the_builtin_scratch(cuda_device):
    from gmmxx_b200 import _native as nat

    x = torch.zeros(1, 4, 128, device=cuda_device)
    k = 20000  # spherical weights alone: 128 x 20032 x 4 bytes > 8 MiB
    means = torch.zeros(1, k, 128, device=cuda_device)
    covp = torch.ones(1, k, device=cuda_device)
    w = torch.full((1, k), 1.0 / k, device=cuda_device)
    rc, _, msg = _noalloc("spherical", x, means, covp, w)
    assert rc == nat.ERR_WORKSPACE
    assert "built-in scratch" in msg
