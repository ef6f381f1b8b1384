"""The reference's large-N entry points (gmmxx/large_n.py:866-1594,
1907-2502): their input contract, checked on the host before any device
work (large_n.py:468-478 and the argument checks at 893-903)."""

import pytest
import torch

import gmmxx_b200 as G

CUDA = torch.device("cuda")


def _fit(x, **kw):
    args = dict(covariance_type="diag", device=CUDA, dtype=torch.float32)
    args.update(kw)
    return G.batch_gmm_largeN_cpu(x, 3, **args)


@pytest.mark.parametrize("x,kw,exc", [
    (torch.zeros(2, 8, 2), {}, NotImplementedError),               # B != 1
    (torch.zeros(8, 2), {}, ValueError),                           # not (B, N, D)
    (torch.zeros(1, 8, 2), dict(device=torch.device("cpu")), ValueError),
    (torch.zeros(1, 8, 2, dtype=torch.int32), {}, TypeError),
    (torch.zeros(1, 8, 2), dict(covariance_type="banded"), ValueError),
    (torch.zeros(1, 8, 2), dict(max_iters=0), ValueError),
    (torch.zeros(1, 8, 2), dict(chunk_size_N=0), ValueError),
    (torch.zeros(1, 8, 2), dict(chunk_size_K=0), ValueError),
    (torch.zeros(1, 8, 2), dict(min_weight=0.0), ValueError),
    (torch.zeros(1, 8, 2), dict(backend="torch"), ValueError),
    (torch.zeros(1, 8, 2), dict(backend="bogus"), ValueError),
    (torch.zeros(1, 8, 2), dict(dtype=torch.float64), TypeError),
])
def test_fit_input_contract(x, kw, exc):
    with pytest.raises(exc):
        _fit(x, **kw)


@pytest.mark.parametrize("fn", [G.large_n_predict_cpu, G.large_n_score_samples_cpu, G.large_n_predict_proba_cpu])
def test_predict_input_contract(fn):
    m, v, w = torch.zeros(1, 3, 2), torch.ones(1, 3, 2), torch.full((1, 3), 1 / 3)
    kw = dict(covariance_type="diag", device=CUDA, dtype=torch.float32, chunk_size_N=4, chunk_size_K=4)
    with pytest.raises(NotImplementedError):
        fn(torch.zeros(2, 8, 2), m, v, w, **kw)
    with pytest.raises(ValueError):
        fn(torch.zeros(1, 8, 2), m, v, w, **dict(kw, device=torch.device("cpu")))
    with pytest.raises(ValueError):
        fn(torch.zeros(1, 8, 2), m, v, w, **dict(kw, chunk_size_N=0))
    with pytest.raises(ValueError):
        fn(torch.zeros(1, 8, 2), m, v, w, **dict(kw, covariance_type="banded"))
    with pytest.raises(ValueError, match="not provided"):
        fn(torch.zeros(1, 8, 2), m, v, w, **dict(kw, backend="triton"))
