"""Saving and loading a fitted GMMXX (an addition over the reference, whose
fitted attributes, gmmxx/interface.py:369-396, live only in memory): the
state round-trips through ``torch.save`` / ``torch.load(weights_only=True)``
with every tensor and fit record intact, for each covariance layout, batched
and unbatched; states of another format, version or shape are refused.
Host-only: the estimator is placed on the CPU and no kernel runs."""

import math

import pytest
import torch

from gmmxx_b200 import GMMXX


def _state(cov_type, batch_size, k=4, d=3, n=10, seed=0):
    g = torch.Generator().manual_seed(seed)
    b = 1 if batch_size is None else batch_size
    a = torch.randn((b, d, d), generator=g)
    spd = a @ a.transpose(1, 2) + torch.eye(d)
    cov = {"spherical": torch.rand((b, k), generator=g) + 0.5,
           "diag": torch.rand((b, k, d), generator=g) + 0.5,
           "tied": spd,
           "full": spd[:, None].expand(b, k, d, d).clone()}[cov_type]
    w = torch.rand((b, k), generator=g) + 0.1
    params = GMMXX(k=k, d=d, covariance_type=cov_type, device="cpu", max_iter=7, tol=1e-3,
                   reg_covar=1e-5, random_state=11, dtype=torch.bfloat16).get_params()
    params["dtype"] = "bfloat16"
    params["device"] = "cpu"
    return {
        "format": "gmmxx_b200.GMMXX",
        "version": 1,
        "params": params,
        "batch_size": batch_size,
        "means": torch.randn((b, k, d), generator=g),
        "covariances": cov,
        "weights": w / w.sum(-1, keepdim=True),
        "labels": torch.randint(0, k, (b, n), generator=g),
        "fit_info": {"n_iter": 5, "lower_bound": -3.25, "lower_bound_history": [-4.0, -3.5, -3.25],
                     "init_source": "random", "cuda_engine": "gmmxx_b200", "backend_breakdown": {"cuda": 5}},
    }


@pytest.mark.parametrize("cov_type", ["spherical", "diag", "tied", "full"])
@pytest.mark.parametrize("batch_size", [None, 3])
def test_state_round_trip(tmp_path, cov_type, batch_size):
    state = _state(cov_type, batch_size)
    m = GMMXX(k=1, device="cpu").load_state_dict(state)
    path = tmp_path / "model.pt"
    m.save(path)
    r = GMMXX.load(path, device="cpu")
    for got, want in ((r.means_b, state["means"]), (r.variances_b, state["covariances"]),
                      (r.weights_b, state["weights"]), (r.cluster_ids_b, state["labels"])):
        assert torch.equal(got, want)
    squeeze = (lambda t: t.squeeze(0)) if batch_size is None else (lambda t: t)
    assert torch.equal(r.means_, squeeze(state["means"]))
    assert torch.equal(r.covariances_, squeeze(state["covariances"]))
    assert torch.equal(r.labels_, squeeze(state["labels"]))
    assert r.covariance_type == cov_type and r.k == 4 and r.d == 3 and r.niter == 7
    assert r.tol == 1e-3 and r.reg_covar == 1e-5 and r.seed == 11 and r.dtype == torch.bfloat16
    assert r.lower_bound_ == -3.25 and r.n_iter_ == 5 and r.lower_bound_history_ == [-4.0, -3.5, -3.25]
    assert r.init_source_ == "random" and r.fit_info_["backend_breakdown"] == {"cuda": 5}
    assert r._n_parameters(1) == m._n_parameters(1)
    # a second save of the loaded model writes the same state
    again = r.state_dict()
    for key in ("means", "covariances", "weights", "labels"):
        assert torch.equal(again[key], state[key])
    assert again["params"] == state["params"]


def test_state_without_labels(tmp_path):
    state = _state("diag", None)
    state["labels"] = None
    r = GMMXX(k=1, device="cpu").load_state_dict(state)
    assert r.labels_ is None and r.cluster_ids_b is None
    assert r.state_dict()["labels"] is None


def test_untrained_model_has_no_state():
    with pytest.raises(RuntimeError):
        GMMXX(k=3, device="cpu").state_dict()


@pytest.mark.parametrize("edit", [
    lambda s: s.update(format="other"),
    lambda s: s.update(version=2),
    lambda s: s.update(covariances=torch.ones(1, 4)),          # spherical layout for a diag model
    lambda s: s.update(weights=torch.ones(1, 5) / 5),
    lambda s: s.update(means=torch.zeros(4, 3)),
    lambda s: s.update(batch_size=2),
    lambda s: s.update(labels=torch.zeros(10, dtype=torch.int64)),
    lambda s: s["params"].update(n_components=5),
    lambda s: s["params"].update(d=4),
    lambda s: s["fit_info"].pop("n_iter"),
    lambda s: s.update(means=torch.zeros(1, 4, 3, dtype=torch.int32)),
])
def test_bad_state_refused(edit):
    state = _state("diag", None)
    edit(state)
    with pytest.raises(ValueError):
        GMMXX(k=1, device="cpu").load_state_dict(state)


def test_loaded_nonfinite_bound_survives(tmp_path):
    state = _state("spherical", None)
    state["fit_info"]["lower_bound"] = float("-inf")
    GMMXX(k=1, device="cpu").load_state_dict(state).save(tmp_path / "m.pt")
    assert math.isinf(GMMXX.load(tmp_path / "m.pt", device="cpu").lower_bound_)


@pytest.mark.parametrize("cov_type,per_component", [("spherical", 1), ("diag", 3), ("full", 6)])
def test_parameter_count_for_bic_and_aic(cov_type, per_component):
    """The free-parameter count of the reference's bic / aic
    (interface.py:2537-2547): means K D + covariances + K - 1 weights, per
    problem; tied shares one D(D+1)/2 block."""
    r = GMMXX(k=1, device="cpu").load_state_dict(_state(cov_type, 3))
    k, d = 4, 3
    assert r._n_parameters(1) == k * d + k * per_component + k - 1
    assert r._n_parameters(3) == 3 * (k * d + k * per_component + k - 1)
    t = GMMXX(k=1, device="cpu").load_state_dict(_state("tied", None))
    assert t._n_parameters(1) == k * d + d * (d + 1) // 2 + k - 1
