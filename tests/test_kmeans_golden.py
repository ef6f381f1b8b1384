"""The oracle's k-means++ (a numpy restatement of the reference's
_kmeans_plus_plus_init_means, torch_fallback.py:1390-1451) against centroids
recorded from the reference itself (tests/golden/make_kmeans_golden.py), with
the reference's random draws reproduced from torch's seeded CPU generator.
Centroids are rows of the data, so the comparison is exact."""

import numpy as np
import pytest
import torch

import oracle
from conftest import golden_cases, kmeans_pp_reference_draws, load_golden


@pytest.mark.parametrize("case", golden_cases("init_kmeanspp_"))
def test_oracle_kmeans_pp_matches_reference(case):
    g = load_golden(case)
    x = torch.from_numpy(g["x"])
    k = int(g["k"])
    sample, first, u = kmeans_pp_reference_draws(x, k, int(g["seed"]))
    got = oracle.kmeans_plus_plus(sample.numpy(), k, first.numpy(), u.numpy())
    np.testing.assert_array_equal(got, g["centers"])


def test_fixture_cases_cover_the_reference_paths():
    cases = golden_cases("init_kmeanspp_")
    assert len(cases) >= 5
    ks = set()
    sampled = False
    for case in cases:
        g = load_golden(case)
        k, n = int(g["k"]), g["x"].shape[1]
        ks.add(k)
        sampled |= oracle.kmeans_pp_sample_size(n, k) < n
    assert sampled and 256 in ks and 1 in ks
    assert oracle.kmeans_pp_sample_size(20_000, 257) is None  # the reference declines K > 256


def test_lloyd_and_hard_label_init_are_consistent():
    """Lloyd from k-means++ seeds never raises the k-means objective, and the
    hard-label weights sum to one with every covariance type positive."""
    g = load_golden("init_kmeanspp_sampled_b2")
    x = g["x"]
    seeds = g["centers"]
    lab0 = oracle.nearest_centroid(x, seeds)
    lab, means = oracle.lloyd(x, seeds, 10, 1e-4)
    obj = lambda lb, m: float(np.square(x - np.take_along_axis(m, lb[..., None], 1)).sum())
    assert obj(lab, means) <= obj(lab0, seeds) + 1e-3
    for cov in ("spherical", "diag", "tied", "full"):
        w, c = oracle.hard_label_init(cov, x, means, lab, 1e-6)
        np.testing.assert_allclose(w.sum(-1), 1.0, rtol=1e-6)
        if cov in ("spherical", "diag"):
            assert (c > 0).all()
        else:
            assert (np.linalg.eigvalsh(c) > 0).all()
