"""Record golden k-means++ centroids from the reference's own function.

Run in a container that has the reference checkout (read-only) available:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_kmeans_golden.py /path/to/reference

For each case it seeds torch's CPU generator, calls the reference's
``gmmxx.torch_fallback._kmeans_plus_plus_init_means`` on CPU rows (which
draws the row sample's ``randperm``, the first centre's ``randint`` and the
per-centre uniforms from that generator), and records the rows, the seed and
the returned centroids into ``tests/golden/init_kmeanspp_<case>.npz``.  Cases
cover the whole-data path (N below the sample size), the sampled path
(``randperm``), several problems in one batch, local-trial counts 2 .. 7 and
K at the reference's limit of 256.  Nothing at test time reads the reference.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, B, N, D, K, seed)
CASES = [
    ("whole_small", 1, 900, 3, 4, 11),        # N < sample size: no randperm; 3 trials
    ("sampled_b2", 2, 10_000, 8, 16, 12),     # sample of 4096 rows (randperm), 4 trials
    ("sampled_k100", 1, 20_000, 5, 100, 13),  # sample of 6400 rows, 6 trials
    ("k256", 1, 20_000, 4, 256, 14),          # the reference's largest K, 7 trials
    ("k1", 1, 500, 2, 1, 15),                 # the first centre alone
]


def make_rows(seed, b, n, d, k):
    g = torch.Generator().manual_seed(1000 + seed)
    centers = torch.rand((b, k, d), generator=g) * 20.0 - 10.0
    comp = torch.randint(0, k, (b, n), generator=g)
    x = torch.gather(centers, 1, comp[..., None].expand(-1, -1, d)) + torch.randn((b, n, d), generator=g)
    return x.float().contiguous()


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from gmmxx.torch_fallback import _kmeans_plus_plus_init_means

    for name, b, n, d, k, seed in CASES:
        x = make_rows(seed, b, n, d, k)
        torch.manual_seed(seed)
        centers = _kmeans_plus_plus_init_means(x, k)
        assert centers is not None, name
        np.savez(os.path.join(HERE, f"init_kmeanspp_{name}.npz"), x=x.numpy(), k=k, seed=seed,
                 centers=centers.numpy())
        print(name, centers.shape)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GMMXX_REFERENCE_ROOT", "../reference"))
