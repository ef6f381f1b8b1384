"""Record golden vectors from the reference's own PyTorch GMM implementation.

Run in a container that has the reference checkout (read-only) available:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/reference

It imports ``gmmxx.torch_fallback`` from that checkout, runs the four soft-EM
loops (``batch_gmm_{Spherical,Diagonal,Tied,Full}_torch_native``) on small
seeded problems with injected initial parameters, ``tol=0`` and Triton off,
(and, for the APPROX_CASES, ``approx_top_k``), then records the fitted
parameters, the lower-bound history and the three inference outputs (assign / score_samples / predict_proba) on the fitted
parameters into ``tests/golden/<case>.npz``.  The fixtures are what the tests
use; nothing at test time reads the reference.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
KMEANSPP = None

# (name, covariance type, B, N, D, K, iters, reg_covar, chunk_size_N, chunk_size_K, variant)
CASES = [
    ("sph_basic", "spherical", 1, 1200, 6, 4, 8, 1e-6, 32768, 1024, "blobs"),
    ("sph_batched_kchunk", "spherical", 2, 700, 3, 5, 6, 1e-6, 257, 2, "overlap"),
    ("sph_empty_cluster", "spherical", 1, 500, 4, 3, 4, 1e-6, 32768, 1024, "far_init"),
    ("sph_k1_d1", "spherical", 1, 64, 1, 1, 3, 1e-6, 32768, 1024, "blobs"),
    ("sph_cfg0_like", "spherical", 1, 2048, 32, 16, 5, 1e-6, 32768, 1024, "cfg0"),
    ("diag_basic", "diag", 1, 1200, 5, 4, 8, 1e-6, 32768, 1024, "blobs"),
    ("diag_bf16_input", "diag", 1, 1000, 8, 6, 6, 1e-6, 32768, 1024, "bf16"),
    ("diag_batched_kchunk", "diag", 2, 600, 4, 7, 5, 1e-6, 250, 3, "overlap"),
    ("diag_empty_cluster", "diag", 1, 500, 3, 3, 4, 1e-6, 32768, 1024, "far_init"),
    ("tied_basic", "tied", 1, 900, 4, 3, 6, 1e-6, 32768, 1024, "blobs"),
    ("tied_batched_kchunk", "tied", 2, 600, 3, 4, 5, 1e-6, 200, 2, "overlap"),
    ("full_basic", "full", 2, 800, 3, 3, 6, 1e-6, 32768, 1024, "blobs"),
    ("full_empty_cluster", "full", 1, 600, 3, 3, 4, 1e-6, 32768, 1024, "far_init"),
    ("full_jitter_ladder", "full", 1, 400, 3, 2, 3, 0.0, 32768, 1024, "zero_dim"),
]

# Approximate top-k EM (the reference's approx_top_k: each row's
# responsibilities restricted to its top_k logits): the case fields above plus
# top_k.  Seeded after CASES, so adding them leaves the earlier fixtures as
# they were.
APPROX_CASES = [
    ("sph_approx_topk", "spherical", 1, 1000, 5, 8, 5, 1e-6, 32768, 3, "overlap", 3),
    ("sph_approx_topk_k100", "spherical", 1, 2000, 4, 100, 3, 1e-6, 32768, 1024, "blobs", 8),
    ("diag_approx_topk", "diag", 2, 600, 4, 7, 4, 1e-6, 250, 3, "overlap", 2),
    ("diag_approx_topk_k80", "diag", 1, 1500, 6, 80, 3, 1e-6, 32768, 1024, "blobs", 5),
    ("tied_approx_topk", "tied", 1, 700, 3, 5, 4, 1e-6, 32768, 2, "overlap", 2),
    ("full_approx_topk", "full", 1, 600, 3, 4, 4, 1e-6, 32768, 1024, "blobs", 2),
]


def make_data(seed, b, n, d, k, variant):
    g = torch.Generator().manual_seed(seed)
    spread = {"blobs": 6.0, "overlap": 1.5, "far_init": 5.0, "bf16": 4.0, "cfg0": 10.0, "zero_dim": 4.0}[variant]
    centers = (torch.rand(b, k, d, generator=g) * 2 - 1) * spread
    sig = 0.5 + 1.5 * torch.rand(b, k, generator=g)
    comp = torch.randint(0, k, (b, n), generator=g)
    eps = torch.randn(b, n, d, generator=g)
    x = torch.gather(centers, 1, comp[..., None].expand(-1, -1, d)) + sig.gather(1, comp)[..., None] * eps
    if variant == "bf16":
        x = x.to(torch.bfloat16).to(torch.float32)
    if variant == "zero_dim":
        x[..., -1] = 0.0
    # initial means: k distinct sample rows per problem (seeded), unless far_init
    idx = torch.stack([torch.randperm(n, generator=g)[:k] for _ in range(b)])
    init_means = torch.gather(x, 1, idx[..., None].expand(-1, -1, d)).clone()
    if variant == "cfg0":
        # k-means++ seeding, as the benchmark's identical-init recipe prescribes
        torch.manual_seed(seed)
        init_means = KMEANSPP(x, k)
    if variant == "far_init":
        init_means[:, -1, :] = 1.0e3
    init_w = torch.rand(b, k, generator=g) + 0.5
    init_w = init_w / init_w.sum(-1, keepdim=True)
    return x.contiguous(), init_means.contiguous(), init_w.contiguous()


def main(ref_root):
    sys.path.insert(0, ref_root)
    os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")
    from gmmxx import torch_fallback as tf  # noqa: E402  (reference, read-only)

    global KMEANSPP
    KMEANSPP = tf._kmeans_plus_plus_init_means

    fit_fn = {
        "spherical": tf.batch_gmm_Spherical_torch_native,
        "diag": tf.batch_gmm_Diagonal_torch_native,
        "tied": tf.batch_gmm_Tied_torch_native,
        "full": tf.batch_gmm_Full_torch_native,
    }
    infer = {
        "spherical": (tf.spherical_assign_torch_native_chunked, tf.spherical_score_samples_torch_native_chunked,
                      tf.spherical_predict_proba_torch_native_chunked),
        "diag": (tf.diagonal_assign_torch_native_chunked, tf.diagonal_score_samples_torch_native_chunked,
                 tf.diagonal_predict_proba_torch_native_chunked),
        "tied": (tf.tied_assign_torch_native_chunked, tf.tied_score_samples_torch_native_chunked,
                 tf.tied_predict_proba_torch_native_chunked),
        "full": (tf.full_assign_torch_native_chunked, tf.full_score_samples_torch_native_chunked,
                 tf.full_predict_proba_torch_native_chunked),
    }
    torch.set_num_threads(max(1, min(8, os.cpu_count() or 1)))
    cases = [c + (None,) for c in CASES] + APPROX_CASES
    for seed, (name, cov, b, n, d, k, iters, reg, csn, csk, variant, top_k) in enumerate(cases):
        x, init_means, init_w = make_data(1000 + seed, b, n, d, k, variant)
        if cov == "spherical":
            init_var = tf._global_spherical_variance(x, k, reg)
        elif cov == "diag":
            init_var = tf._global_diag_variance(x, k, reg)
        elif cov == "tied":
            init_var = tf._global_tied_covariance(x, reg)
        else:
            init_var = tf._global_full_covariance(x, k, reg)
        kw = dict(reg_covar=reg, chunk_size_N=csn, chunk_size_K=csk, compute_labels=True, approx_top_k=top_k)
        if cov == "spherical":
            kw.update(gmm_use_triton_estep=False, gmm_use_triton_streaming_update=False)
        else:
            kw["gmm_use_triton"] = False
        labels, means, var, w, info = fit_fn[cov](
            x, k, max_iters=iters, tol=0.0, init_means=init_means, init_variances=init_var,
            init_weights=init_w, **kw)
        f_assign, f_score, f_proba = infer[cov]
        ik = dict(chunk_size_N=csn, chunk_size_K=csk)
        a = f_assign(x, means, var, w, **ik)
        s = f_score(x, means, var, w, **ik)
        p = f_proba(x, means, var, w, **ik)
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            cov_type=np.array(cov), x=x.numpy(), init_means=init_means.numpy(), init_var=init_var.numpy(),
            init_weights=init_w.numpy(), n_components=np.array(k), iters=np.array(iters),
            reg_covar=np.array(reg), chunk_size_N=np.array(csn), chunk_size_K=np.array(csk),
            labels=labels.numpy(), means=means.numpy(), cov=var.numpy(), weights=w.numpy(),
            lower_bound_history=np.array(info["lower_bound_history"], dtype=np.float64),
            assign=a.numpy(), score_samples=s.numpy(), predict_proba=p.numpy(),
            **({} if top_k is None else {"approx_top_k": np.array(top_k)}),
        )
        print(f"{name}: lb={info['lower_bound']:.6f} n_iter={info['n_iter']}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GMMXX_REFERENCE_ROOT", "../reference"))
