"""Record golden vectors for the operator-level API (gmmxx_b200.cuda_ops) from
the reference's own operators in gmmxx/_cuda.py.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_operator_golden.py /path/to/reference

The operators recorded here are plain torch code in the reference
(approx_topk_update_spherical, _cuda.py:783-889; full_assign / full_logsumexp
/ full_resp over _full_logits, 1246-1314; tied_project, tied_log_det,
tied_finalize, full_finalize, 1100-1243, 1355-1416), so they run on the CPU
once the module's CUDA-device checks are relaxed for the recording (the
reference's ``require_cuda`` and ``_check_input`` are replaced in the imported
module object only; its files are not touched).  Each case is written to
``tests/golden/ops_<name>.npz`` with its inputs and outputs; nothing at test
time reads the reference.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _lower(g, *shape):
    """Random lower-triangular factors with diagonal >= 1."""
    a = torch.tril(torch.randn(*shape, generator=g))
    d = shape[-1]
    idx = torch.arange(d)
    a[..., idx, idx] = a[..., idx, idx].abs() + 1.0
    return a


def _spherical_inputs(g, b, n, d, k):
    x = torch.randn(b, n, d, generator=g) * 2.0
    means = torch.randn(b, k, d, generator=g) * 2.0
    var = torch.rand(b, k, generator=g).clamp_min(0.5)
    log_w = torch.log_softmax(torch.randn(b, k, generator=g), dim=-1)
    return x, means, var, log_w


def main(ref_root):
    sys.path.insert(0, ref_root)
    from gmmxx import _cuda as C  # noqa: E402  (reference, read-only)

    # run the reference's torch operators on CPU tensors for the recording
    C.require_cuda = lambda: None
    C._check_input = lambda t, name, dtype=None: t.contiguous()

    def save(name, **arrays):
        np.savez_compressed(os.path.join(HERE, f"ops_{name}.npz"),
                            **{k: (v.numpy() if torch.is_tensor(v) else np.asarray(v)) for k, v in arrays.items()})
        print(name)

    g = torch.Generator().manual_seed(2024)
    # approximate top-k statistics: the reference test's shape, and a larger K
    # whose rows lie near their components (the k-th and (k+1)-th logits of a
    # row are then far enough apart that float rounding cannot swap them)
    for name, (b, n, d, k, top_k) in {"approx_small": (2, 97, 13, 11, 4),
                                     "approx_k150": (1, 3000, 16, 150, 6)}.items():
        x, means, var, log_w = _spherical_inputs(g, b, n, d, k)
        if k > 100:
            means = means * 3.0
            z = torch.randint(0, k, (b, n), generator=g)
            x = torch.gather(means, 1, z[..., None].expand(-1, -1, d)) + torch.randn(b, n, d, generator=g)
        nk, sx, sxx, ll = C.approx_topk_update_spherical(x, means, var, log_w, top_k=top_k, chunk_size_K=64)
        save(name, x=x, means=means, var=var, log_w=log_w, top_k=top_k, nk=nk, sum_x=sx, sum_x_sq=sxx, ll=ll)

    # full-covariance E-step operators
    b, n, d, k = 2, 300, 5, 4
    x = torch.randn(b, n, d, generator=g) * 2.0
    means = torch.randn(b, k, d, generator=g) * 2.0
    L = _lower(g, b, k, d, d)
    log_w = torch.log_softmax(torch.randn(b, k, generator=g), dim=-1)
    lse = C.full_logsumexp(x, means, L, log_w)
    save("full_estep", x=x, means=means, L=L, log_w=log_w, assign=C.full_assign(x, means, L, log_w), lse=lse,
         resp=C.full_resp(x, means, L, log_w, lse))

    # tied projection and log-determinant
    Lt = _lower(g, 2, 6, 6)
    xt = torch.randn(2, 50, 6, generator=g)
    save("tied_project", x=xt, L=Lt, y=C.tied_project(xt, Lt), log_det=C.tied_log_det(Lt))

    # tied finalize from soft statistics (fp32 counts) and from int32 counts
    b, n, d, k = 2, 400, 4, 3
    x = torch.randn(b, n, d, generator=g) + 3.0 * torch.randn(b, 1, d, generator=g)
    r = torch.softmax(torch.randn(b, n, k, generator=g) * 2.0, dim=-1)
    sums = r.transpose(1, 2) @ x
    counts = r.sum(1)
    xx = x.transpose(1, 2) @ x
    m, Lf, w = C.tied_finalize(sums, xx, counts, n, 1e-6)
    save("tied_finalize_soft", sums=sums, xx_total=xx, counts=counts, total_n=n, reg_covar=1e-6, means=m, L=Lf,
         weights=w)
    ids = torch.randint(0, k, (b, n), generator=g)
    onehot = torch.nn.functional.one_hot(ids, k).float()
    counts_i = onehot.sum(1).to(torch.int32)
    sums_i = onehot.transpose(1, 2) @ x
    m, Lf, w = C.tied_finalize(sums_i, xx, counts_i, n, 1e-4)
    save("tied_finalize_hard", sums=sums_i, xx_total=xx, counts=counts_i, total_n=n, reg_covar=1e-4, means=m, L=Lf,
         weights=w)

    # full finalize: soft statistics, one empty component and one whose
    # covariance has no Cholesky factor (both keep their old mean and factor)
    b, n, d, k = 1, 500, 3, 4
    x = torch.randn(b, n, d, generator=g) * 1.5
    r = torch.softmax(torch.randn(b, n, k, generator=g) * 2.0, dim=-1)
    r[..., 2] = 0.0
    sums = r.transpose(1, 2) @ x
    outer = torch.einsum("bnk,bnd,bne->bkde", r, x, x)
    counts = r.sum(1)
    outer[0, 3] = 0.0  # Sigma = -mu mu^T (+ reg): not positive definite
    old_means = torch.randn(b, k, d, generator=g)
    old_L = _lower(g, b, k, d, d)
    m, Lf, w = C.full_finalize(sums, outer, counts, old_means, old_L, n, 1e-6)
    save("full_finalize", sums=sums, outer_sums=outer, counts=counts, old_means=old_means, old_L=old_L, total_n=n,
         reg_covar=1e-6, means=m, L=Lf, weights=w)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GMMXX_REFERENCE_ROOT", "../reference"))
