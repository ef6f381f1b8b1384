// prepare_finalize.cu -- per-iteration component table (prologue, batch
// Cholesky with the reference's jitter ladder) and the M-step finalize.
//
// Semantics follow the reference's torch loops exactly:
//   prologue   torch_fallback.py:2062-2064 (spherical), 2486-2488 (diag),
//              2866-2867 (tied/full)
//   precision  torch_fallback.py:316-334 (_precision_and_logdet)
//   terms      torch_fallback.py:2491-2494 (diag), 2868-2873 (tied/full)
//   finalize   torch_fallback.py:2293-2305, 2654-2666, 3141-3167
#include "gmm_common.cuh"

#include <math.h>

namespace gmmxx {

constexpr double kLog2PiD = 1.8378770664093453;

// ---------------------------------------------------------------------------
// weights: optional clamp + renormalise (in place), log-weights -> table
// ---------------------------------------------------------------------------
__global__ void prep_weights_kernel(int K, float* weights, float min_weight, int prologue, CompConst* cc) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  float* w = weights + (int64_t)b * K;
  float inv = 1.f;
  if (prologue) {
    float part = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) part += fmaxf(w[k], min_weight);
    const float tot = block_sum<float>(part, red);
    inv = tot;
  }
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    float v = w[k];
    if (prologue) {
      v = fmaxf(v, min_weight) / inv;
      w[k] = v;
    }
    cc[(int64_t)b * K + k].lw = logf(v);
  }
}

// ---------------------------------------------------------------------------
// batch Cholesky (one CTA per matrix, D <= 128)
// ---------------------------------------------------------------------------

// Left-looking Cholesky of the symmetric matrix in `a` (lower triangle used),
// in place; returns false if a pivot is not > 0 (LAPACK potrf's criterion).
__device__ bool chol_inplace(float* a, int D, int ld) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  for (int j = 0; j < D; ++j) {
    if (threadIdx.x == 0) {
      float s = a[j * ld + j];
      for (int k = 0; k < j; ++k) s -= a[j * ld + k] * a[j * ld + k];
      if (!(s > 0.f)) { ok = 0; s = 1.f; }
      a[j * ld + j] = sqrtf(s);
    }
    __syncthreads();
    const float ljj = a[j * ld + j];
    for (int i = j + 1 + threadIdx.x; i < D; i += blockDim.x) {
      float s = a[i * ld + j];
      for (int k = 0; k < j; ++k) s -= a[i * ld + k] * a[j * ld + k];
      a[i * ld + j] = s / ljj;
    }
    __syncthreads();
  }
  const bool r = ok != 0;
  __syncthreads();
  return r;
}

__device__ __forceinline__ float jitter_for(int level) {
  // level 0: plain factorisation; level l >= 1: jitter 1e-6 * 10^(l-1)
  if (level <= 0) return 0.f;
  double j = 1e-6;
  for (int i = 1; i < level; ++i) j *= 10.0;
  return (float)j;
}

__device__ void load_sym(const float* src, float* a, int D, int ld, float jitter) {
  for (int e = threadIdx.x; e < D * D; e += blockDim.x) {
    const int i = e / D, j = e - i * D;
    float v = 0.5f * (src[i * D + j] + src[j * D + i]);
    if (i == j) v = v + jitter;
    a[i * ld + j] = v;
  }
  __syncthreads();
}

__global__ void chol_level_kernel(const float* mats, int D, int* level_out) {
  extern __shared__ __align__(16) float sa[];
  const int ld = D + 1;
  const float* src = mats + (int64_t)blockIdx.x * D * D;
  int found = 7;
  for (int level = 0; level <= 6; ++level) {
    load_sym(src, sa, D, ld, jitter_for(level));
    if (chol_inplace(sa, D, ld)) { found = level; break; }
  }
  if (threadIdx.x == 0 && found > 0) atomicMax(level_out, found);
}

// Factor at the batch-wide level; write precision = (L L^T)^-1,
// log det = 2 sum log L_ii and, when linv_out is given, L^-1 (row-major,
// zero above the diagonal).
__global__ void chol_factor_kernel(const float* mats, int D, const int* level_in, float* prec,
                                   float* logdet, int* status, float* linv_out) {
  extern __shared__ __align__(16) float sa[];
  const int ld = D + 1;
  float* linv = sa + D * ld;
  const int64_t m = blockIdx.x;
  int level = *level_in;
  if (level > 6) {
    if (threadIdx.x == 0 && m == 0) atomicOr(status, 1 << GMMXX_ERR_NOT_PD);
    level = 6;
  }
  load_sym(mats + m * D * D, sa, D, ld, jitter_for(level));
  chol_inplace(sa, D, ld);
  // L^-1 (lower): column c by forward substitution
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    for (int i = 0; i < D; ++i) {
      if (i < c) { linv[i * ld + c] = 0.f; continue; }
      float s = (i == c) ? 1.f : 0.f;
      for (int k = c; k < i; ++k) s -= sa[i * ld + k] * linv[k * ld + c];
      linv[i * ld + c] = s / sa[i * ld + i];
    }
  }
  __syncthreads();
  if (linv_out != nullptr)
    for (int e = threadIdx.x; e < D * D; e += blockDim.x) linv_out[m * D * D + e] = linv[(e / D) * ld + e % D];
  float* pm = prec + m * D * D;
  for (int e = threadIdx.x; e < D * D; e += blockDim.x) {
    const int i = e / D, j = e - i * D;
    const int k0 = i > j ? i : j;
    float s = 0.f;
    for (int k = k0; k < D; ++k) s += linv[k * ld + i] * linv[k * ld + j];
    pm[e] = s;
  }
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < D; ++i) s += logf(sa[i * ld + i]);
    logdet[m] = 2.f * s;
  }
}

// ---------------------------------------------------------------------------
// component table: one warp per component
// ---------------------------------------------------------------------------
template <int COV>
__global__ void prep_table_kernel(int K, int D, int64_t Kp, const float* means, float* cov,
                                  const float* prec, const float* logdet, float reg, int prologue,
                                  CompConst* cc, float* wt) {
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int k = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (k >= Kp) return;
  const int FE = feat_width(COV, D);
  float* w = wt + (int64_t)b * FE * Kp + k;
  if (k >= K) {
    for (int f = lane; f < FE; f += 32) w[(int64_t)f * Kp] = 0.f;
    return;
  }
  const float* mu = means + ((int64_t)b * K + k) * D;
  const float d_log2pi = (float)((double)D * kLog2PiD);
  float mpm = 0.f, ln = 0.f, sc = 1.f;
  if (COV == GMMXX_SPHERICAL) {
    float* vp = cov + (int64_t)b * K + k;
    float v = *vp;
    if (prologue) v = fmaxf(v, reg);
    __syncwarp();
    if (prologue && lane == 0) *vp = v;
    float part = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float m = mu[d];
      part = fmaf(m, m, part);
      w[(int64_t)d * Kp] = -2.f * m;
    }
    mpm = warp_sum(part);
    sc = 1.f / v;
    ln = (float)D * ((float)kLog2PiD + logf(v));
  } else if (COV == GMMXX_DIAG) {
    float* vp = cov + ((int64_t)b * K + k) * D;
    float pmm = 0.f, ld = 0.f;
    for (int d = lane; d < D; d += 32) {
      float v = vp[d];
      if (prologue) { v = fmaxf(v, reg); vp[d] = v; }
      const float vc = fmaxf(v, 1e-30f);
      const float p = 1.f / vc;
      const float wm = mu[d] * p;
      pmm = fmaf(mu[d], wm, pmm);
      ld += logf(vc);
      w[(int64_t)d * Kp] = p;
      w[(int64_t)(D + d) * Kp] = -2.f * wm;
    }
    mpm = warp_sum(pmm);
    ln = d_log2pi + warp_sum(ld);
  } else {
    const bool full = (COV == GMMXX_FULL);
    const float* P = prec + (full ? ((int64_t)b * K + k) : (int64_t)b) * D * D;
    float pmm = 0.f;
    for (int d = lane; d < D; d += 32) {
      float t = 0.f;
      if (full) {
        for (int e = 0; e < D; ++e) t = fmaf(P[d * D + e], mu[e], t);
      } else {
        for (int e = 0; e < D; ++e) t = fmaf(mu[e], P[d * D + e], t);
      }
      pmm = fmaf(mu[d], t, pmm);
      w[(int64_t)d * Kp] = -2.f * t;
    }
    mpm = warp_sum(pmm);
    if (full) {
      // quadratic features x_i x_j (i <= j): weight P_ii or P_ij + P_ji
      const int npairs = D * (D + 1) / 2;
      for (int p = lane; p < npairs; p += 32) {
        int i = 0, rem = p;
        while (rem >= D - i) { rem -= D - i; ++i; }
        const int j = i + rem;
        const float v = (i == j) ? P[i * D + i] : (P[i * D + j] + P[j * D + i]);
        w[(int64_t)(D + p) * Kp] = v;
      }
      ln = d_log2pi + logdet[(int64_t)b * K + k];
    } else {
      ln = d_log2pi + logdet[b];
    }
  }
  if (lane == 0) {
    CompConst* c = cc + (int64_t)b * K + k;
    c->s = sc;
    c->ln = ln;
    c->mpm = mpm;
  }
}

// ---------------------------------------------------------------------------
// finalize: one warp per component, then one CTA per problem
// ---------------------------------------------------------------------------
// M-step finalize, per component: one warp per component k (lanes over the
// feature index), the same element arithmetic as the reference's finalize
// (torch_fallback.py:2293-2305, 2654-2666, 3145-3162).  Weights are written
// unnormalised; finalize_kernel renormalises them.
template <int COV>
__global__ void finalize_comp_kernel(int K, int D, int64_t n_total, const float* stats, float reg, float mw,
                                     float* means, float* cov, float* weights) {
  const int b = blockIdx.y;
  const int k = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (k >= K) return;
  const int FM = stat_width(COV, D);
  const float* s = stats + ((int64_t)b * K + k) * FM;
  const float nk = s[0];
  const bool active = nk > mw;
  const float nks = fmaxf(nk, mw);
  float* mu = means + ((int64_t)b * K + k) * D;
  if (active)
    for (int d = lane; d < D; d += 32) mu[d] = s[1 + d] / nks;
  if (COV == GMMXX_SPHERICAL) {
    if (active && lane == 0) {
      float msq = 0.f;  // sequential over d, as the means were formed
      for (int d = 0; d < D; ++d) {
        const float m = s[1 + d] / nks;
        msq = fmaf(m, m, msq);
      }
      float v = fmaxf(s[1 + D] - nk * msq, 0.f) / (nks * (float)D);
      cov[(int64_t)b * K + k] = fmaxf(v, reg);
    }
  } else if (COV == GMMXX_DIAG) {
    if (active) {
      float* vp = cov + ((int64_t)b * K + k) * D;
      for (int d = lane; d < D; d += 32) {
        const float m = s[1 + d] / nks;
        vp[d] = fmaxf(s[1 + D + d] / nks - m * m, reg);
      }
    }
  } else if (COV == GMMXX_FULL) {
    if (active) {
      float* cp = cov + ((int64_t)b * K + k) * D * D;
      for (int i = 0; i < D; ++i) {
        const float mi = s[1 + i] / nks;
        const int p0 = i * D - i * (i - 1) / 2;  // packed index of (i, i)
        for (int j = i + lane; j < D; j += 32) {
          const float mj = s[1 + j] / nks;
          float c = (s[1 + D + p0 + (j - i)] - nk * (mi * mj)) / nks;
          c = 0.5f * (c + c);
          if (i == j) c = c + reg;
          cp[i * D + j] = c;
          cp[j * D + i] = c;
        }
      }
    }
  }
  if (lane == 0) weights[(int64_t)b * K + k] = fmaxf(nk / (float)n_total, mw);
}

// Per problem: weights renormalised, the tied covariance (from X^T X and
// the new means), the lower bound.
template <int COV>
__global__ void finalize_kernel(int K, int D, int64_t n_total, int64_t B, const float* stats,
                                const double* ll, const float* xx, float reg, float* means,
                                float* cov, float* weights, float* lb_out) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  const int FM = stat_width(COV, D);
  const float* st = stats + (int64_t)b * K * FM;
  const float* mub = means + (int64_t)b * K * D;
  const float nf = (float)n_total;
  float wpart = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) wpart += weights[(int64_t)b * K + k];
  const float wsum = block_sum<float>(wpart, red);
  for (int k = threadIdx.x; k < K; k += blockDim.x) weights[(int64_t)b * K + k] /= wsum;
  if (COV == GMMXX_TIED) {
    const float* xb = xx + (int64_t)b * D * D;
    float* cb = cov + (int64_t)b * D * D;
    for (int e = threadIdx.x; e < D * D; e += blockDim.x) {
      const int i = e / D, j = e - i * D;
      float aij = 0.f, aji = 0.f;
      for (int k = 0; k < K; ++k) {
        const float nk = st[(int64_t)k * FM];
        const float* mu = mub + (int64_t)k * D;
        aij += nk * (mu[i] * mu[j]);
        aji += nk * (mu[j] * mu[i]);
      }
      const float cij = (xb[i * D + j] - aij) / nf;
      const float cji = (xb[j * D + i] - aji) / nf;
      float c = 0.5f * (cij + cji);
      if (i == j) c = c + reg;
      cb[e] = c;  // every thread writes only its own entry; reads use xx and means
    }
  }
  if (b == 0 && threadIdx.x == 0 && lb_out != nullptr) *lb_out = (float)(*ll / ((double)B * (double)n_total));
}

__global__ void canary_kernel(const int32_t* in, int32_t* out, int64_t n, int32_t offset) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = in[i] + offset;
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------

int launch_prepare(int cov, int64_t B, int64_t D, int64_t K, float* means, float* covp, float* weights,
                   float reg, float mw, int prologue, const Layout& L, char* ws, cudaStream_t st) {
  int* status = reinterpret_cast<int*>(ws + L.status);
  CompConst* cc = reinterpret_cast<CompConst*>(ws + L.cc);
  float* wt = reinterpret_cast<float*>(ws + L.wt);
  float* prec = reinterpret_cast<float*>(ws + L.prec);
  // the per-matrix log-determinants live in the (not yet written) lse area
  float* logdet = reinterpret_cast<float*>(ws + L.lse);
  prep_weights_kernel<<<(unsigned)B, 256, 0, st>>>((int)K, weights, mw, prologue, cc);
  if (int rc = check_launch("prep_weights_kernel")) return rc;
  if (cov == GMMXX_TIED || cov == GMMXX_FULL) {
    const int64_t nmat = (cov == GMMXX_TIED) ? B : B * K;
    cudaError_t e = cudaMemsetAsync(status + 1, 0, sizeof(int), st);
    if (e != cudaSuccess) return set_error(GMMXX_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    const int64_t sm1 = D * (D + 1) * 4, sm2 = 2 * sm1;
    if (sm2 > 48 * 1024) {
      cudaFuncSetAttribute(chol_level_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1);
      cudaFuncSetAttribute(chol_factor_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2);
    }
    const int thr = D <= 32 ? 32 : 128;
    chol_level_kernel<<<(unsigned)nmat, thr, sm1, st>>>(covp, (int)D, status + 1);
    if (int rc = check_launch("chol_level_kernel")) return rc;
    float* linv = (cov == GMMXX_TIED) ? reinterpret_cast<float*>(ws + L.linv) : nullptr;
    chol_factor_kernel<<<(unsigned)nmat, thr, sm2, st>>>(covp, (int)D, status + 1, prec, logdet, status, linv);
    if (int rc = check_launch("chol_factor_kernel")) return rc;
  }
  dim3 grid((unsigned)ceil_div(L.Kp, 8), (unsigned)B);
  switch (cov) {
    case GMMXX_SPHERICAL:
      prep_table_kernel<GMMXX_SPHERICAL><<<grid, 256, 0, st>>>((int)K, (int)D, L.Kp, means, covp, prec, logdet, reg, prologue, cc, wt);
      break;
    case GMMXX_DIAG:
      prep_table_kernel<GMMXX_DIAG><<<grid, 256, 0, st>>>((int)K, (int)D, L.Kp, means, covp, prec, logdet, reg, prologue, cc, wt);
      break;
    case GMMXX_TIED:
      prep_table_kernel<GMMXX_TIED><<<grid, 256, 0, st>>>((int)K, (int)D, L.Kp, means, covp, prec, logdet, reg, prologue, cc, wt);
      break;
    default:
      prep_table_kernel<GMMXX_FULL><<<grid, 256, 0, st>>>((int)K, (int)D, L.Kp, means, covp, prec, logdet, reg, prologue, cc, wt);
      break;
  }
  return check_launch("prep_table_kernel");
}

int launch_finalize(int cov, int64_t B, int64_t D, int64_t K, int64_t n_total, const float* stats,
                    const double* ll, const float* xx, float reg, float mw, float* means, float* covp,
                    float* weights, float* lb_out, cudaStream_t st) {
  const dim3 cgrid((unsigned)ceil_div(K, 8), (unsigned)B);
  switch (cov) {
    case GMMXX_SPHERICAL:
      finalize_comp_kernel<GMMXX_SPHERICAL><<<cgrid, 256, 0, st>>>((int)K, (int)D, n_total, stats, reg, mw, means, covp, weights);
      break;
    case GMMXX_DIAG:
      finalize_comp_kernel<GMMXX_DIAG><<<cgrid, 256, 0, st>>>((int)K, (int)D, n_total, stats, reg, mw, means, covp, weights);
      break;
    case GMMXX_TIED:
      finalize_comp_kernel<GMMXX_TIED><<<cgrid, 256, 0, st>>>((int)K, (int)D, n_total, stats, reg, mw, means, covp, weights);
      break;
    default:
      finalize_comp_kernel<GMMXX_FULL><<<cgrid, 256, 0, st>>>((int)K, (int)D, n_total, stats, reg, mw, means, covp, weights);
      break;
  }
  if (int rc = check_launch("finalize_comp_kernel")) return rc;
  switch (cov) {
    case GMMXX_SPHERICAL:
      finalize_kernel<GMMXX_SPHERICAL><<<(unsigned)B, 256, 0, st>>>((int)K, (int)D, n_total, B, stats, ll, xx, reg, means, covp, weights, lb_out);
      break;
    case GMMXX_DIAG:
      finalize_kernel<GMMXX_DIAG><<<(unsigned)B, 256, 0, st>>>((int)K, (int)D, n_total, B, stats, ll, xx, reg, means, covp, weights, lb_out);
      break;
    case GMMXX_TIED:
      finalize_kernel<GMMXX_TIED><<<(unsigned)B, 256, 0, st>>>((int)K, (int)D, n_total, B, stats, ll, xx, reg, means, covp, weights, lb_out);
      break;
    default:
      finalize_kernel<GMMXX_FULL><<<(unsigned)B, 256, 0, st>>>((int)K, (int)D, n_total, B, stats, ll, xx, reg, means, covp, weights, lb_out);
      break;
  }
  return check_launch("finalize_kernel");
}

int launch_canary(const int32_t* in, int32_t* out, int64_t n, int32_t offset, cudaStream_t st) {
  if (n == 0) return GMMXX_OK;
  canary_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(in, out, n, offset);
  return check_launch("canary_kernel");
}

}  // namespace gmmxx
