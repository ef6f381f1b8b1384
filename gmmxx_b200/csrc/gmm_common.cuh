// gmm_common.cuh -- shared definitions of the B200 GMM EM engine.
//
// The engine writes every covariance type as one "feature" contraction:
//
//   dist[n,k]  = q_n + sum_f phi_f(x_n) * W[f,k] + mpm_k          (clamped >= 0)
//   logit[n,k] = lw_k - 0.5 * (s_k * dist[n,k] + ln_k)
//
// which is the reference's expanded-distance logit
// (gmmxx/torch_fallback.py:337-465) with the loop-invariant terms folded into
// a per-iteration "component table":
//
//   type       phi (E-step features)          W[f,k]                         q_n        s_k
//   spherical  x_d                            -2 mu_kd                       |x|^2      1/var_k
//   diag       [x_d^2, x_d]                   [1/var_kd, -2 mu_kd/var_kd]    0          1
//   tied       x_d                            -2 (P mu_k)_d                  x^T P x    1
//   full       [x_d, x_i x_j (i<=j)]          [-2 (P_k mu_k)_d, P_ij+P_ji]   0          1
//
// The M-step statistics of one row are r_nk * psi(x_n) with
//   psi = [1, x, |x|^2] (spherical) | [1, x, x^2] (diag) | [1, x] (tied) |
//         [1, x, x_i x_j (i<=j)] (full);
// their sum over n is the (B, K, F) stats buffer of the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/gmmxx_b200.h"

namespace gmmxx {

constexpr float kLog2Pi = 1.8378770664093453f;  // log(2*pi)

// Tile shape of the SIMT kernels: 64 rows x 64 components, 256 threads,
// 4x4 register micro-tiles.
constexpr int kBN = 64;
constexpr int kBK = 64;
constexpr int kThreads = 256;
constexpr int kFC = 32;  // feature chunk staged in shared memory

// SIMT windows (shapes outside return GMMXX_ERR_UNSUPPORTED).
constexpr int kMaxD = 128;      // spherical / diag / tied
constexpr int kMaxDFull = 26;   // full: stat width 1 + D + D(D+1)/2 <= 384
constexpr int kMaxStatChunks = 6;

__host__ __device__ inline int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }
__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

__host__ __device__ inline int feat_width(int cov, int D) {
  switch (cov) {
    case GMMXX_SPHERICAL: return D;
    case GMMXX_DIAG: return 2 * D;
    case GMMXX_TIED: return D;
    default: return D + D * (D + 1) / 2;
  }
}

__host__ __device__ inline int stat_width(int cov, int D) {
  switch (cov) {
    case GMMXX_SPHERICAL: return D + 2;
    case GMMXX_DIAG: return 2 * D + 1;
    case GMMXX_TIED: return D + 1;
    default: return 1 + D + D * (D + 1) / 2;
  }
}

// Tensor-core path window (em_tc.cu, em_tc_diag.cu): B == 1, N >= 64K;
// bf16 X: diag D == 64 with K <= 512, spherical D in {64, 128} with
// K <= 16384 (one pass up to 1024 components, else two passes per group);
// fp32 X: tied D == 64 with K <= 512.
constexpr int kTcMaxClusters = 160;
constexpr int kMaxClusterDiag = 4;
constexpr int kMaxClusterSph = 8;      // spherical one-pass: up to 8 CTAs (1024 components) per cluster
constexpr int kMaxComponentsSph = 16384;
// Spherical K > 1024: groups of 4 chunks (512 components).  Clusters of 4
// co-reside 33 at a time (132 SMs) against 15 of 8 (120 SMs), for the same
// work per CTA; the price is twice the passes over X, which HBM absorbs.
constexpr int kGroupChunks = 4;
// The row-statistics (first) pass of the diag-layout spherical kernel runs
// in groups of 2 chunks: 74 co-resident clusters of 2 use all 148 SMs, and
// the cluster exchange has one peer; its row partials take 8 B per row per
// group (32 groups at K = 8192).
constexpr int kRowStatChunks = 2;
__host__ __device__ inline bool tc_eligible(int cov, int64_t B, int64_t N, int64_t D, int64_t K) {
  if (B != 1 || N < 65536) return false;
  if (cov == GMMXX_DIAG) return D == 64 && K <= 128 * kMaxClusterDiag;
  if (cov == GMMXX_SPHERICAL) return (D == 64 || D == 128) && K <= kMaxComponentsSph;
  if (cov == GMMXX_TIED) return D == 64 && K <= 128 * kMaxClusterDiag;
  return false;
}
// the X dtype each covariance type's tensor-core kernel reads
__host__ __device__ inline bool tc_dtype_ok(int cov, int dt) {
  return cov == GMMXX_TIED ? dt == GMMXX_FLOAT32 : dt == GMMXX_BFLOAT16;
}
// 128-component chunks per group of one tensor-core launch: all of K up to
// 8 chunks (one pass), else kGroupChunks (spherical large K, two passes)
__host__ __device__ inline int tc_group_chunks(int64_t K) {
  const int nch = (int)((K + 127) / 128);
  return nch <= kMaxClusterSph ? nch : kGroupChunks;
}
__host__ __device__ inline int tc_groups(int64_t K) {
  const int nch = (int)((K + 127) / 128), gc = tc_group_chunks(K);
  return (nch + gc - 1) / gc;
}
// row-partial groups of the grouped spherical path: the larger of
// em_tc_kernel's groups (kGroupChunks) and the first pass's (kRowStatChunks)
__host__ __device__ inline int tc_rowstat_groups(int64_t K) {
  const int nch = (int)((K + 127) / 128);
  if (nch <= kMaxClusterSph) return 1;
  return (nch + kRowStatChunks - 1) / kRowStatChunks;
}
// three bf16 terms per weight: a_j (and v_j for diag), 16 KB blocks of
// [128 components][64 features]; tied: three blocks of [192 rows][64] (the
// components' weights and up to 64 rows of L^-1)
constexpr int kTiedTermBytes = 192 * 128;
__host__ __device__ inline int64_t tc_param_bytes(int cov, int D) {
  if (cov == GMMXX_TIED) return 3 * kTiedTermBytes;
  return (int64_t)(cov == GMMXX_DIAG ? 6 : 3) * (D / 64) * 16384;
}

// Row blocks of the CUDA-core M-step kernel (grid x): about 640 CTAs in total,
// fixed so that the workspace size and the launch agree (deterministic partials).
__host__ __device__ inline int64_t mstep_blocks(int64_t B, int64_t N, int64_t Kp) {
  const int64_t ktiles = Kp / 64, tiles = (N + 63) / 64;
  int64_t nblk = (640 + ktiles * B - 1) / (ktiles * B);
  if (nblk > tiles) nblk = tiles;
  if (nblk < 1) nblk = 1;
  return nblk;
}

// Row blocks of the X^T X kernel (tied covariance), fixed like mstep_blocks.
__host__ __device__ inline int64_t xx_blocks(int64_t B, int64_t N) {
  const int64_t tiles = (N + 63) / 64;
  int64_t nblk = (296 + B - 1) / B;
  if (nblk > tiles) nblk = tiles;
  if (nblk < 1) nblk = 1;
  return nblk;
}

// Per-component constants of the logit epilogue.
struct __align__(16) CompConst {
  float lw;   // log weight
  float s;    // distance scale (1/var for spherical, else 1)
  float ln;   // log-normaliser (D log 2pi + log det)
  float mpm;  // mu^T P mu (or |mu|^2 for spherical)
};

// Workspace layout (all offsets 256-byte aligned).
struct Layout {
  int64_t status;   // int[4]: [0] sticky status, [1] Cholesky jitter level
  int64_t cc;       // CompConst[B][K]
  int64_t wt;       // float[B][FE][Kp]  (feature-major component weights)
  int64_t prec;     // float[B][D][D] (tied) or float[B][K][D][D] (full)
  int64_t linv;     // float[B][D][D] inverse Cholesky factor L^-1 of the tied covariance
  int64_t lse;      // float[B][max(N, K)] (per-row lse; per-matrix log det while preparing)
  int64_t qrow;     // float[B][N] x^T P x per row (tied)
  int64_t mpart;    // float[B][mstep_blocks][Kp][F]  CUDA-core M-step partials
  int64_t llpart;   // double[B][ceil(N/64)]          per-CTA log-likelihood partials
  int64_t xxpart;   // float[B][xx_blocks][D][D]      X^T X partials (tied)
  // tensor-core path (present when the shape is eligible)
  int64_t tc_params;  // split-bf16 weight images [C][blocks][16 KB]
  int64_t tc_consts;  // float[C][3][128]
  int64_t tc_part;    // float[kTcMaxClusters][C*128][F]
  int64_t tc_part_ll; // double[kTcMaxClusters]
  int64_t tc_rowstat; // float2[groups][N] per-row partials of the grouped large-K path
  int64_t tc_lse;     // float[N]          per-row log-sum-exp (log2 units), grouped path
  int tc_cluster;     // C (0: tensor-core path not available)
  int tc_chunks;      // 128-component chunks of K
  int64_t total;
  int64_t Kp;
  int FE;
};

inline Layout make_layout(int cov, int64_t B, int64_t N, int64_t D, int64_t K) {
  Layout L;
  auto al = [](int64_t v) { return round_up(v, 256); };
  L.Kp = round_up(K, kBK);
  L.FE = feat_width(cov, (int)D);
  int64_t off = 0;
  L.status = off; off += al(16);
  L.cc = off; off += al(B * K * (int64_t)sizeof(CompConst));
  L.wt = off; off += al(B * L.FE * L.Kp * 4);
  L.prec = off;
  if (cov == GMMXX_TIED) off += al(B * D * D * 4);
  else if (cov == GMMXX_FULL) off += al(B * K * D * D * 4);
  L.linv = off;
  if (cov == GMMXX_TIED) off += al(B * D * D * 4);
  L.lse = off; off += al(B * (N > K ? N : K) * 4);
  L.qrow = off;
  if (cov == GMMXX_TIED) off += al(B * N * 4);
  L.mpart = off; off += al(B * mstep_blocks(B, N, L.Kp) * L.Kp * stat_width(cov, (int)D) * 4);
  L.llpart = off; off += al(B * ((N + 63) / 64) * 8);
  L.xxpart = off;
  if (cov == GMMXX_TIED) off += al(B * xx_blocks(B, N) * D * D * 4);
  L.tc_cluster = L.tc_chunks = 0;
  L.tc_params = L.tc_consts = L.tc_part = L.tc_part_ll = L.tc_rowstat = L.tc_lse = 0;
  if (tc_eligible(cov, B, N, D, K)) {
    const int nch = (int)((K + 127) / 128);
    const int G = tc_rowstat_groups(K) > tc_groups(K) ? tc_rowstat_groups(K) : tc_groups(K);
    const int C = tc_group_chunks(K);
    L.tc_cluster = C;
    L.tc_chunks = nch;
    L.tc_params = off; off += al((int64_t)nch * tc_param_bytes(cov, (int)D));
    L.tc_consts = off; off += al((int64_t)nch * 3 * 128 * 4);
    L.tc_part = off; off += al((int64_t)kTcMaxClusters * C * 128 * stat_width(cov, (int)D) * 4);
    L.tc_part_ll = off; off += al((int64_t)kTcMaxClusters * kMaxClusterSph * 8);  // per cluster (and rank)
    if (G > 1) {
      L.tc_rowstat = off; off += al((int64_t)G * N * 8);
      L.tc_lse = off; off += al(N * 4);
    }
  }
  L.total = off;
  return L;
}

// --- dtype-generic loads -----------------------------------------------------

__device__ __forceinline__ float load_x(const void* p, int64_t i, int dt) {
  if (dt == GMMXX_FLOAT32) return static_cast<const float*>(p)[i];
  if (dt == GMMXX_BFLOAT16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum; every thread gets the result.  `red` needs blockDim/32 slots.
template <typename V>
__device__ V block_sum(V v, V* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  V t = 0;
  for (int i = 0; i < nw; ++i) t += red[i];
  __syncthreads();
  return t;
}

}  // namespace gmmxx

// --- host-side error plumbing (defined in capi.cu) ---------------------------
namespace gmmxx {
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);
}  // namespace gmmxx
