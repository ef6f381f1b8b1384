// kmeans.cu -- k-means initialisation on the GPU: greedy k-means++ seeding
// and the per-label statistics of Lloyd iterations and of the hard-label
// initial parameters.
//
// k-means++ (reference: gmmxx/torch_fallback.py:1390-1451,
// _kmeans_plus_plus_init_means).  On a row sample S (B problems of S rows):
// the first centre is a given row; then for every further centre c the
// caller's uniforms u[c][b][t] (t < L local trials) pick L candidate rows by
// inverse-CDF sampling of the rows' squared distance to their closest centre
// (first row whose running sum reaches u * total), each candidate's
// potential sum_n min(closest_n, |s_n - s_cand|^2) is formed, and the
// candidate with the smallest potential (first on ties) becomes the centre.
// One step is four launches: draw (one block per problem), trial potentials
// (grid over rows, per-block partials), pick (one block per problem, fixed
// order), update of the closest distances (grid over rows, per-block sums
// for the next draw).  Running sums, totals and potentials accumulate in
// float64 and are rounded to float32 where they are compared, as torch's CPU
// cumsum / sum of float32 do (double accumulator), so a seeded call picks the
// reference's rows.  Every sum is a fixed-order reduction (bitwise
// repeatable).
//
// Label statistics (Lloyd's centroid update, reference hard-label init
// statistics torch_fallback.py:1454-1581): per label its row count, the sum
// of its rows and, by mode, the per-dimension sum of (x - mu_label)^2 or the
// sums of x_i x_j (i <= j).  A block owns a contiguous row range; thread l
// owns label l and walks the range in order, so every partial is a
// fixed-order sum; the partials are reduced in block order.
#include "gmm_common.cuh"

#include <math.h>

namespace gmmxx {
namespace {

constexpr int kKppThreads = 256;
constexpr int kKppMaxTrials = 16;

// squared distance of sample row n to sample row m (fp32, dimension order)
__device__ __forceinline__ float row_dist2(const float* s, int64_t n, int64_t m, int D) {
  const float* a = s + n * D;
  const float* b = s + m * D;
  float acc = 0.f;
  for (int d = 0; d < D; ++d) {
    const float t = a[d] - b[d];
    acc = fmaf(t, t, acc);
  }
  return acc;
}

// Rows per block of the row-parallel k-means++ kernels (fixed, so that the
// partial sums and their reduction order depend only on S).
__host__ __device__ inline int kpp_blocks(int64_t S) { return (int)((S + kKppThreads - 1) / kKppThreads); }

// closest[n] = min(closest[n], |s_n - s_best|^2) (or = for the first centre),
// and per-block sums of closest for the next draw
__global__ void kpp_update_kernel(const float* sample, int64_t S, int D, const int64_t* best, int first,
                                  float* closest, double* bsum) {
  __shared__ double red[kKppThreads / 32];
  const int b = blockIdx.y;
  const float* s = sample + (int64_t)b * S * D;
  const int64_t n = (int64_t)blockIdx.x * kKppThreads + threadIdx.x;
  double v = 0.0;
  if (n < S) {
    const float dn = row_dist2(s, n, best[b], D);
    float* c = closest + (int64_t)b * S + n;
    const float cv = first ? dn : fminf(*c, dn);
    *c = cv;
    v = (double)cv;
  }
  v = warp_sum_d(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kKppThreads / 32; ++w) t += red[w];
    bsum[(int64_t)b * gridDim.x + blockIdx.x] = t;
  }
}

// L candidates of centre c for problem b: the first row whose running sum of
// closest distances reaches u * total (clamped to the last row; row 0 when
// every distance is zero)
__global__ void kpp_draw_kernel(const float* closest, const double* bsum, int64_t S, int nblk, int L,
                                const float* u, int64_t* cand) {
  const int b = blockIdx.x;
  const float* cl = closest + (int64_t)b * S;
  const double* bs = bsum + (int64_t)b * nblk;
  __shared__ float total;
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < nblk; ++i) t += bs[i];
    total = (float)t;
  }
  __syncthreads();
  for (int t = threadIdx.x; t < L; t += blockDim.x) {
    int64_t idx = 0;
    if (total > 0.f) {
      const float target = u[(int64_t)b * L + t] * total;
      double run = 0.0;  // the running sum; compared as the float32 it rounds to
      int blk = 0;
      while (blk < nblk - 1 && (float)(run + bs[blk]) < target) run += bs[blk++];
      int64_t n = (int64_t)blk * kKppThreads;
      const int64_t end = n + kKppThreads < S ? n + kKppThreads : S;
      while (n < end - 1 && (float)(run + (double)cl[n]) < target) run += (double)cl[n++];
      idx = n;
    }
    cand[(int64_t)b * L + t] = idx;
  }
}

// per-block partial potentials of the L candidates
__global__ void kpp_trials_kernel(const float* sample, int64_t S, int D, int L, const float* closest,
                                  const int64_t* cand, double* part) {
  __shared__ double red[kKppThreads / 32][kKppMaxTrials];
  const int b = blockIdx.y;
  const float* s = sample + (int64_t)b * S * D;
  const int64_t n = (int64_t)blockIdx.x * kKppThreads + threadIdx.x;
  const float cn = n < S ? closest[(int64_t)b * S + n] : 0.f;
  for (int t = 0; t < L; ++t) {
    double v = n < S ? (double)fminf(cn, row_dist2(s, n, cand[(int64_t)b * L + t], D)) : 0.0;
    v = warp_sum_d(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5][t] = v;
  }
  __syncthreads();
  if (threadIdx.x < L) {
    double t = 0.0;
    for (int w = 0; w < kKppThreads / 32; ++w) t += red[w][threadIdx.x];
    part[((int64_t)b * gridDim.x + blockIdx.x) * L + threadIdx.x] = t;
  }
}

// the candidate of smallest potential (first on ties) becomes centre c
__global__ void kpp_pick_kernel(const float* sample, int64_t S, int D, int L, int nblk, const double* part,
                                const int64_t* cand, int c, int K, int64_t* best, float* centers) {
  const int b = blockIdx.x;
  __shared__ int64_t pick;
  if (threadIdx.x == 0) {
    float bp = INFINITY;
    int bt = 0;
    for (int t = 0; t < L; ++t) {
      double pot = 0.0;
      for (int i = 0; i < nblk; ++i) pot += part[((int64_t)b * nblk + i) * L + t];
      if ((float)pot < bp) { bp = (float)pot; bt = t; }  // compared as float32 potentials
    }
    pick = cand[(int64_t)b * L + bt];
    best[b] = pick;
  }
  __syncthreads();
  const float* row = sample + ((int64_t)b * S + pick) * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) centers[((int64_t)b * K + c) * D + d] = row[d];
}

// ---------------------------------------------------------------------------
// label statistics
// ---------------------------------------------------------------------------

// Per (problem, block): for label l = threadIdx.x (K <= blockDim.x), the
// fixed-order sums over the block's rows with that label of
//   mode 0: [1, x]                    (F = 1 + D)
//   mode 1: [1, x, (x - mu_l)^2]      (F = 1 + 2D)
//   mode 2: [1, x, x_i x_j (i <= j)]  (F = 1 + D + D(D+1)/2)
// written to part[b][block][l][F] (accumulated in place there).
__global__ void label_stats_kernel(const void* x, int dt, int64_t N, int D, int K, const int64_t* labels,
                                   const float* means, int mode, int F, int64_t rows_per_block, float* part) {
  extern __shared__ int64_t lab[];  // a tile of labels
  constexpr int kTile = 2048;
  const int b = blockIdx.y;
  const int l = threadIdx.x;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_block;
  const int64_t r1 = r0 + rows_per_block < N ? r0 + rows_per_block : N;
  float* acc = part + (((int64_t)b * gridDim.x + blockIdx.x) * K + (l < K ? l : 0)) * F;
  if (l < K)
    for (int f = 0; f < F; ++f) acc[f] = 0.f;
  const float* mu = means != nullptr ? means + ((int64_t)b * K + (l < K ? l : 0)) * D : nullptr;
  for (int64_t t0 = r0; t0 < r1; t0 += kTile) {
    const int64_t t1 = t0 + kTile < r1 ? t0 + kTile : r1;
    __syncthreads();
    for (int64_t i = t0 + threadIdx.x; i < t1; i += blockDim.x) lab[i - t0] = labels[(int64_t)b * N + i];
    __syncthreads();
    if (l >= K) continue;
    for (int64_t i = t0; i < t1; ++i) {
      if (lab[i - t0] != l) continue;
      const int64_t base = ((int64_t)b * N + i) * D;
      acc[0] += 1.f;
      if (mode == 2) {
        float xr[kMaxDFull];  // the row, read once
        for (int d = 0; d < D; ++d) xr[d] = load_x(x, base + d, dt);
        int p = 1 + D;
        for (int di = 0; di < D; ++di) {
          acc[1 + di] += xr[di];
          for (int dj = di; dj < D; ++dj) acc[p++] += xr[di] * xr[dj];
        }
      } else {
        for (int d = 0; d < D; ++d) {
          const float xd = load_x(x, base + d, dt);
          acc[1 + d] += xd;
          if (mode == 1) {
            const float e = xd - mu[d];
            acc[1 + D + d] += e * e;
          }
        }
      }
    }
  }
}

// stats[b][l][f] = sum over blocks of part[b][block][l][f] (block order)
__global__ void label_stats_reduce_kernel(const float* part, int nblk, int K, int F, int64_t B, float* stats) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * K * F) return;
  const int64_t b = i / ((int64_t)K * F), r = i - b * K * F;
  float s = 0.f;
  for (int j = 0; j < nblk; ++j) s += part[((int64_t)b * nblk + j) * K * F + r];
  stats[i] = s;
}

int64_t label_stats_blocks(int64_t B, int64_t N) {
  int64_t nb = (296 + B - 1) / B;  // about two blocks per SM in all
  const int64_t need = (N + 4095) / 4096;
  if (nb > need) nb = need;
  return nb < 1 ? 1 : nb;
}

int label_stats_width(int mode, int D) { return mode == 0 ? 1 + D : mode == 1 ? 1 + 2 * D : 1 + D + D * (D + 1) / 2; }

}  // namespace
}  // namespace gmmxx

using namespace gmmxx;

extern "C" {

size_t gmmxx_kmeans_pp_workspace_bytes(int64_t B, int64_t S, int64_t trials) {
  if (B <= 0 || S <= 0 || trials <= 0) return 0;
  const int64_t nb = kpp_blocks(S);
  auto al = [](int64_t v) { return round_up(v, 256); };
  return (size_t)(al(B * S * 4) + al(B * nb * 8) + al(B * nb * trials * 8) + al(B * trials * 8) + al(B * 8));
}

int gmmxx_kmeans_pp(const float* sample, int64_t B, int64_t S, int64_t D, int64_t K, int64_t trials,
                    const int64_t* first_idx, const float* uniforms, float* centers_out, void* workspace,
                    size_t workspace_bytes, void* stream) {
  if (B <= 0 || S <= 0 || D <= 0 || K <= 0 || K > S)
    return set_error(GMMXX_ERR_INVALID, "k-means++: bad sizes B=%lld S=%lld D=%lld K=%lld", (long long)B,
                     (long long)S, (long long)D, (long long)K);
  if (trials < 1 || trials > kKppMaxTrials)
    return set_error(GMMXX_ERR_UNSUPPORTED, "k-means++: %lld local trials (1 .. %d)", (long long)trials,
                     kKppMaxTrials);
  if (B > 65535) return set_error(GMMXX_ERR_UNSUPPORTED, "k-means++: B=%lld too large", (long long)B);
  if (sample == nullptr || first_idx == nullptr || centers_out == nullptr || (K > 1 && uniforms == nullptr))
    return set_error(GMMXX_ERR_INVALID, "k-means++: NULL argument");
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return set_error(GMMXX_ERR_INVALID, "k-means++: workspace must be 256-byte aligned");
  if (workspace_bytes < gmmxx_kmeans_pp_workspace_bytes(B, S, trials))
    return set_error(GMMXX_ERR_WORKSPACE, "k-means++: workspace of %zu bytes is too small", workspace_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nb = kpp_blocks(S);
  const int L = (int)trials;
  auto al = [](int64_t v) { return round_up(v, 256); };
  char* ws = static_cast<char*>(workspace);
  float* closest = reinterpret_cast<float*>(ws);
  double* bsum = reinterpret_cast<double*>(ws + al(B * S * 4));
  double* part = reinterpret_cast<double*>(ws + al(B * S * 4) + al(B * nb * 8));
  int64_t* cand = reinterpret_cast<int64_t*>(ws + al(B * S * 4) + al(B * nb * 8) + al(B * nb * trials * 8));
  int64_t* best = reinterpret_cast<int64_t*>(ws + al(B * S * 4) + al(B * nb * 8) + al(B * nb * trials * 8) +
                                             al(B * trials * 8));
  const dim3 rows(nb, (unsigned)B);
  // first centre: the given rows
  cudaError_t e = cudaMemcpyAsync(best, first_idx, B * sizeof(int64_t), cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return set_error(GMMXX_ERR_CUDA, "k-means++: %s", cudaGetErrorString(e));
  kpp_pick_kernel<<<(unsigned)B, 128, 0, st>>>(sample, S, (int)D, 1, 0, nullptr, best, 0, (int)K, best,
                                              centers_out);
  if (int rc = check_launch("kpp_pick_kernel")) return rc;
  kpp_update_kernel<<<rows, kKppThreads, 0, st>>>(sample, S, (int)D, best, 1, closest, bsum);
  if (int rc = check_launch("kpp_update_kernel")) return rc;
  for (int c = 1; c < K; ++c) {
    kpp_draw_kernel<<<(unsigned)B, 32, 0, st>>>(closest, bsum, S, nb, L, uniforms + (int64_t)(c - 1) * B * L, cand);
    kpp_trials_kernel<<<rows, kKppThreads, 0, st>>>(sample, S, (int)D, L, closest, cand, part);
    kpp_pick_kernel<<<(unsigned)B, 128, 0, st>>>(sample, S, (int)D, L, nb, part, cand, c, (int)K, best,
                                                centers_out);
    kpp_update_kernel<<<rows, kKppThreads, 0, st>>>(sample, S, (int)D, best, 0, closest, bsum);
    if (int rc = check_launch("k-means++ step")) return rc;
  }
  return GMMXX_OK;
}

int64_t gmmxx_label_stats_width(int mode, int64_t D) {
  if (mode < 0 || mode > 2 || D <= 0) return -1;
  return label_stats_width(mode, (int)D);
}

size_t gmmxx_label_stats_workspace_bytes(int mode, int64_t B, int64_t N, int64_t D, int64_t K) {
  if (mode < 0 || mode > 2 || B <= 0 || N < 0 || D <= 0 || K <= 0) return 0;
  return (size_t)round_up(B * label_stats_blocks(B, N) * K * label_stats_width(mode, (int)D) * 4, 256);
}

int gmmxx_label_stats(int x_dtype, const void* x, int64_t B, int64_t N, int64_t D, int64_t K, const int64_t* labels,
                      const float* means, int mode, float* stats_out, void* workspace, size_t workspace_bytes,
                      void* stream) {
  if (x_dtype < GMMXX_FLOAT32 || x_dtype > GMMXX_FLOAT16) return set_error(GMMXX_ERR_INVALID, "unknown x dtype");
  if (mode < 0 || mode > 2) return set_error(GMMXX_ERR_INVALID, "label statistics mode %d", mode);
  if (B <= 0 || N < 0 || D <= 0 || K <= 0) return set_error(GMMXX_ERR_INVALID, "label statistics: bad sizes");
  if (K > 1024) return set_error(GMMXX_ERR_UNSUPPORTED, "label statistics: K=%lld > 1024", (long long)K);
  if (B > 65535) return set_error(GMMXX_ERR_UNSUPPORTED, "label statistics: B too large");
  if (mode == 2 && D > kMaxDFull) return set_error(GMMXX_ERR_UNSUPPORTED, "label statistics: D=%lld > %d for mode 2",
                                                   (long long)D, kMaxDFull);
  if (stats_out == nullptr || (N > 0 && (x == nullptr || labels == nullptr)) || (mode == 1 && means == nullptr))
    return set_error(GMMXX_ERR_INVALID, "label statistics: NULL argument");
  if (workspace == nullptr || workspace_bytes < gmmxx_label_stats_workspace_bytes(mode, B, N, D, K))
    return set_error(GMMXX_ERR_WORKSPACE, "label statistics: workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int F = label_stats_width(mode, (int)D);
  const int64_t nb = label_stats_blocks(B, N);
  const int64_t rpb = N > 0 ? (N + nb - 1) / nb : 1;
  float* part = static_cast<float*>(workspace);
  const int threads = (int)round_up(K, 32);
  label_stats_kernel<<<dim3((unsigned)nb, (unsigned)B), threads, 2048 * sizeof(int64_t), st>>>(
      x, x_dtype, N, (int)D, (int)K, labels, means, mode, F, rpb, part);
  if (int rc = check_launch("label_stats_kernel")) return rc;
  const int64_t tot = B * K * F;
  label_stats_reduce_kernel<<<(unsigned)ceil_div(tot, 256), 256, 0, st>>>(part, (int)nb, (int)K, F, B, stats_out);
  return check_launch("label_stats_reduce_kernel");
}

}  // extern "C"
