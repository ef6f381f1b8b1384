// rows_api.cuh -- argument block and launchers of the row-tile kernels
// (estep_simt.cu), shared with the C ABI layer.
#pragma once

#include "gmm_common.cuh"

namespace gmmxx {

struct RowArgs {
  const void* x;
  int dt;
  int64_t N;
  int D, K, FE;
  int64_t Kp;
  const CompConst* cc;  // [B][K]
  const float* wt;      // [B][FE][Kp]
  const float* prec;    // tied precision [B][D][D]
  const float* lse_in;  // [B][N]
  float* lse_out;       // [B][N]
  double* ll;           // log-likelihood accumulator (may be null)
  double* ll_part;      // per-CTA log-likelihood partials [B][gridDim.x] (LSE mode, may be null)
  float* part;          // M-step partials [B][part_blocks][Kp][FM]
  int64_t* labels;      // [B][N]
  float* out;           // [B][N][K]
  float* stats;         // [B][K][FM]
  int FM;
  int64_t rows_per_cta;
  int64_t part_blocks;
  // tied: x^T P x per row, written by the LSE pass and read by the M-step
  // instead of being recomputed for every component tile (may be null)
  float* q_out;         // [B][N]
  const float* q_in;    // [B][N]
  // approximate top-k EM: per row, its top_k components and their
  // responsibilities, written by the selection pass and read by the M-step
  int top_k;
  int32_t* topk_idx;    // [B][N][top_k] (-1: no entry)
  float* topk_r;        // [B][N][top_k]
};

// largest top_k of the approximate EM passes (the selection pass keeps each
// row's sorted list in shared memory)
constexpr int kMaxTopK = 64;
__host__ __device__ inline int64_t topk_scratch_bytes(int64_t B, int64_t N, int64_t top_k) {
  return 2 * round_up(B * N * top_k * 4, 256);
}

enum { MODE_LSE = 0, MODE_ARGMAX = 1, MODE_RESP = 2 };

int launch_rows(int cov, int mode, const RowArgs& a, int B, cudaStream_t st);
// records the grid it chose in a.rows_per_cta (read by launch_stats_reduce)
int launch_mstep(int cov, RowArgs& a, int B, cudaStream_t st);
// stats += sum of the M-step partials, ll += sum of the LSE partials (fixed order)
int launch_stats_reduce(const RowArgs& a, int B, cudaStream_t st);
// K <= 64: statistics and log-likelihood in one pass, then their fixed-order
// reduction (replaces launch_rows(LSE) + launch_mstep + launch_stats_reduce)
int launch_em_small(int cov, const RowArgs& a, int B, cudaStream_t st);
// approximate top-k EM: the selection pass (top_k lists, log-likelihood
// partials as the LSE pass writes them) and the M-step over the lists; then
// launch_stats_reduce as for exact EM
int launch_topk_rows(int cov, const RowArgs& a, int B, cudaStream_t st);
int launch_topk_mstep(int cov, RowArgs& a, int B, cudaStream_t st);

}  // namespace gmmxx
