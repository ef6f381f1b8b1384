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
};

enum { MODE_LSE = 0, MODE_ARGMAX = 1, MODE_RESP = 2 };

int launch_rows(int cov, int mode, const RowArgs& a, int B, cudaStream_t st);
// records the grid it chose in a.rows_per_cta (read by launch_stats_reduce)
int launch_mstep(int cov, RowArgs& a, int B, cudaStream_t st);
// stats += sum of the M-step partials, ll += sum of the LSE partials (fixed order)
int launch_stats_reduce(const RowArgs& a, int B, cudaStream_t st);
// K <= 64: statistics and log-likelihood in one pass, then their fixed-order
// reduction (replaces launch_rows(LSE) + launch_mstep + launch_stats_reduce)
int launch_em_small(int cov, const RowArgs& a, int B, cudaStream_t st);

}  // namespace gmmxx
