// tc_api.cuh -- argument blocks of the tensor-core EM kernel (em_tc.cu),
// shared with the C ABI layer.
#pragma once

#include "gmm_common.cuh"

namespace gmmxx {
namespace tc {

constexpr int kMaxClusters = kTcMaxClusters;  // upper bound of co-resident clusters (partials buffer)

// Kernel parameters (passed by value).
struct TcArgs {
  int64_t N;
  int64_t Kp;        // padded component count of the partials (cluster_size * 128)
  int F;             // statistics width
  int cluster_size;  // CTAs per cluster = ceil(K / 128)
  const char* params;
  const float* consts;
  float* part;       // [kMaxClusters][Kp][F]
  double* part_ll;   // [kMaxClusters]
  int* status;       // sticky workspace status word
};

struct TcLaunch {
  const void* x;
  int64_t N;
  int D, K;
  int64_t Kp_table;  // padded K of the CUDA-core component table
  int64_t Kp_part;
  int F;
  int cluster_size;
  const float* wt;
  const CompConst* cc;
  char* params;
  float* consts;
  float* part;
  double* part_ll;
  int* status;
  float* stats;
  double* ll;
};

int launch_em_tc(int cov, const TcLaunch& L, cudaStream_t st);

}  // namespace tc
}  // namespace gmmxx
