// tc_api.cuh -- argument blocks of the tensor-core EM kernel (em_tc.cu),
// shared with the C ABI layer.
#pragma once

#include "gmm_common.cuh"

#include <cuda.h>

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
  // grouped large-K passes (spherical, K > 1024): the cluster covers chunks
  // [chunk0, chunk0 + cluster_size) of 128 components
  int chunk0;
  const float* lse_in;  // external per-row log-sum-exp over all K (log2 units)
  float2* rowstat;      // per-row (max, scaled sum) over this group (log2 units)
  uint64_t wait_ns;     // limit of every bounded wait (diag kernel)
  int test_stall;       // test hook (diag kernel): the producer issues no X loads
  // inference modes of the diag kernel (TcLaunch::infer != 0)
  int K;                // real component count (row stride of out_f for predict_proba)
  float* out_f;         // [N] log-sum-exp (natural log) or [N][K] responsibilities
  int64_t* out_i;       // [N] labels
  int out_vec;          // out_f 16-byte aligned and K % 4 == 0: 16-byte stores allowed
  // spherical per-row passes (row statistics / argmax): where the row's
  // result goes -- 0: rowstat[row] (per-group partial), 1: out_f[row] =
  // natural-log log-sum-exp, 2: out_f[row] = log-sum-exp in log2 units,
  // 3: out_i[row] = label
  int row_out;
  // > 0: launched without thread-block clusters, CTA i acting as rank
  // i % vcluster of cluster i / vcluster (passes that exchange nothing)
  int vcluster;
};

struct TcLaunch {
  const void* x;
  int64_t N;
  int D, K;
  int64_t Kp_table;  // padded K of the CUDA-core component table
  int64_t Kp_part;
  int F;
  int cluster_size;
  int nchunks;       // 128-component chunks of the weight images (>= cluster_size)
  const float* wt;
  const CompConst* cc;
  const float* linv;  // tied: L^-1 of the covariance (D x D, row-major)
  char* params;
  float* consts;
  float* part;
  double* part_ll;
  int* status;
  float* stats;
  double* ll;
  float2* rowstat;   // [groups][N] (grouped large-K path)
  float* lse;        // [N]         per-row log-sum-exp, log2 units (grouped path; spherical predict_proba)
  uint64_t wait_ns;  // bounded-wait limit (0: 2 s)
  int test_stall;    // GMMXX_B200_TEST_STALL=1: make the diag kernel's waits run out
  // diag kernel only: 0 = EM statistics; inference without the M-step:
  // 1 = per-row log-sum-exp into out_f, 2 = labels into out_i,
  // 3 = responsibilities exp(logit - lse) into out_f [N][K]
  int infer;
  float* out_f;
  int64_t* out_i;
};

int launch_em_tc(int cov, const TcLaunch& L, cudaStream_t st);

// pieces shared by the tensor-core kernels (em_tc.cu, em_tc_diag.cu)
int launch_em_tc_diag(const TcLaunch& L, cudaStream_t st);
int launch_em_tc_tied(const TcLaunch& L, cudaStream_t st);
int launch_em_tc_sph128(const TcLaunch& L, cudaStream_t st);  // spherical D = 128 EM and inference, diag-kernel layout
// grouped large-K passes: each row's log-sum-exp over the groups' row
// statistics into L.lse (log2 units) and the log-likelihood into *L.ll
int launch_rowstat_combine(const TcLaunch& L, int groups, cudaStream_t st);
// grouped inference: fold the groups' row statistics into labels (infer 2),
// the natural-log log-sum-exp in L.out_f (1) or the log2 one in L.lse (3)
int launch_infer_combine(const TcLaunch& L, int groups, int infer, cudaStream_t st);
int launch_tc_pack(int cov, int db, const TcLaunch& L, cudaStream_t st);  // weight images + logit constants
// spherical D = 128, grouped second pass over chunks [chunk0, chunk0 + csize):
// responsibilities from L.lse and the group's M-step statistics partials
// (em_tc_sph_ext_kernel, components on the MMA's M dimension); *ncl_out
// receives the number of virtual clusters (partials rows)
int launch_sph_ext(const TcLaunch& L, const CUtensorMap& tmap, int chunk0, int csize, cudaStream_t st, int* ncl_out);
bool sph_ext_enabled();  // GMMXX_B200_SPH_PASS2=diag keeps em_tc_diag_kernel's pass
// X boxes of 128 rows x 128 bytes with 128-byte swizzle: 64 bf16 columns, or
// (fp32) 32 columns -- an fp32 tile of 64 columns is two boxes
int make_x_tensor_map(const TcLaunch& L, CUtensorMap* tmap, bool fp32 = false);
// fixed-order partials -> stats; n_ll log-likelihood partials (default: one per cluster)
int launch_tc_reduce(const TcLaunch& L, int ncl, cudaStream_t st, int n_ll = -1);
// Sets the kernel's shared-memory attribute and returns in *ncl_out how many
// clusters of L.cluster_size CTAs (threads x smem each) run at once, capped by
// the partials buffer and the tile count.
int clustered_launch(const void* kern, int threads, int smem, const TcLaunch& L, int* ncl_out);

}  // namespace tc
}  // namespace gmmxx
