// capi.cu -- the extern "C" boundary (include/gmmxx_b200.h): argument
// validation, workspace carving, kernel orchestration and error reporting.
//
// Error convention (mirrors the reference's TORCH_CHECK -> RuntimeError,
// gmmxx/csrc/canary/canary.cu:28-46): every entry point returns a status code;
// the message of the last failure on the calling host thread is kept in a
// thread-local buffer exposed by gmmxx_last_error().
#include "gmm_common.cuh"

#include <stdarg.h>
#include <stdio.h>

namespace gmmxx {

static thread_local char g_err[1024] = {0};
// statistics path of the last successful gmmxx_em_accumulate on this thread
// (gmmxx_last_accumulate_path): -1 none, 0 CUDA cores, 1 tensor cores,
// 2 CUDA cores after the tensor-core launch found no co-resident cluster
static thread_local int g_last_path = -1;

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(GMMXX_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return GMMXX_OK;
}

int launch_prepare(int cov, int64_t B, int64_t D, int64_t K, float* means, float* covp, float* weights,
                   float reg, float mw, int prologue, const Layout& L, char* ws, cudaStream_t st);
int launch_finalize(int cov, int64_t B, int64_t D, int64_t K, int64_t n_total, const float* stats,
                    const double* ll, const float* xx, float reg, float mw, float* means, float* covp,
                    float* weights, float* lb_out, cudaStream_t st);
int launch_canary(const int32_t* in, int32_t* out, int64_t n, int32_t offset, cudaStream_t st);
int launch_xx_total(const void* x, int dt, int64_t B, int64_t N, int D, float* xx, float* part, cudaStream_t st);

}  // namespace gmmxx

#include "rows_api.cuh"
#include "tc_api.cuh"

#include <stdlib.h>
#include <string.h>

using namespace gmmxx;

namespace {

int check_shape(int cov, int dt, int64_t B, int64_t N, int64_t D, int64_t K) {
  if (cov < GMMXX_SPHERICAL || cov > GMMXX_FULL) return set_error(GMMXX_ERR_INVALID, "unknown covariance type %d", cov);
  if (dt < GMMXX_FLOAT32 || dt > GMMXX_FLOAT16) return set_error(GMMXX_ERR_INVALID, "unknown x dtype %d", dt);
  if (B <= 0 || N < 0 || D <= 0 || K <= 0)
    return set_error(GMMXX_ERR_INVALID, "bad sizes B=%lld N=%lld D=%lld K=%lld", (long long)B, (long long)N,
                     (long long)D, (long long)K);
  const int64_t maxd = (cov == GMMXX_FULL) ? kMaxDFull : kMaxD;
  if (D > maxd)
    return set_error(GMMXX_ERR_UNSUPPORTED, "D=%lld exceeds the engine window (D <= %lld for this covariance type)",
                     (long long)D, (long long)maxd);
  if (K > (1 << 24)) return set_error(GMMXX_ERR_UNSUPPORTED, "K=%lld too large", (long long)K);
  if (B > 65535) return set_error(GMMXX_ERR_UNSUPPORTED, "B=%lld too large (max 65535)", (long long)B);
  return GMMXX_OK;
}

int check_ws(const void* ws, size_t bytes, const Layout& L) {
  if (ws == nullptr) return set_error(GMMXX_ERR_INVALID, "workspace is NULL");
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) return set_error(GMMXX_ERR_INVALID, "workspace must be 256-byte aligned");
  if ((int64_t)bytes < L.total)
    return set_error(GMMXX_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %lld bytes required", bytes,
                     (long long)L.total);
  return GMMXX_OK;
}

// Kernel selection (GMMXX_B200_KERNEL): "auto" (default) uses the
// tensor-core kernel where the shape allows it and the CUDA-core kernels
// otherwise; "simt" always uses the exact-fp32 CUDA-core kernels; "tc"
// requires the tensor-core kernel and fails if it cannot run.
int kernel_mode() {
  const char* e = getenv("GMMXX_B200_KERNEL");
  if (e == nullptr) return 0;
  if (strcmp(e, "simt") == 0) return 1;
  if (strcmp(e, "tc") == 0) return 2;
  return 0;
}

#define GMMXX_REQUIRE(p, name) \
  if ((p) == nullptr) return set_error(GMMXX_ERR_INVALID, "%s is NULL", name)

RowArgs make_rows(int cov, int dt, const void* x, int64_t B, int64_t N, int64_t D, int64_t K, const Layout& L,
                  char* ws) {
  RowArgs a{};
  a.x = x;
  a.dt = dt;
  a.N = N;
  a.D = (int)D;
  a.K = (int)K;
  a.FE = L.FE;
  a.Kp = L.Kp;
  a.cc = reinterpret_cast<const CompConst*>(ws + L.cc);
  a.wt = reinterpret_cast<const float*>(ws + L.wt);
  a.prec = reinterpret_cast<const float*>(ws + L.prec);
  a.FM = stat_width(cov, (int)D);
  return a;
}

// tensor-core launch block over the workspace buffers of layout L
tc::TcLaunch make_tc(int cov, const void* x, int64_t N, int64_t D, int64_t K, const Layout& L, char* ws) {
  tc::TcLaunch t{};
  t.x = x;
  t.N = N;
  t.D = (int)D;
  t.K = (int)K;
  t.Kp_table = L.Kp;
  t.Kp_part = (int64_t)L.tc_cluster * 128;  // per group for the grouped large-K path
  t.F = stat_width(cov, (int)D);
  t.cluster_size = L.tc_cluster;
  t.nchunks = L.tc_chunks;
  t.rowstat = L.tc_rowstat ? reinterpret_cast<float2*>(ws + L.tc_rowstat) : nullptr;
  // the grouped path's per-row buffer, else the CUDA-core path's (N floats)
  t.lse = reinterpret_cast<float*>(ws + (L.tc_lse ? L.tc_lse : L.lse));
  t.wt = reinterpret_cast<const float*>(ws + L.wt);
  t.cc = reinterpret_cast<const CompConst*>(ws + L.cc);
  t.linv = cov == GMMXX_TIED ? reinterpret_cast<const float*>(ws + L.linv) : nullptr;
  t.params = ws + L.tc_params;
  t.consts = reinterpret_cast<float*>(ws + L.tc_consts);
  t.part = reinterpret_cast<float*>(ws + L.tc_part);
  t.part_ll = reinterpret_cast<double*>(ws + L.tc_part_ll);
  t.status = reinterpret_cast<int*>(ws + L.status);
  t.wait_ns = 2000000000ull;
  return t;
}

// Inference on the tensor-core kernels (bf16 X, the EM kernels' shape
// windows): labels (mode 2), log-sum-exp (1) or responsibilities (3); diag
// in one pass, spherical in per-row passes per group of components.  *done
// stays false when the call belongs to the CUDA-core kernels.
int tc_infer(int cov, int dt, const void* x, int64_t N, int64_t D, int64_t K, const Layout& L, char* ws, int infer,
             float* out_f, int64_t* out_i, cudaStream_t st, bool* done) {
  *done = false;
  const int km = kernel_mode();
  if ((cov != GMMXX_DIAG && cov != GMMXX_SPHERICAL) || dt != GMMXX_BFLOAT16 || L.tc_cluster == 0 || km == 1)
    return GMMXX_OK;
  tc::TcLaunch t = make_tc(cov, x, N, D, K, L, ws);
  t.infer = infer;
  t.out_f = out_f;
  t.out_i = out_i;
  const int rc = tc::launch_em_tc(cov, t, st);
  if (rc == GMMXX_ERR_UNSUPPORTED && km != 2) return GMMXX_OK;  // no co-resident cluster: CUDA cores
  *done = true;
  return rc;
}

// parameters, x and workspace of an inference call whose sizes and output
// pointers the caller has checked; then the component table
int infer_common(int cov, const void* x, int64_t B, int64_t N, int64_t D, int64_t K, const float* means,
                 const float* covp, const float* weights, void* ws, size_t wsb, cudaStream_t st, Layout* L) {
  GMMXX_REQUIRE(means, "means");
  GMMXX_REQUIRE(covp, "cov");
  GMMXX_REQUIRE(weights, "weights");
  if (N > 0) GMMXX_REQUIRE(x, "x");
  *L = make_layout(cov, B, N, D, K);
  if (int rc = check_ws(ws, wsb, *L)) return rc;
  // prologue off: parameters are read, never written
  return launch_prepare(cov, B, D, K, const_cast<float*>(means), const_cast<float*>(covp),
                        const_cast<float*>(weights), 0.f, 0.f, 0, *L, static_cast<char*>(ws), st);
}

// the CUDA-core statistics kernels of gmmxx_em_accumulate
int accumulate_simt(int cov_type, int x_dtype, const void* x, int64_t B, int64_t N, int64_t D, int64_t K,
                    const Layout& L, char* ws, float* stats, double* log_likelihood, cudaStream_t st) {
  RowArgs a = make_rows(cov_type, x_dtype, x, B, N, D, K, L, ws);
  a.ll_part = reinterpret_cast<double*>(ws + L.llpart);
  a.ll = log_likelihood;
  if (L.Kp == kBK) {  // one component tile: logsumexp and statistics in one pass
    a.stats = stats;
    a.part = reinterpret_cast<float*>(ws + L.mpart);
    return launch_em_small(cov_type, a, (int)B, st);
  }
  a.lse_out = reinterpret_cast<float*>(ws + L.lse);
  if (cov_type == GMMXX_TIED) a.q_out = reinterpret_cast<float*>(ws + L.qrow);
  if (int rc = launch_rows(cov_type, MODE_LSE, a, (int)B, st)) return rc;
  a.lse_in = a.lse_out;
  a.q_in = a.q_out;  // the M-step reads x^T P x instead of recomputing it per component tile
  a.q_out = nullptr;
  a.stats = stats;
  a.part = reinterpret_cast<float*>(ws + L.mpart);
  if (int rc = launch_mstep(cov_type, a, (int)B, st)) return rc;
  return launch_stats_reduce(a, (int)B, st);
}

}  // namespace

extern "C" {

int gmmxx_abi_version(void) { return GMMXX_ABI_VERSION; }

const char* gmmxx_last_error(void) { return g_err; }

int gmmxx_canary_add_offset(const int32_t* in, int32_t* out, int64_t n, int32_t offset, void* stream) {
  if (n < 0) return set_error(GMMXX_ERR_INVALID, "n < 0");
  if (n > 0) {
    GMMXX_REQUIRE(in, "in");
    GMMXX_REQUIRE(out, "out");
  }
  return launch_canary(in, out, n, offset, static_cast<cudaStream_t>(stream));
}

int64_t gmmxx_stat_width(int cov_type, int64_t D) {
  if (cov_type < GMMXX_SPHERICAL || cov_type > GMMXX_FULL || D <= 0) return -1;
  return stat_width(cov_type, (int)D);
}

size_t gmmxx_workspace_bytes(int cov_type, int64_t B, int64_t N, int64_t D, int64_t K) {
  if (cov_type < GMMXX_SPHERICAL || cov_type > GMMXX_FULL || B <= 0 || N < 0 || D <= 0 || K <= 0) return 0;
  return (size_t)make_layout(cov_type, B, N, D, K).total;
}

int gmmxx_workspace_status(void* workspace, int* status_out, void* stream) {
  GMMXX_REQUIRE(workspace, "workspace");
  GMMXX_REQUIRE(status_out, "status_out");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, workspace, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaMemsetAsync(workspace, 0, sizeof(int), st);
  if (e != cudaSuccess) return set_error(GMMXX_ERR_CUDA, "workspace status read: %s", cudaGetErrorString(e));
  *status_out = (host & (1 << GMMXX_ERR_TIMEOUT))       ? GMMXX_ERR_TIMEOUT
                : (host & (1 << GMMXX_ERR_UNSUPPORTED)) ? GMMXX_ERR_UNSUPPORTED
                : (host & (1 << GMMXX_ERR_NOT_PD))      ? GMMXX_ERR_NOT_PD
                                                        : GMMXX_OK;
  return GMMXX_OK;
}

int gmmxx_em_prepare(int cov_type, int64_t B, int64_t D, int64_t K, float* means, float* cov, float* weights,
                     float reg_covar, float min_weight, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_shape(cov_type, GMMXX_FLOAT32, B, 0, D, K)) return rc;
  GMMXX_REQUIRE(means, "means");
  GMMXX_REQUIRE(cov, "cov");
  GMMXX_REQUIRE(weights, "weights");
  if (!(min_weight > 0.f)) return set_error(GMMXX_ERR_INVALID, "min_weight must be positive");
  if (!(reg_covar >= 0.f)) return set_error(GMMXX_ERR_INVALID, "reg_covar must be non-negative");
  const Layout L = make_layout(cov_type, B, 0, D, K);
  if (int rc = check_ws(workspace, workspace_bytes, L)) return rc;
  return launch_prepare(cov_type, B, D, K, means, cov, weights, reg_covar, min_weight, 1, L,
                        static_cast<char*>(workspace), static_cast<cudaStream_t>(stream));
}

int gmmxx_accumulate_path(int cov_type, int x_dtype, int64_t B, int64_t N, int64_t D, int64_t K, int* path_out) {
  if (int rc = check_shape(cov_type, x_dtype, B, N, D, K)) return rc;
  GMMXX_REQUIRE(path_out, "path_out");
  const Layout L = make_layout(cov_type, B, N, D, K);
  const bool tc_ok = L.tc_cluster > 0 && tc_dtype_ok(cov_type, x_dtype);
  *path_out = (tc_ok && kernel_mode() != 1) ? 1 : 0;
  return GMMXX_OK;
}

int gmmxx_em_accumulate(int cov_type, int x_dtype, const void* x, int64_t B, int64_t N, int64_t D, int64_t K,
                        void* workspace, size_t workspace_bytes, float* stats, double* log_likelihood,
                        void* stream) {
  if (int rc = check_shape(cov_type, x_dtype, B, N, D, K)) return rc;
  GMMXX_REQUIRE(stats, "stats");
  GMMXX_REQUIRE(log_likelihood, "log_likelihood");
  if (N > 0) GMMXX_REQUIRE(x, "x");
  const Layout L = make_layout(cov_type, B, N, D, K);
  if (int rc = check_ws(workspace, workspace_bytes, L)) return rc;
  char* ws = static_cast<char*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int mode = kernel_mode();
  const bool tc_ok = L.tc_cluster > 0 && tc_dtype_ok(cov_type, x_dtype);
  bool fallback = false;
  if (mode == 2 && !tc_ok)
    return set_error(GMMXX_ERR_UNSUPPORTED, "tensor-core kernel required but the shape / dtype is outside its window");
  if (tc_ok && mode != 1) {
    tc::TcLaunch t = make_tc(cov_type, x, N, D, K, L, ws);
    t.stats = stats;
    t.ll = log_likelihood;
    {  // test hook: GMMXX_B200_TEST_STALL=1 makes the tensor-core kernel's bounded waits run out (100 ms)
      const char* e = getenv("GMMXX_B200_TEST_STALL");
      t.test_stall = (e != nullptr && strcmp(e, "1") == 0) ? 1 : 0;
      t.wait_ns = t.test_stall ? 100000000ull : 2000000000ull;
    }
    const int rc = tc::launch_em_tc(cov_type, t, st);
    if (rc != GMMXX_ERR_UNSUPPORTED || mode == 2) {
      if (rc == GMMXX_OK) g_last_path = 1;
      return rc;
    }
    fallback = true;  // no co-resident cluster: the CUDA-core kernels below
  }
  const int rc = accumulate_simt(cov_type, x_dtype, x, B, N, D, K, L, ws, stats, log_likelihood, st);
  if (rc == GMMXX_OK) g_last_path = fallback ? 2 : 0;
  return rc;
}

int gmmxx_last_accumulate_path(void) { return g_last_path; }

size_t gmmxx_topk_scratch_bytes(int64_t B, int64_t N, int64_t top_k) {
  if (B <= 0 || N < 0 || top_k <= 0) return 0;
  return (size_t)topk_scratch_bytes(B, N, top_k);
}

int gmmxx_em_accumulate_topk(int cov_type, int x_dtype, const void* x, int64_t B, int64_t N, int64_t D, int64_t K,
                             int64_t top_k, void* workspace, size_t workspace_bytes, void* scratch,
                             size_t scratch_bytes, float* stats, double* log_likelihood, void* stream) {
  if (int rc = check_shape(cov_type, x_dtype, B, N, D, K)) return rc;
  GMMXX_REQUIRE(stats, "stats");
  GMMXX_REQUIRE(log_likelihood, "log_likelihood");
  if (top_k < 1 || top_k >= K)
    return set_error(GMMXX_ERR_INVALID, "top_k=%lld must be in [1, K - 1] (K=%lld)", (long long)top_k, (long long)K);
  if (top_k > kMaxTopK)
    return set_error(GMMXX_ERR_UNSUPPORTED, "top_k=%lld exceeds the engine window (top_k <= %d)", (long long)top_k,
                     kMaxTopK);
  const Layout L = make_layout(cov_type, B, N, D, K);
  if (int rc = check_ws(workspace, workspace_bytes, L)) return rc;
  if (N == 0) return GMMXX_OK;
  GMMXX_REQUIRE(x, "x");
  GMMXX_REQUIRE(scratch, "scratch");
  if ((reinterpret_cast<uintptr_t>(scratch) & 15) != 0) return set_error(GMMXX_ERR_INVALID, "scratch must be 16-byte aligned");
  const int64_t need = topk_scratch_bytes(B, N, top_k);
  if ((int64_t)scratch_bytes < need)
    return set_error(GMMXX_ERR_WORKSPACE, "scratch of %zu bytes is smaller than the %lld bytes required",
                     scratch_bytes, (long long)need);
  char* ws = static_cast<char*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  RowArgs a = make_rows(cov_type, x_dtype, x, B, N, D, K, L, ws);
  a.top_k = (int)top_k;
  a.topk_idx = static_cast<int32_t*>(scratch);
  a.topk_r = reinterpret_cast<float*>(static_cast<char*>(scratch) + need / 2);
  a.ll_part = reinterpret_cast<double*>(ws + L.llpart);
  a.ll = log_likelihood;
  if (cov_type == GMMXX_TIED) a.q_out = reinterpret_cast<float*>(ws + L.qrow);
  if (int rc = launch_topk_rows(cov_type, a, (int)B, st)) return rc;
  a.q_in = a.q_out;  // x^T P x for the M-step's row loads
  a.q_out = nullptr;
  a.stats = stats;
  a.part = reinterpret_cast<float*>(ws + L.mpart);
  if (int rc = launch_topk_mstep(cov_type, a, (int)B, st)) return rc;
  return launch_stats_reduce(a, (int)B, st);
}

int gmmxx_em_finalize(int cov_type, int64_t B, int64_t D, int64_t K, int64_t n_total, const float* stats,
                      const double* log_likelihood, const float* xx_total, float reg_covar, float min_weight,
                      float* means, float* cov, float* weights, float* lower_bound_out, void* stream) {
  if (int rc = check_shape(cov_type, GMMXX_FLOAT32, B, 0, D, K)) return rc;
  GMMXX_REQUIRE(stats, "stats");
  GMMXX_REQUIRE(log_likelihood, "log_likelihood");
  GMMXX_REQUIRE(means, "means");
  GMMXX_REQUIRE(cov, "cov");
  GMMXX_REQUIRE(weights, "weights");
  if (cov_type == GMMXX_TIED) GMMXX_REQUIRE(xx_total, "xx_total");
  if (n_total <= 0) return set_error(GMMXX_ERR_INVALID, "n_total must be positive");
  if (!(min_weight > 0.f)) return set_error(GMMXX_ERR_INVALID, "min_weight must be positive");
  return launch_finalize(cov_type, B, D, K, n_total, stats, log_likelihood, xx_total, reg_covar, min_weight, means,
                         cov, weights, lower_bound_out, static_cast<cudaStream_t>(stream));
}

int gmmxx_xx_total(int x_dtype, const void* x, int64_t B, int64_t N, int64_t D, float* xx_out, void* workspace,
                   size_t workspace_bytes, void* stream) {
  if (int rc = check_shape(GMMXX_TIED, x_dtype, B, N, D, 1)) return rc;
  GMMXX_REQUIRE(xx_out, "xx_out");
  if (N > 0) GMMXX_REQUIRE(x, "x");
  const Layout L = make_layout(GMMXX_TIED, B, N, D, 1);
  if (int rc = check_ws(workspace, workspace_bytes, L)) return rc;
  return launch_xx_total(x, x_dtype, B, N, (int)D, xx_out, reinterpret_cast<float*>(static_cast<char*>(workspace) + L.xxpart),
                         static_cast<cudaStream_t>(stream));
}

int gmmxx_assign(int cov_type, int x_dtype, const void* x, int64_t B, int64_t N, int64_t D, int64_t K,
                 const float* means, const float* cov, const float* weights, int64_t* labels_out, void* workspace,
                 size_t workspace_bytes, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = check_shape(cov_type, x_dtype, B, N, D, K)) return rc;
  if (N > 0) GMMXX_REQUIRE(labels_out, "labels_out");
  Layout L;
  if (int rc = infer_common(cov_type, x, B, N, D, K, means, cov, weights, workspace, workspace_bytes, st, &L))
    return rc;
  bool done = false;
  const int rc = tc_infer(cov_type, x_dtype, x, N, D, K, L, static_cast<char*>(workspace), 2, nullptr, labels_out, st,
                          &done);
  if (done) return rc;
  RowArgs a = make_rows(cov_type, x_dtype, x, B, N, D, K, L, static_cast<char*>(workspace));
  a.labels = labels_out;
  return launch_rows(cov_type, MODE_ARGMAX, a, (int)B, st);
}

int gmmxx_logsumexp(int cov_type, int x_dtype, const void* x, int64_t B, int64_t N, int64_t D, int64_t K,
                    const float* means, const float* cov, const float* weights, float* lse_out, void* workspace,
                    size_t workspace_bytes, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = check_shape(cov_type, x_dtype, B, N, D, K)) return rc;
  if (N > 0) GMMXX_REQUIRE(lse_out, "lse_out");
  Layout L;
  if (int rc = infer_common(cov_type, x, B, N, D, K, means, cov, weights, workspace, workspace_bytes, st, &L))
    return rc;
  bool done = false;
  const int rc = tc_infer(cov_type, x_dtype, x, N, D, K, L, static_cast<char*>(workspace), 1, lse_out, nullptr, st,
                          &done);
  if (done) return rc;
  RowArgs a = make_rows(cov_type, x_dtype, x, B, N, D, K, L, static_cast<char*>(workspace));
  a.lse_out = lse_out;
  return launch_rows(cov_type, MODE_LSE, a, (int)B, st);
}

int gmmxx_resp(int cov_type, int x_dtype, const void* x, int64_t B, int64_t N, int64_t D, int64_t K,
               const float* means, const float* cov, const float* weights, const float* log_norm, float* resp_out,
               void* workspace, size_t workspace_bytes, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = check_shape(cov_type, x_dtype, B, N, D, K)) return rc;
  if (N > 0) {
    GMMXX_REQUIRE(log_norm, "log_norm");
    GMMXX_REQUIRE(resp_out, "resp_out");
  }
  Layout L;
  if (int rc = infer_common(cov_type, x, B, N, D, K, means, cov, weights, workspace, workspace_bytes, st, &L))
    return rc;
  RowArgs a = make_rows(cov_type, x_dtype, x, B, N, D, K, L, static_cast<char*>(workspace));
  a.lse_in = log_norm;
  a.out = resp_out;
  return launch_rows(cov_type, MODE_RESP, a, (int)B, st);
}

int gmmxx_predict_proba(int cov_type, int x_dtype, const void* x, int64_t B, int64_t N, int64_t D, int64_t K,
                        const float* means, const float* cov, const float* weights, float* proba_out,
                        void* workspace, size_t workspace_bytes, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = check_shape(cov_type, x_dtype, B, N, D, K)) return rc;
  if (N > 0) GMMXX_REQUIRE(proba_out, "proba_out");
  Layout L;
  if (int rc = infer_common(cov_type, x, B, N, D, K, means, cov, weights, workspace, workspace_bytes, st, &L))
    return rc;
  char* ws = static_cast<char*>(workspace);
  bool done = false;
  const int rc = tc_infer(cov_type, x_dtype, x, N, D, K, L, ws, 3, proba_out, nullptr, st, &done);
  if (done) return rc;
  RowArgs a = make_rows(cov_type, x_dtype, x, B, N, D, K, L, ws);
  a.lse_out = reinterpret_cast<float*>(ws + L.lse);
  if (int rc = launch_rows(cov_type, MODE_LSE, a, (int)B, st)) return rc;
  a.lse_in = a.lse_out;
  a.out = proba_out;
  return launch_rows(cov_type, MODE_RESP, a, (int)B, st);
}

}  // extern "C"
