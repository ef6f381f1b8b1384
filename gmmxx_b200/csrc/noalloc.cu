// noalloc.cu -- per-sample log-likelihood (score_samples) for callers that
// cannot allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc at the point where they
// score samples: code running inside a memory pool owned by another framework,
// callbacks that must not allocate, or deployments where every device
// allocation is made once at start-up.  gmmxx_logsumexp_noalloc serves them:
// the caller passes only inputs and outputs, and the component table that
// gmmxx_logsumexp keeps in the caller's workspace lives here instead in a
// fixed, file-scope device array of kStaticScratchBytes (8 MiB).  Every GPU
// that loads the library holds that array until the process exits.
//
// The array is shared by every call on a device and keeps the last call's
// contents; calls whose work overlaps on the GPU (different streams, or
// several host threads) race on it.  Its status word is cleared at the start
// of each call; every other byte a call reads is written earlier in the same
// call.
#include "gmm_common.cuh"
#include "rows_api.cuh"

#include <cuda.h>

#include <mutex>

namespace gmmxx {

int launch_prepare(int cov, int64_t B, int64_t D, int64_t K, float* means, float* covp, float* weights, float reg,
                   float mw, int prologue, const Layout& L, char* ws, cudaStream_t st);

namespace {

constexpr int64_t kStaticScratchBytes = 8ll << 20;

static __device__ __align__(256) char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
struct ScratchEntry {
  char* ptr;
  unsigned long long ctx_id;  // the context the address belongs to (0: not known)
};
ScratchEntry g_scratch[kMaxDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Unique id of the current context, or 0 when the driver cannot say.  A
// device's primary context that was torn down and created again (for
// instance after cudaDeviceReset) gets a new id, and with it the array a new
// address.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (get_current == nullptr || get_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of the scratch array on the current device.  The symbol's
// name in host code is only a host-side handle, so the address is looked up
// with the device current and cached per device together with the id of the
// context it was found in; a call in another context (the device was reset)
// looks it up again.  While no context id can be had the address is looked
// up on every call.
int scratch_address(char** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(GMMXX_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(GMMXX_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchEntry& ent = g_scratch[dev];
  if (ent.ptr == nullptr || ctx == 0 || ent.ctx_id != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(GMMXX_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
    ent.ptr = static_cast<char*>(p);
    // the lookup made the device's primary context current if none was
    ent.ctx_id = current_context_id();
  }
  *out = ent.ptr;
  return GMMXX_OK;
}

// Only the component-table regions of the regular workspace layout: status,
// per-component constants, feature weights, precisions and log-determinants.
Layout table_layout(int cov, int64_t B, int64_t D, int64_t K) {
  Layout L = make_layout(cov, B, 0, D, K);  // same table offsets as the workspace path
  Layout C = L;
  auto al = [](int64_t v) { return round_up(v, 256); };
  int64_t off = 0;
  C.status = off; off += al(16);
  C.cc = off; off += al(B * K * (int64_t)sizeof(CompConst));
  C.wt = off; off += al(B * L.FE * L.Kp * 4);
  C.prec = off;
  if (cov == GMMXX_TIED) off += al(B * D * D * 4);
  else if (cov == GMMXX_FULL) off += al(B * K * D * D * 4);
  C.linv = off;
  if (cov == GMMXX_TIED) off += al(B * D * D * 4);
  C.lse = off; off += al(B * K * 4);
  C.mpart = C.llpart = C.xxpart = off;
  C.tc_cluster = 0;
  C.tc_params = C.tc_consts = C.tc_part = C.tc_part_ll = 0;
  C.total = off;
  return C;
}

}  // namespace
}  // namespace gmmxx

using namespace gmmxx;

extern "C" GMMXX_API int gmmxx_logsumexp_noalloc(int cov_type, int x_dtype, const void* x, int64_t B, int64_t N,
                                                 int64_t D, int64_t K, const float* means, const float* cov,
                                                 const float* weights, float* lse_out, void* stream) {
  if (cov_type < GMMXX_SPHERICAL || cov_type > GMMXX_FULL)
    return set_error(GMMXX_ERR_INVALID, "unknown covariance type %d", cov_type);
  if (x_dtype < GMMXX_FLOAT32 || x_dtype > GMMXX_FLOAT16) return set_error(GMMXX_ERR_INVALID, "unknown x dtype %d", x_dtype);
  if (B <= 0 || N < 0 || D <= 0 || K <= 0) return set_error(GMMXX_ERR_INVALID, "bad sizes");
  const int64_t maxd = (cov_type == GMMXX_FULL) ? kMaxDFull : kMaxD;
  if (D > maxd || B > 65535 || K > (1 << 24))
    return set_error(GMMXX_ERR_UNSUPPORTED, "shape outside the engine window (D=%lld, B=%lld, K=%lld)", (long long)D,
                     (long long)B, (long long)K);
  if (means == nullptr || cov == nullptr || weights == nullptr) return set_error(GMMXX_ERR_INVALID, "parameter pointer is NULL");
  if (N > 0 && (x == nullptr || lse_out == nullptr)) return set_error(GMMXX_ERR_INVALID, "x or lse_out is NULL");
  const Layout L = table_layout(cov_type, B, D, K);
  if (L.total > kStaticScratchBytes)
    return set_error(GMMXX_ERR_WORKSPACE,
                     "component table needs %lld bytes but the built-in scratch holds %lld bytes; use "
                     "gmmxx_logsumexp with a caller workspace for this size",
                     (long long)L.total, (long long)kStaticScratchBytes);
  char* ws = nullptr;
  if (int rc = scratch_address(&ws)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the sticky status word must start at zero; the table itself is rewritten below
  cudaError_t e = cudaMemsetAsync(ws, 0, 16, st);
  if (e != cudaSuccess) return set_error(GMMXX_ERR_CUDA, "cudaMemsetAsync(static scratch): %s", cudaGetErrorString(e));
  if (int rc = launch_prepare(cov_type, B, D, K, const_cast<float*>(means), const_cast<float*>(cov),
                              const_cast<float*>(weights), 0.f, 0.f, 0, L, ws, st))
    return rc;
  RowArgs a{};
  a.x = x;
  a.dt = x_dtype;
  a.N = N;
  a.D = (int)D;
  a.K = (int)K;
  a.FE = L.FE;
  a.Kp = L.Kp;
  a.cc = reinterpret_cast<const CompConst*>(ws + L.cc);
  a.wt = reinterpret_cast<const float*>(ws + L.wt);
  a.prec = reinterpret_cast<const float*>(ws + L.prec);
  a.FM = stat_width(cov_type, (int)D);
  a.lse_out = lse_out;
  return launch_rows(cov_type, MODE_LSE, a, (int)B, st);
}
