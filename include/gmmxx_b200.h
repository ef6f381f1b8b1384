/*
 * gmmxx_b200.h -- C ABI of the B200 (sm_100a) GMM EM engine.
 *
 * Plain C: pointers, sizes and a CUDA stream passed as `void*` (a
 * cudaStream_t; NULL means the legacy default stream).  No framework types
 * cross this boundary.  Every device pointer must be on the device that is
 * current when the call is made; every call is asynchronous on `stream`
 * unless stated otherwise.
 *
 * Return value: GMMXX_OK (0) or a gmmxx_status error code; a readable
 * message for the last failing call on this host thread is available from
 * gmmxx_last_error().
 *
 * Layouts (row-major, contiguous):
 *   x          (B, N, D)      float32 / bfloat16 / float16 (x_dtype)
 *   means      (B, K, D)      float32
 *   cov        spherical (B, K) variances | diag (B, K, D) variances |
 *              tied (B, D, D) covariance  | full (B, K, D, D) covariances
 *   weights    (B, K)         float32 mixing weights
 *   stats      (B, K, F)      float32 sufficient statistics, F from
 *              gmmxx_stat_width(): [n_k, sum r*x (D), second-order block]
 *              second-order block: spherical sum r*|x|^2 (1), diag sum r*x^2
 *              (D), tied none, full sum r*x_i*x_j for i<=j (D(D+1)/2).
 *
 * Reference interfaces these entry points replace (OpsiClear/GMMXX, paths
 * inside that project):
 *   gmmxx/csrc/bindings.cpp:16-191   the nanobind `gmmxx._C` module
 *   gmmxx/_cuda.py:328-1416          the Python wrappers around it
 *   gmmxx/torch_fallback.py:1897-3244 the soft-EM loops whose semantics the
 *                                     engine reproduces (parity target)
 */
#ifndef GMMXX_B200_H
#define GMMXX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GMMXX_ABI_VERSION 1

#if defined(__GNUC__)
#define GMMXX_API __attribute__((visibility("default")))
#else
#define GMMXX_API
#endif

enum gmmxx_cov_type {
  GMMXX_SPHERICAL = 0,
  GMMXX_DIAG = 1,
  GMMXX_TIED = 2,
  GMMXX_FULL = 3
};

enum gmmxx_dtype {
  GMMXX_FLOAT32 = 0,
  GMMXX_BFLOAT16 = 1,
  GMMXX_FLOAT16 = 2
};

enum gmmxx_status {
  GMMXX_OK = 0,
  GMMXX_ERR_INVALID = 1,      /* bad argument (shape, pointer, enum)          */
  GMMXX_ERR_UNSUPPORTED = 2,  /* shape outside the compiled kernel windows    */
  GMMXX_ERR_CUDA = 3,         /* CUDA runtime / launch error                  */
  GMMXX_ERR_NOT_PD = 4,       /* covariance not positive definite (device)    */
  GMMXX_ERR_WORKSPACE = 5,    /* workspace too small                          */
  GMMXX_ERR_TIMEOUT = 6       /* a bounded device-side wait expired (device)  */
};

/* ---- library / lifecycle ------------------------------------------------ */

/* ABI version of the loaded library (GMMXX_ABI_VERSION). */
GMMXX_API int gmmxx_abi_version(void);

/* Message of the last failing call on this host thread ("" if none). */
GMMXX_API const char* gmmxx_last_error(void);

/* Smoke kernel: out[i] = in[i] + offset for n int32 values.
 * Replaces: gmmxx/csrc/canary/canary.cu:8-48 (canary_add_offset). */
GMMXX_API int gmmxx_canary_add_offset(const int32_t* in, int32_t* out, int64_t n, int32_t offset, void* stream);

/* Width F of one (b, k) row of the sufficient-statistics buffer. */
GMMXX_API int64_t gmmxx_stat_width(int cov_type, int64_t D);

/* Bytes of device scratch a call needs for these sizes.  One workspace may be
 * reused by successive calls on the same stream.  A new workspace must start
 * zero-filled (its first word is the sticky status word read by
 * gmmxx_workspace_status). */
GMMXX_API size_t gmmxx_workspace_bytes(int cov_type, int64_t B, int64_t N, int64_t D, int64_t K);

/* Which statistics kernels gmmxx_em_accumulate launches for this shape:
 * *path_out = 1 for the tensor-core kernels (tc_pack_kernel, then
 * em_tc_diag_kernel for diag (bf16 X) and tied (fp32 X) or em_tc_kernel for
 * spherical (bf16 X), then tc_reduce_kernel), 0 for the CUDA-core kernels (rows_kernel, mstep_kernel
 * and stats_reduce_kernel; em_small_kernel and stats_reduce_kernel when
 * K <= 64).  Honours GMMXX_B200_KERNEL.  A device that cannot
 * co-schedule the kernel's thread-block cluster falls back to the CUDA-core
 * kernels at launch time, which this query does not predict; read
 * gmmxx_last_accumulate_path after the call for the path that ran.  No
 * counterpart in the reference (its dispatch is the Python table in
 * _runtime.py:31-216). */
GMMXX_API int gmmxx_accumulate_path(int cov_type, int x_dtype, int64_t B, int64_t N, int64_t D, int64_t K,
                                    int* path_out);

/* The statistics kernels the last successful gmmxx_em_accumulate call on this
 * host thread launched: 1 tensor-core kernels, 0 CUDA-core kernels as
 * planned, 2 CUDA-core kernels because the tensor-core launch found no
 * co-resident thread-block cluster (the fallback), -1 no call yet.  The
 * choice is made on the host when the call launches, so the value is exact
 * without a synchronisation.  No counterpart in the reference. */
GMMXX_API int gmmxx_last_accumulate_path(void);

/* Reads (and clears) the sticky device status word kept in `workspace`
 * (GMMXX_OK, GMMXX_ERR_NOT_PD, GMMXX_ERR_TIMEOUT, or GMMXX_ERR_UNSUPPORTED when
 * a kernel found its launch configuration unusable, e.g. a misaligned shared
 * memory block).  Synchronises `stream`. */
GMMXX_API int gmmxx_workspace_status(void* workspace, int* status_out, void* stream);

/* ---- one soft-EM iteration, in the three steps a sharded driver needs ---- */

/* Per-iteration prologue + component table.
 * In place: spherical/diag variances clamped to >= reg_covar; weights clamped
 * to >= min_weight and renormalised (torch_fallback.py:2062-2064, 2486-2488,
 * 2866-2867).  Then the loop-invariant logit terms (log-weights, precisions
 * via batch Cholesky with the reference's jitter ladder, log-determinants,
 * precision-weighted means) are written into `workspace`.
 * Replaces: gmmxx/csrc/estep/prepare_spherical.cu:19-90 and the torch
 * prologue of the reference loops. */
GMMXX_API int gmmxx_em_prepare(int cov_type, int64_t B, int64_t D, int64_t K,
                     float* means, float* cov, float* weights,
                     float reg_covar, float min_weight,
                     void* workspace, size_t workspace_bytes, void* stream);

/* E-step + M-step statistics over this shard's rows: adds sum_n r_nk * phi(x_n)
 * into `stats` (B, K, F) and sum_n lse_n into `*log_likelihood`; both are
 * accumulated into (callers zero them per iteration).  Uses the table written
 * by gmmxx_em_prepare.  Never materialises the (N, K) responsibilities.
 * Replaces: gmmxx/csrc/fused/spherical_fused.cu:31-187 (fused_safe_kernel),
 * gmmxx/_cuda.py:415-682 (soft_update_spherical) and the E/M chunk loops of
 * torch_fallback.py:2097-2291, 2508-2651, 2912-3139. */
GMMXX_API int gmmxx_em_accumulate(int cov_type, int x_dtype, const void* x,
                        int64_t B, int64_t N, int64_t D, int64_t K,
                        void* workspace, size_t workspace_bytes,
                        float* stats, double* log_likelihood, void* stream);

/* Approximate top-k EM (the reference's approx_top_k option): as
 * gmmxx_em_accumulate, but each row's responsibilities are the softmax of its
 * top_k largest logits (equal logits: the lower component index ranks first)
 * and zero for the other components, and *log_likelihood receives the sum of
 * those top_k log-sum-exps.  1 <= top_k < K and top_k <= 64.  Runs on the
 * CUDA-core kernels (topk_rows_kernel, topk_mstep_kernel,
 * stats_reduce_kernel) for every covariance type and x dtype.  `scratch`
 * (16-byte aligned, gmmxx_topk_scratch_bytes(B, N, top_k) bytes, contents
 * ignored) holds the per-row lists between the two passes.
 * Replaces: gmmxx/_cuda.py:783-889 (approx_topk_update_spherical) and the
 * torch path torch_fallback.py:667-767 (_topk_logits_for_chunk,
 * _accumulate_topk_stats) used by the four loops (2101-2141, 2504-2530,
 * 2915-2942). */
GMMXX_API size_t gmmxx_topk_scratch_bytes(int64_t B, int64_t N, int64_t top_k);
GMMXX_API int gmmxx_em_accumulate_topk(int cov_type, int x_dtype, const void* x,
                        int64_t B, int64_t N, int64_t D, int64_t K, int64_t top_k,
                        void* workspace, size_t workspace_bytes,
                        void* scratch, size_t scratch_bytes,
                        float* stats, double* log_likelihood, void* stream);

/* M-step finalize from reduced statistics (torch_fallback.py:2293-2305,
 * 2654-2666, 3141-3167): new means / covariances / weights written in place,
 * empty components (n_k <= min_weight) keep their old means (and, except
 * tied, covariances).  `n_total` is the per-problem sample count N summed
 * over shards.  `xx_total` (B, D, D) = sum_n x_n x_n^T is required for tied
 * and ignored otherwise.  `lower_bound_out` (may be NULL) receives
 * (*log_likelihood) / (B * n_total).
 * Replaces: gmmxx/csrc/mstep/finalize_spherical.cu:141-223,
 * gmmxx/csrc/mstep/finalize_diag.cu:6-44, gmmxx/_cuda.py:1204-1238
 * (tied_finalize) and gmmxx/_cuda.py:1355-1416 (full_finalize). */
GMMXX_API int gmmxx_em_finalize(int cov_type, int64_t B, int64_t D, int64_t K, int64_t n_total,
                      const float* stats, const double* log_likelihood,
                      const float* xx_total, float reg_covar, float min_weight,
                      float* means, float* cov, float* weights,
                      float* lower_bound_out, void* stream);

/* xx_out (B, D, D) += sum_n x_n x_n^T (tied covariance, once per fit;
 * torch_fallback.py:2856-2862).  Per-CTA partials go through `workspace`
 * (sized by gmmxx_workspace_bytes(GMMXX_TIED, B, N, D, 1) or larger) and are
 * reduced in a fixed order. */
GMMXX_API int gmmxx_xx_total(int x_dtype, const void* x, int64_t B, int64_t N, int64_t D,
                             float* xx_out, void* workspace, size_t workspace_bytes, void* stream);

/* ---- inference on fixed parameters ---------------------------------------
 * Parameters are used as given (no clamp/renormalisation), like the
 * reference's *_torch_native_chunked inference functions. */

/* labels (B, N) int64: argmax_k logit, first maximal component wins
 * (torch_fallback.py:780-965). Replaces _C.spherical_assign / diag_assign. */
GMMXX_API int gmmxx_assign(int cov_type, int x_dtype, const void* x,
                 int64_t B, int64_t N, int64_t D, int64_t K,
                 const float* means, const float* cov, const float* weights,
                 int64_t* labels_out, void* workspace, size_t workspace_bytes, void* stream);

/* lse (B, N) float32 = log sum_k exp(logit) (torch_fallback.py:983-1130).
 * Replaces _C.spherical_logsumexp / diag_logsumexp. */
GMMXX_API int gmmxx_logsumexp(int cov_type, int x_dtype, const void* x,
                    int64_t B, int64_t N, int64_t D, int64_t K,
                    const float* means, const float* cov, const float* weights,
                    float* lse_out, void* workspace, size_t workspace_bytes, void* stream);

/* resp (B, N, K) float32 = exp(logit - log_norm) for a caller-supplied
 * log_norm (B, N).  Replaces _C.spherical_resp / diag_resp. */
GMMXX_API int gmmxx_resp(int cov_type, int x_dtype, const void* x,
               int64_t B, int64_t N, int64_t D, int64_t K,
               const float* means, const float* cov, const float* weights,
               const float* log_norm, float* resp_out,
               void* workspace, size_t workspace_bytes, void* stream);

/* predict_proba (B, N, K) float32 = exp(logit - lse) in one call
 * (torch_fallback.py:1133-1345). */
GMMXX_API int gmmxx_predict_proba(int cov_type, int x_dtype, const void* x,
                        int64_t B, int64_t N, int64_t D, int64_t K,
                        const float* means, const float* cov, const float* weights,
                        float* proba_out, void* workspace, size_t workspace_bytes, void* stream);

/* Per-sample log-likelihood like gmmxx_logsumexp, for callers that cannot
 * allocate device memory (no workspace argument; nothing is allocated).  No
 * counterpart in the reference.  The component table lives in a built-in
 * device array of 8 MiB that every GPU loading this library keeps until the
 * process exits; shapes whose table does not fit return GMMXX_ERR_WORKSPACE.
 * The first call on a device looks up that array's device address (make it
 * before any stream capture); so does the first call after the device's
 * context was torn down and created again.  All calls on a device share the array, so
 * calls that overlap on the GPU race; the covariance status word (jitter
 * ladder) is cleared per call and not reported. */
GMMXX_API int gmmxx_logsumexp_noalloc(int cov_type, int x_dtype, const void* x,
                                      int64_t B, int64_t N, int64_t D, int64_t K,
                                      const float* means, const float* cov, const float* weights,
                                      float* lse_out, void* stream);

/* ---- k-means initialisation (init_params="kmeans") ---------------------- */

/* Greedy k-means++ centroids of a row sample (torch_fallback.py:1390-1451,
 * _kmeans_plus_plus_init_means): sample (B, S, D) float32; the first centre
 * of problem b is row first_idx[b] (int64 device array); centre c >= 1 takes
 * `trials` candidates, candidate t the first row whose running sum of squared
 * distances to the closest centre reaches uniforms[c-1][b][t] * total
 * (uniforms (K-1, B, trials) float32 in [0, 1), row 0 when every distance is
 * zero), and keeps the candidate of smallest potential
 * sum_n min(closest_n, |s_n - cand|^2), the first on ties.  centers_out
 * (B, K, D) float32.  1 <= K <= S, 1 <= trials <= 16; workspace 256-byte
 * aligned, gmmxx_kmeans_pp_workspace_bytes(B, S, trials) bytes.  Every sum is
 * a fixed-order reduction (bitwise repeatable).  Replaces the reference's
 * torch loop (its flash-kmeans seeding step). */
GMMXX_API size_t gmmxx_kmeans_pp_workspace_bytes(int64_t B, int64_t S, int64_t trials);
GMMXX_API int gmmxx_kmeans_pp(const float* sample, int64_t B, int64_t S, int64_t D, int64_t K, int64_t trials,
                              const int64_t* first_idx, const float* uniforms, float* centers_out,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Per-label sums over the rows of x (B, N, D) with labels (B, N) int64 in
 * [0, K): stats_out (B, K, F) float32 with, by `mode`, 0: [count, sum x]
 * (F = 1 + D), 1: [count, sum x, sum (x - means[label])^2 per dimension]
 * (F = 1 + 2D; means (B, K, D) float32), 2: [count, sum x, sum x_i x_j for
 * i <= j] (F = 1 + D + D(D+1)/2, D <= 26).  K <= 1024.  Fixed-order sums
 * through `workspace` (gmmxx_label_stats_workspace_bytes bytes).  The
 * centroid update of Lloyd's k-means (the reference's flash-kmeans step,
 * torch_fallback.py:1585-1623) and the sums of its hard-label initial
 * parameters (torch_fallback.py:1454-1569). */
GMMXX_API int64_t gmmxx_label_stats_width(int mode, int64_t D);
GMMXX_API size_t gmmxx_label_stats_workspace_bytes(int mode, int64_t B, int64_t N, int64_t D, int64_t K);
GMMXX_API int gmmxx_label_stats(int x_dtype, const void* x, int64_t B, int64_t N, int64_t D, int64_t K,
                                const int64_t* labels, const float* means, int mode, float* stats_out,
                                void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* GMMXX_B200_H */
