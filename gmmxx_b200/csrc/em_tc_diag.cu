// em_tc_diag.cu -- fused soft-EM statistics for diagonal covariance on the
// 5th-generation tensor cores, bf16 X, D = 64, K <= 512, B == 1; the same
// kernel without the M-step computes labels, per-row log-sum-exp or the
// responsibilities (the inference modes, see Mode below).
//
// A thread-block cluster of C = ceil(K / 128) CTAs works on one 128-row tile
// of X at a time; CTA `rank` owns components [128 rank, 128 rank + 128) whose
// split-bf16 logit weights stay resident in its shared memory.  Per tile t:
//
//   TMA       X(t) -> the staging slot (bf16, 128-byte swizzle); once the
//             M-step of t-1 is done, X(t) again (an L2 hit) -> the M-step stage
//   prep      (4 warps, thread = row) exact x^2 = s_hi + s_lo; the E-step
//             operand [x | s_hi | s_lo] goes straight into tensor memory (which
//             frees the staging slot), and [s_hi | s_lo] next to X(t) in the
//             M-step stage
//   MMA       E-step S(t)[rows, comps] = [x | s_hi | s_lo] . W^T with the
//             A operand read from tensor memory (32 instructions, N = 128)
//   softmax   (16 warps, four threads per row) logits, row max / exp / sum,
//             (max, sum) combined across the row's four threads, exchanged with
//             the cluster through DSMEM, r = exp(l - lse) split r_hi + r_lo
//   MMA       M-step stats[comps, x | s_hi | s_lo | 1] += R^T . [x | s_hi | s_lo | 1],
//             one N = 208 instruction per 16 rows and R part (the four
//             operand groups sit 16 KB apart; the last is a constant ones block)
//
// The E-step of tile t+1 therefore depends only on X(t+1), on the E-step of
// tile t (the tensor-memory operand) and on the softmax having loaded S(t)
// (one logit slot), never on the M-step buffers; and the softmax warps are
// software-pipelined: the residual part r_lo of tile t-1 is written after
// the logits of tile t, so the wait for the M-step's high part overlaps
// useful work.
//
// Precision as in em_tc.cu: X exact in bf16, x^2 split exactly into two bf16
// terms, weights into three (24 significant bits), r into two; products exact,
// fp32 accumulation.  Statistics leave the kernel once per cluster as
// partials that tc_reduce_kernel sums in a fixed order.
//
// Tied covariance, fp32 X (kTied): the same pipeline with
//   TMA       X(t) fp32 as two 32-column boxes (32 KB staging)
//   prep      x split exactly into three bf16 planes x_hi + x_mid + x_lo (24
//             significant bits); the E-step operand [x_hi | x_mid | x_lo] in
//             tensor memory; the M-step stage receives X(t) again by TMA and
//             the prep turns it into the three planes in place
//   MMA       E-step S(t) = x . (-2 P mu_k) over the plane / weight-term pairs
//             whose term indices sum to <= 2 (6 products, 24 instructions), in
//             the same instructions 16-64 extra columns y = L^-1 x (this
//             rank's pieces of it, P = L^-T L^-1); M-step
//             R^T . [x_hi | x_mid | x_lo | 1] (the diag kernel's N = 208 shape)
//   softmax   logits without the per-row term x^T P x (it cancels in r), which
//             enters the log-likelihood per row as -|y|^2 / 2, summed over the
//             cluster ranks' pieces
// so the distance is not clamped at zero as in the reference's
// (x^T P x - 2 x.P mu + mu^T P mu).clamp_min(0): the unclamped value is a
// positive definite quadratic form and differs from zero by rounding only.
//
// Spherical covariance, bf16 X, D = 128 (kSph): the E-step operand is x
// (two 64-feature boxes), |x|^2 comes from the prep warps in fp32, the
// logit is c2 - h_k max(S + |x|^2 + |mu_k|^2, 0), and the M-step stage is
// [x[0:64] | x[64:128] | aux] with |x|^2 in three bf16 terms next to the
// constant 1 in the aux group.  K <= 512 runs in one pass (kModeEm).  For
// K > 1024 the first pass (kModeRowStat) writes each row's (max, scaled sum)
// over a group of 2 chunks: it has no M-step, so X gets a three-slot staging
// ring in the M-step stage and R buffer and the E-step reads X from its slot
// (A from shared memory), S has two slots in the M-step accumulator columns,
// and the softmax is pipelined over three tiles (part table in the R
// buffer).  The second pass runs in em_tc_sph_ext.cu (or, for comparison,
// here as kModeExtLse).  Inference: labels, log-sum-exp and responsibilities
// in one pass for K <= 512, else per group with the combine kernels and, for
// the responsibilities, kModeProbaExt from the combined log-sum-exp.
//
// Reference semantics: gmmxx/torch_fallback.py:2508-2651 (diag E/M chunk
// loop), expanded-distance logits 357-397; tied 435-465 (logits), 2912-3139
// (matrix E/M loop); spherical 2097-2291 (E/M chunk loop), logits 337-354.
#include "gmm_common.cuh"
#include "tc_ptx.cuh"
#include "tc_api.cuh"

#include <math.h>

#include <algorithm>
#include <type_traits>

namespace gmmxx {
namespace tc {
namespace {

using namespace ptx;

constexpr int kBM = 128;        // rows per tile
constexpr int kKC = 128;        // components per CTA
constexpr int kNS = 3;          // bf16 terms of the split weights
constexpr int kSplit = 4;                // softmax threads per row
constexpr int kPart = kKC / kSplit;      // components per softmax thread
constexpr int kSoftWarps = 4 * kSplit;   // every TMEM lane quarter kSplit times
constexpr int kBlock = 16384;   // one [128][64] bf16 swizzled block
constexpr uint32_t kTmemCols = 512;
constexpr int kFdm = 208;       // M-step columns [x | s_hi | s_lo | 1] (tied: [x_hi | x_mid | x_lo | 1])
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kHalfLog2e = 0.5f * kLog2e;  // logit scale of a unit distance (diag: s = 1)
constexpr int kMaxCluster = kMaxClusterDiag;

// EM modes issue the E-steps from warp kWarpMma and the M-steps from warp
// kWarpMmaM, on another SM sub-partition (warp % 4): one thread issuing every
// MMA of a tile shares its sub-partition with four busy softmax warps
enum Warp { kWarpPrep0 = 0, kWarpTma = 4, kWarpMma = 5, kWarpSoftmax0 = 6, kWarpMmaM = 22 };
// EM statistics, or inference without the M-step (TcLaunch::infer); the
// spherical large-K passes: each row's (max, scaled sum) over the cluster's
// components (kModeRowStat), then the M-step with r = 2^(l - lse) from the
// row's log-sum-exp over all K (kModeExtLse: no exchange); grouped
// predict_proba: the responsibilities from that log-sum-exp, written as
// kModeProba writes them (kModeProbaExt: no exchange either)
enum Mode {
  kModeEm = 0, kModeLse = 1, kModeArgmax = 2, kModeProba = 3, kModeRowStat = 4, kModeExtLse = 5, kModeProbaExt = 6
};
constexpr int kThreads = (kWarpMmaM + 1) * 32;  // 23 warps, <= 80 registers each

// Shared memory carve-up (byte offsets from the 1024-aligned dynamic block)
// and tensor memory columns of each covariance type's layout: diag (bf16 X,
// D = 64), tied (fp32 X, D = 64), spherical (bf16 X, D = 128).
template <int kCov>
struct Lay {
  static constexpr bool kTied = kCov == GMMXX_TIED;
  static constexpr bool kSph = kCov == GMMXX_SPHERICAL;
  // weights: diag a_0 a_1 a_2 | v_0 v_1 v_2 (16 KB each); tied three terms of
  // [192 rows][64] (components, then this rank's rows of L^-1); spherical
  // three terms of two [128][64] feature halves
  static constexpr int kWBytes = kTied ? kTiedTermBytes : kBlock;
  static constexpr int kWBlocks = kTied ? kNS : 2 * kNS;
  static constexpr int kParams = 0;
  // X staging slot: one bf16 box (diag), two fp32 boxes (tied), two bf16 boxes (spherical D = 128)
  static constexpr int kStaging = kParams + kWBlocks * kWBytes;
  // M-step stage: diag x | s_hi | s_lo | ones; tied x_hi | x_mid | x_lo | ones;
  // spherical x[0:64] | x[64:128] | aux (column 0 = 1, columns 1-3 = |x|^2 in
  // three bf16 terms); predict_proba: the tile's fp32 rows
  static constexpr int kMX = kStaging + (kCov == GMMXX_DIAG ? 1 : 2) * kBlock;
  static constexpr int kMSH = kMX + kBlock;
  static constexpr int kMSL = kMSH + kBlock;
  static constexpr int kOnes = kMSL + kBlock;                   // MN-major, column 0 = 1 (constant)
  static constexpr int kR = kMX + (kSph ? 3 : 4) * kBlock;      // R: two 64-component MN groups
  static constexpr int kConsts = kR + 2 * kBlock;               // lz[128], c2[128] (spherical: c2, h, mpm)
  static constexpr int kQ = kConsts + 3 * 128 * 4;              // spherical: |x|^2 [2 tile slots][128 rows]
  static constexpr int kHalfX = kQ + (kSph ? 2 * 128 * 4 : 0);  // [2 slots][kSplit parts][128 rows] float2
  static constexpr int kXch = kHalfX + 2 * kSplit * 128 * 8;  // [2 slots][C][128 rows] float2
  __host__ __device__ static constexpr int bars(int c) { return kXch + 2 * c * 128 * 8; }
  // the log-likelihood reduction slot: 4 doubles (diag), 16 (tied)
  __host__ __device__ static constexpr int red(int c) { return bars(c) + 256; }
  __host__ __device__ static constexpr int total(int c) { return bars(c) + (kTied ? 384 : 288); }
  // tensor memory: S (+ tied: up to 64 columns of y) | M-step statistics | E-step operand
  // (diag [x | s_hi | s_lo], tied [x_hi | x_mid | x_lo]: 96 columns; spherical x: 64)
  static constexpr int kFdmCols = kSph ? 144 : kFdm;  // spherical [x (128) | aux (16)]
  static constexpr uint32_t kSCol = 0;
  static constexpr uint32_t kDmCol = kTied ? 192 : 128;
  static constexpr uint32_t kFCol = kDmCol + kFdmCols;
  static constexpr uint32_t kFEnd = kFCol + (kSph ? 64 : 96);
};
static_assert(Lay<GMMXX_DIAG>::total(kMaxCluster) <= 232448 && Lay<GMMXX_TIED>::total(kMaxCluster) <= 232448 &&
                  Lay<GMMXX_SPHERICAL>::total(kMaxCluster) <= 232448,
              "shared memory budget");
static_assert(Lay<GMMXX_DIAG>::kFEnd <= kTmemCols && Lay<GMMXX_TIED>::kFEnd <= kTmemCols &&
                  Lay<GMMXX_SPHERICAL>::kFEnd <= kTmemCols,
              "tensor memory budget");
static_assert(Lay<GMMXX_TIED>::kStaging % 1024 == 0 && Lay<GMMXX_TIED>::kMX % 1024 == 0 &&
                  Lay<GMMXX_TIED>::kR % 1024 == 0 && Lay<GMMXX_SPHERICAL>::kMX % 1024 == 0 &&
                  Lay<GMMXX_SPHERICAL>::kR % 1024 == 0,
              "swizzled blocks need 1024-byte alignment");

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct Bars {
  uint64_t params;
  uint64_t xfull[3];   // TMA: staging slot holds X(t) (slots 1, 2: spherical kModeRowStat only)
  uint64_t sempty[3];  // prep: staging slot read (128 threads)
  uint64_t mxfull;     // TMA: M-step stage holds X(t)
  uint64_t ffull;      // prep: E-step operand of tile t in tensor memory (4 warps)
  uint64_t mfull;      // prep: M-step stage holds [x | s_hi | s_lo] of tile t (4 warps)
  uint64_t mfree;      // MMA: M-step of tile t done reading the stage
  uint64_t sfull[2];   // MMA: S(t) complete (the E-step operand is free again); slot 1: ring mode
  uint64_t sfree[2];   // softmax: S(t) loaded (16 warps)
  uint64_t rfull;      // softmax: an R part written (16 warps)
  uint64_t rfree;      // MMA: that R part consumed
  uint64_t xch[2];     // cluster exchange of (row max, row sum)
  uint64_t hx[4];      // every part of the row wrote its (max, sum) (16 warps; kModeRowStat: four slots)
  uint64_t mdone;      // MMA: all MMAs complete
  uint64_t pfull;      // predict_proba: the tile's rows staged in shared memory (16 warps)
  uint64_t pfree;      // predict_proba: the staged rows stored to global memory (16 warps)
  uint64_t qfull[2];   // spherical: |x|^2 of the tile in slot s written (4 prep warps)
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Bars) <= 256, "barrier block overlaps the reduction slot");

__device__ __forceinline__ void set_abort(Bars* b, int* status) {
  b->abort = 1;
  atomicOr(status, 1 << GMMXX_ERR_TIMEOUT);
}

// x -> (s_hi, s_lo) for one packed pair of bf16 values: x^2 is exact in fp32
// (8-bit significands) and splits exactly into two bf16 terms.
__device__ __forceinline__ void square_split(uint32_t w, uint32_t& hi, uint32_t& lo) {
  const float x0 = bf16lo_to_f32(w), x1 = bf16hi_to_f32(w);
  const float s0 = x0 * x0, s1 = x1 * x1;
  hi = pack_bf16(s0, s1);
  lo = pack_bf16(s0 - bf16lo_to_f32(hi), s1 - bf16hi_to_f32(hi));
}

// two fp32 values -> three packed bf16 pairs with x = hi + mid + lo to 24
// significant bits (each residual is exact in fp32)
__device__ __forceinline__ void split3(float x0, float x1, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
  hi = pack_bf16(x0, x1);
  const float r0 = x0 - bf16lo_to_f32(hi), r1 = x1 - bf16hi_to_f32(hi);
  mid = pack_bf16(r0, r1);
  lo = pack_bf16(r0 - bf16lo_to_f32(mid), r1 - bf16hi_to_f32(mid));
}

template <int kMode, int kCov>
__global__ void __launch_bounds__(kThreads, 1)
    em_tc_diag_kernel(const __grid_constant__ CUtensorMap tmap, TcArgs a) {
  constexpr bool kTied = kCov == GMMXX_TIED;
  constexpr bool kSph = kCov == GMMXX_SPHERICAL;
  constexpr bool kExt = kMode == kModeExtLse;             // r from the row's external log-sum-exp
  constexpr bool kEm = kMode == kModeEm || kExt;          // the M-step runs
  constexpr bool kNoXch = kExt || kMode == kModeProbaExt;  // passes that exchange nothing in the cluster
  static_assert(kCov == GMMXX_DIAG ? kMode <= kModeProba : (kSph || kMode == kModeEm),
                "modes of each covariance type");
  using Y = Lay<kCov>;
  constexpr int kParams = Y::kParams, kStaging = Y::kStaging, kMX = Y::kMX, kMSH = Y::kMSH, kMSL = Y::kMSL;
  // X staging slots: one, or (spherical row statistics, which has no M-step)
  // three -- the M-step stage and the R buffer's first block hold slots 1
  // and 2 -- so that the TMA loads run two tiles ahead of the prep warps
  // instead of exposing one HBM round trip per tile
  constexpr int kNStage = (kSph && kMode == kModeRowStat) ? 3 : 1;
  // with the ring, the E-step reads X straight from its staging slot (A from
  // shared memory) and the slot is freed by the prep warps and the E-step's
  // completion; otherwise the prep warps copy X into tensor memory
  constexpr bool kRing = kNStage > 1;
  // ring mode: a second S slot in the (unused) M-step accumulator columns
  constexpr uint32_t kS1Off = kRing ? Y::kDmCol - Y::kSCol : 0;
  static_assert(!kRing || Y::kDmCol + 128 <= Y::kFCol, "second S slot in the M-step columns");
  auto stage_off = [](int slot) { return slot == 0 ? kStaging : kMX + (slot - 1) * 2 * kBlock; };
  constexpr int kOnes = Y::kOnes, kR = Y::kR, kConsts = Y::kConsts, kHalfX = Y::kHalfX, kXch = Y::kXch;
  constexpr uint32_t kSCol = Y::kSCol, kDmCol = Y::kDmCol, kFCol = Y::kFCol;
  extern __shared__ __align__(1024) char smem_raw[];
  char* sm = smem_raw;
  if ((smem_u32(smem_raw) & 1023u) != 0) {  // uniform across the grid: no CTA proceeds
    if (threadIdx.x == 0) atomicOr(a.status, 1 << GMMXX_ERR_UNSUPPORTED);
    return;
  }
  const int nclus = a.cluster_size;
  Bars* bars = reinterpret_cast<Bars*>(sm + Y::bars(nclus));
  float* c_lz = reinterpret_cast<float*>(sm + kConsts);  // c2 - h mpm: the logit at S = 0 (spherical: c2)
  float* c_c2 = c_lz + 128;                               // (spherical: h = log2(e) / (2 var))
  float* c_mpm = c_lz + 256;                              // spherical: |mu|^2
  float* qbuf = reinterpret_cast<float*>(sm + Y::kQ);     // spherical: |x|^2 per row, two tile slots
  float2* xch = reinterpret_cast<float2*>(sm + kXch);
  volatile int* abort = &bars->abort;
  const uint64_t lim = a.wait_ns;  // every wait below gives up after this long

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // hardware cluster, or (kModeExtLse, which exchanges nothing) a virtual one
  // of a.vcluster consecutive CTAs of a cluster-free launch
  const int vc = kNoXch ? a.vcluster : 0;
  const uint32_t rank = vc > 0 ? blockIdx.x % (uint32_t)vc : cluster_rank();
  const uint32_t cid = vc > 0 ? blockIdx.x / (uint32_t)vc : cluster_id_x();
  const uint32_t ncl = vc > 0 ? gridDim.x / (uint32_t)vc : ncluster_x();
  const int64_t ntiles = (a.N + kBM - 1) / kBM;
  const int T = (int)((ntiles > (int64_t)cid) ? (ntiles - 1 - cid) / ncl + 1 : 0);
  // tied: this rank's pieces [p0, p1) of the 4 sixteen-column pieces of y = L^-1 x
  const int ny = kTied ? 4 * ((int)rank + 1) / nclus - 4 * (int)rank / nclus : 0;

  if (tid == 0) {
    mbar_init(&bars->params, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&bars->xfull[i], 1);
      mbar_init(&bars->sempty[i], kRing ? 129 : 128);
    }
    mbar_init(&bars->mxfull, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->sfull[i], 1);
      mbar_init(&bars->sfree[i], kSoftWarps);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&bars->xch[i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&bars->hx[i], kSoftWarps);
    mbar_init(&bars->ffull, 4);
    mbar_init(&bars->mfull, 4);
    mbar_init(&bars->mfree, 1);
    mbar_init(&bars->rfull, kSoftWarps);
    mbar_init(&bars->rfree, 1);
    mbar_init(&bars->mdone, 2);  // both issuing threads commit
    mbar_init(&bars->pfull, kSoftWarps);
    mbar_init(&bars->pfree, kSoftWarps);
    mbar_init(&bars->qfull[0], 4);
    mbar_init(&bars->qfull[1], 4);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == kWarpMma) tmem_alloc(&bars->tmem_base, kTmemCols);
  // logit = c2 - h max(S + mpm, 0) = min(lz - h S, c2) with lz = c2 - h mpm
  // (h > 0); a padding component has c2 = -inf, so lz = -inf too.  Spherical:
  // c2 - h_k max(S + |x|^2 + mpm_k, 0), per-component h and mpm.
  // (grouped passes: this CTA's chunk of 128 components is a.chunk0 + rank)
  const int chunk = a.chunk0 + (int)rank;
  for (int i = tid; i < 128; i += kThreads) {
    const float* cs = a.consts + (int64_t)chunk * 3 * 128;
    if constexpr (kSph) {
      c_lz[i] = cs[256 + i];
      c_c2[i] = cs[128 + i];
      c_mpm[i] = cs[i];
    } else {
      c_lz[i] = fmaf(-kHalfLog2e, cs[i], cs[256 + i]);
      c_c2[i] = cs[256 + i];
    }
  }
  // ones group of the M-step operand (n_k): MN-major like X, element (row, 0)
  // = 1 and the rest 0, i.e. 16-byte chunk 0 of every row holds bf16 1.0 in
  // its first element; the chunk sits at position (row & 7) after the swizzle.
  // Spherical: the aux group (kMSL) starts the same; the prep warps then
  // write |x|^2 into columns 1-3 of each tile's rows.
  for (int i = tid; i < kBlock / 16; i += kThreads) {
    const int row = i >> 3, chunk16 = i & 7;
    reinterpret_cast<uint4*>(sm + (kSph ? kMSL : kOnes))[i] =
        make_uint4(chunk16 == (row & 7) ? 0x3F80u : 0u, 0u, 0u, 0u);
  }
  fence_proxy_async();
  tmem_fence_before();
  __syncthreads();
  cluster_sync();  // peers' barriers initialised before any DSMEM traffic
  tmem_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp < kWarpTma) {
    // ---------------- prep: 4 warps, thread = row (its TMEM lane) ----------------
    const int r = warp * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(warp * 32) << 16;
    const uint32_t swz = (uint32_t)(r & 7);
    // the 32 words (64 bf16) of row r of a swizzled X block, in element order
    auto load_row = [&](int off, uint32_t (&w)[32]) {
      const char* base = sm + off + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = *reinterpret_cast<const uint4*>(base + ((c ^ swz) << 4));
        w[4 * c] = v.x;
        w[4 * c + 1] = v.y;
        w[4 * c + 2] = v.z;
        w[4 * c + 3] = v.w;
      }
    };
    // M-step stage of tile u: X(u) lands there by TMA once the M-step of u-1
    // is done; add [s_hi | s_lo] (same swizzled layout).  Spherical: the row's
    // |x|^2 (qu, kept since the tile's E-step operand was written) into the
    // aux group as three bf16 terms next to the constant 1.
    auto fill_mstage = [&](int u, float qu) -> bool {
      if (!mbar_wait_warp(&bars->mxfull, u & 1, abort, lim)) return false;
      if constexpr (kSph) {
        const float q0 = __bfloat162float(__float2bfloat16(qu));
        const float q1 = __bfloat162float(__float2bfloat16(qu - q0));
        const uint32_t w0 = pack_bf16(1.f, q0), w1 = pack_bf16(q1, qu - q0 - q1);
        *reinterpret_cast<uint4*>(sm + kMSL + r * 128 + (int)(swz << 4)) = make_uint4(w0, w1, 0u, 0u);
      } else if constexpr (kTied) {
        // fp32 X(u) landed as two 32-column boxes in the x_hi and x_mid
        // blocks; this thread's row is read whole, then its three bf16 planes
        // overwrite it (rows are thread-private)
        float f[64];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 v = *reinterpret_cast<const float4*>(sm + (h ? kMSH : kMX) + r * 128 + ((c ^ swz) << 4));
            f[32 * h + 4 * c] = v.x;
            f[32 * h + 4 * c + 1] = v.y;
            f[32 * h + 4 * c + 2] = v.z;
            f[32 * h + 4 * c + 3] = v.w;
          }
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // features 8c .. 8c + 7
          uint32_t hi[4], mid[4], lo[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) split3(f[8 * c + 2 * i], f[8 * c + 2 * i + 1], hi[i], mid[i], lo[i]);
          const int off = r * 128 + (int)((c ^ swz) << 4);
          *reinterpret_cast<uint4*>(sm + kMX + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(sm + kMSH + off) = make_uint4(mid[0], mid[1], mid[2], mid[3]);
          *reinterpret_cast<uint4*>(sm + kMSL + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
      } else {
        uint32_t w[32];
        load_row(kMX, w);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) square_split(w[4 * c + i], hi[i], lo[i]);
          const int off = r * 128 + (int)((c ^ swz) << 4);
          *reinterpret_cast<uint4*>(sm + kMSH + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(sm + kMSL + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->mfull);
      return true;
    };
    bool ok = true;
    float q_cur = 0.f, q_prev = 0.f;  // spherical: |x|^2 of this row in tiles t and t - 1
    for (int t = 0; t < T; ++t) {
      const int xs = t % kNStage;
      if (!mbar_wait_warp(&bars->xfull[xs], (t / kNStage) & 1, abort, lim)) { ok = false; break; }
      if constexpr (kSph) {
        if constexpr (kRing) {
          // the |x|^2 slot of tile t was last read by the softmax for tile
          // t-2, before it released S(t-2); wait for S(t-1) released (the
          // softmax waits for this tile's |x|^2 before releasing S(t), so
          // this barrier cannot be a phase ahead)
          if (t >= 1 && !mbar_wait_warp(&bars->sfree[(t - 1) & 1], ((t - 1) >> 1) & 1, abort, lim)) { ok = false; break; }
        } else {
          // the E-step of t-1 read the operand region: wait for its completion
          if (t >= 1 && !mbar_wait_warp(&bars->sfull[0], (t - 1) & 1, abort, lim)) { ok = false; break; }
          tmem_fence_after();
        }
        float q = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // bf16 box h: features 64h .. 64h + 63 -> operand columns 32h .. 32h + 31
          uint32_t w[32];
          load_row(stage_off(xs) + h * kBlock, w);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float x0 = bf16lo_to_f32(w[i]), x1 = bf16hi_to_f32(w[i]);
            q = fmaf(x0, x0, q);
            q = fmaf(x1, x1, q);
          }
          if constexpr (!kRing) tmem_st32(tmem + lane_addr + kFCol + 32 * h, w);
        }
        q_prev = q_cur;
        q_cur = q;
        // the softmax reads the slot of tile t before it releases S(t), which
        // the E-step of t+1 (and so the prep of t+2) waits for (ring: see above)
        qbuf[(t & 1) * 128 + r] = q;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->qfull[t & 1]);
      } else if constexpr (kTied) {
        // the E-step of t-1 read the operand region: wait for its completion
        if (t >= 1 && !mbar_wait_warp(&bars->sfull[0], (t - 1) & 1, abort, lim)) { ok = false; break; }
        tmem_fence_after();
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // fp32 box h: features 32h .. 32h + 31 -> operand words 16h .. 16h + 15
          uint32_t hi[16], mid[16], lo[16];
          const char* base = sm + kStaging + h * kBlock + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 v = *reinterpret_cast<const float4*>(base + ((c ^ swz) << 4));
            split3(v.x, v.y, hi[2 * c], mid[2 * c], lo[2 * c]);
            split3(v.z, v.w, hi[2 * c + 1], mid[2 * c + 1], lo[2 * c + 1]);
          }
          tmem_st16(tmem + lane_addr + kFCol + 16 * h, hi);
          tmem_st16(tmem + lane_addr + kFCol + 32 + 16 * h, mid);
          tmem_st16(tmem + lane_addr + kFCol + 64 + 16 * h, lo);
        }
      } else {
        uint32_t w[32];
        load_row(kStaging, w);
        // the E-step of t-1 read the operand region: wait for its completion
        if (t >= 1 && !mbar_wait_warp(&bars->sfull[0], (t - 1) & 1, abort, lim)) { ok = false; break; }
        tmem_fence_after();
        tmem_st32(tmem + lane_addr + kFCol, w);
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // s_hi / s_lo in 16-column pieces
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) square_split(w[16 * h + i], hi[i], lo[i]);
          tmem_st16(tmem + lane_addr + kFCol + 32 + 16 * h, hi);
          tmem_st16(tmem + lane_addr + kFCol + 64 + 16 * h, lo);
        }
      }
      tmem_wait_st();
      // the TMA may now refill the staging slot.  Every thread releases it
      // itself, once its loaded words have been consumed (the tensor-memory
      // stores above read them): an arrive right after the loads, or one lane's
      // arrive after __syncwarp, let the next TMA copy (async proxy) overtake
      // loads still in flight -- rows of the next tile then leaked into this
      // one when the softmax ran slow (measured with predict_proba).
      mbar_arrive(&bars->sempty[xs]);
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ffull);
      if (kEm && t >= 1 && !fill_mstage(t - 1, q_prev)) { ok = false; break; }
      if (*abort) { ok = false; break; }
    }
    if (kEm && ok && T >= 1 && !fill_mstage(T - 1, q_cur)) ok = false;
    if (!ok) set_abort(bars, a.status);
  } else if (warp == kWarpTma) {
    // ---------------- producer: weights once, then X tiles (staging slot and M-step stage) ----------------
    if (lane == 0) {
      prefetch_tmap(&tmap);
      constexpr int kParamBlocks = Y::kWBlocks, kWBytes = Y::kWBytes;
      mbar_expect_tx(&bars->params, kParamBlocks * kWBytes);
      const char* src = a.params + (int64_t)chunk * kParamBlocks * kWBytes;
      for (int i = 0; i < kParamBlocks; ++i)
        bulk_load(sm + kParams + i * kWBytes, src + (int64_t)i * kWBytes, kWBytes, &bars->params);
      // one X tile: a bf16 box (diag), two fp32 boxes of 32 columns (tied) or
      // two bf16 boxes of 64 columns (spherical D = 128)
      constexpr uint32_t kTileBytes = (kCov == GMMXX_DIAG ? 1 : 2) * kBlock;
      auto load_tile = [&](int dst0, int dst1, int row, uint64_t* bar) {
        tma_load_2d(sm + dst0, &tmap, 0, row, bar);
        if constexpr (kCov != GMMXX_DIAG) tma_load_2d(sm + dst1, &tmap, kTied ? 32 : 64, row, bar);
      };
      auto row0 = [&](int t) { return (int)((cid + (int64_t)t * ncl) * kBM); };
      int issued = 0, missued = 0;
      // X(u) into the M-step stage once the M-step of u-1 released it
      auto load_m = [&](int u) -> bool {
        if (u >= 1 && !mbar_wait(&bars->mfree, (u - 1) & 1, abort, lim)) return false;
        mbar_expect_tx(&bars->mxfull, kTileBytes);
        load_tile(kMX, kMSH, row0(u), &bars->mxfull);
        missued = u + 1;
        return true;
      };
      bool ok = true;
      for (int t = 0; t < T && ok; ++t) {
        const int xs = t % kNStage;
        if (t >= kNStage && !mbar_wait(&bars->sempty[xs], ((t / kNStage) - 1) & 1, abort, lim)) { ok = false; break; }
        if (a.test_stall) break;  // test hook: no X tile ever lands, every wait on it runs out
        mbar_expect_tx(&bars->xfull[xs], kTileBytes);
        load_tile(stage_off(xs), stage_off(xs) + kBlock, row0(t), &bars->xfull[xs]);
        issued = t + 1;
        if (kEm && t >= 1) ok = load_m(t - 1);
      }
      if (kEm && ok && T >= 1 && issued == T) ok = load_m(T - 1);
      if (!ok) set_abort(bars, a.status);
      // before the CTA can exit, every copy it started has landed (bounded,
      // also after an abort): the weights and the last load of each buffer
      mbar_wait(&bars->params, 0, nullptr, lim);
      for (int u = issued > kNStage ? issued - kNStage : 0; u < issued; ++u)
        mbar_wait(&bars->xfull[u % kNStage], (u / kNStage) & 1, nullptr, lim);
      if (missued > 0) mbar_wait(&bars->mxfull, (missued - 1) & 1, nullptr, lim);
    }
  } else if (warp == kWarpMma || warp == kWarpMmaM) {
    // ---------------- MMA issuers (one thread each) ----------------
    if (lane == 0) {
      // A (TMEM) x W^T (K-major); tied: N also covers this rank's y columns
      const uint32_t id_e = idesc_bf16(128, kKC + 16 * ny, 0, 0);
      // R^T x [x | s_hi | s_lo | 1] (spherical [x | x | aux]), both MN-major
      const uint32_t id_m = idesc_bf16(128, Y::kFdmCols, 1, 1);
      const uint32_t base = smem_u32(sm);
      bool ok = mbar_wait(&bars->params, 0, abort, lim);
      tmem_fence_after();
      // weight descriptors: K-major blocks, +32 B per 16-feature step
      // (spherical: wa the features 0-63 of term j, wv the features 64-127)
      uint64_t wa[kNS], wv[kNS];
#pragma unroll
      for (int j = 0; j < kNS; ++j) {
        wa[j] = desc_kmajor(base + kParams + (kSph ? 2 * j : j) * Y::kWBytes);
        wv[j] = kTied ? 0 : desc_kmajor(base + kParams + (kSph ? 2 * j + 1 : kNS + j) * Y::kWBytes);
      }
      // E-step of tile t into S: x.a_j, s_hi.v_j (j < 3), s_lo.v_j (j < 2)
      auto issue_e = [&](int t) -> bool {
        if constexpr (kRing) {
          // A = X(t) in its staging slot (K-major, rows x features), the
          // instruction order of the tensor-memory form below; the commit on
          // the slot's barrier frees it once the E-step has read it
          const int xs = t % kNStage;
          if (!mbar_wait(&bars->xfull[xs], (t / kNStage) & 1, abort, lim)) return false;
          // two S slots: S(t) overwrites S(t-2) once the softmax loaded it
          if (t >= 2 && !mbar_wait(&bars->sfree[t & 1], ((t >> 1) - 1) & 1, abort, lim)) return false;
          tmem_fence_after();
          const uint32_t d = tmem + kSCol + (uint32_t)((t & 1) * kS1Off);
          const uint32_t xa = base + (uint32_t)stage_off(xs);
          uint32_t acc = 0;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint64_t xd = desc_kmajor(xa + (uint32_t)(h * kBlock));
#pragma unroll
            for (int j = 0; j < kNS; ++j)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                mma_bf16(d, xd + 2 * kk, (h ? wv[j] : wa[j]) + 2 * kk, id_e, acc);
                acc = 1;
              }
          }
          mma_commit(&bars->sfull[t & 1]);
          mma_commit(&bars->sempty[xs]);
          return true;
        }
        if (!mbar_wait(&bars->ffull, t & 1, abort, lim)) return false;
        if (t >= 1 && !mbar_wait(&bars->sfree[0], (t - 1) & 1, abort, lim)) return false;
        tmem_fence_after();
        const uint32_t d = tmem + kSCol;
        uint32_t acc = 0;
#pragma unroll
        for (int j = 0; j < kNS; ++j)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            mma_bf16_ts(d, tmem + kFCol + kk * 8, wa[j] + 2 * kk, id_e, acc);
            acc = 1;
          }
        if constexpr (kTied) {  // x_mid . (w_0 + w_1), x_lo . w_0
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) mma_bf16_ts(d, tmem + kFCol + 32 + kk * 8, wa[j] + 2 * kk, id_e, 1u);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_bf16_ts(d, tmem + kFCol + 64 + kk * 8, wa[0] + 2 * kk, id_e, 1u);
        } else {  // diag s_hi . v_j, spherical x[64:128] . a_j
#pragma unroll
          for (int j = 0; j < kNS; ++j)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) mma_bf16_ts(d, tmem + kFCol + 32 + kk * 8, wv[j] + 2 * kk, id_e, 1u);
          if constexpr (!kSph) {  // diag s_lo . v_j (j < 2)
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) mma_bf16_ts(d, tmem + kFCol + 64 + kk * 8, wv[j] + 2 * kk, id_e, 1u);
          }
        }
        mma_commit(&bars->sfull[0]);
        return true;
      };
      const uint64_t r0 = desc_mnmajor(base + kR, kBlock);
      const uint64_t x0 = desc_mnmajor(base + kMX, kBlock);  // [x | s_hi | s_lo | 1]: 16 KB apart
      // M-step of tile t with R part PART (0 = high bf16 terms, 1 = residual)
      auto issue_m = [&](int t, auto part_tag) -> bool {
        constexpr int part = decltype(part_tag)::value;
        const int use = 2 * t + part;
        if (!mbar_wait(&bars->rfull, use & 1, abort, lim)) return false;
        if (part == 0 && !mbar_wait(&bars->mfull, t & 1, abort, lim)) return false;
        tmem_fence_after();
        const uint32_t acc0 = (t == 0 && part == 0) ? 0u : 1u;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {  // 16 rows per instruction: +2048 B (MN-major)
          const uint64_t step = (uint64_t)(ks * 128);
          mma_bf16(tmem + kDmCol, r0 + step, x0 + step, id_m, ks == 0 ? acc0 : 1u);
        }
        mma_commit(&bars->rfree);
        if constexpr (part == 1) mma_commit(&bars->mfree);
        return true;
      };
      using Hi = std::integral_constant<int, 0>;
      using Lo = std::integral_constant<int, 1>;
      // Two issuing threads: the E-steps in tile order, each once the
      // softmax loaded S(t-1) and the prep wrote the operand of t; the M-steps
      // M_hi(t), M_lo(t) as the softmax writes the two R parts (M_lo(t) after
      // the logits of t+1).  The tensor pipe takes them in arrival order.
      if (warp == kWarpMma) {  // E-steps, each as soon as S is free and the operand written
        for (int t = 0; ok && t < T; ++t) ok = issue_e(t);
      } else if constexpr (kEm) {  // M-steps
        for (int t = 0; ok && t < T; ++t) {
          if (!issue_m(t, Hi{})) { ok = false; break; }
          if (!issue_m(t, Lo{})) { ok = false; break; }
        }
      }
      if (!ok) set_abort(bars, a.status);
      mma_commit(&bars->mdone);
    }
  } else if (warp >= kWarpSoftmax0 && warp < kWarpSoftmax0 + kSoftWarps) {
    // ---------------- softmax: 16 warps, kSplit per TMEM lane quarter ----------------
    // warp w reads lanes 32 (w % 4) .. +31 (the tensor-memory access rule);
    // part qc of the row owns components [qc kPart, qc kPart + kPart)
    const int q4 = warp & 3;
    const int qc = (warp - kWarpSoftmax0) >> 2;
    const int row = q4 * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q4 * 32) << 16;
    const int k0 = qc * kPart;
    double ll_acc = 0.0;
    float p[kPart];
    uint32_t lo[kPart / 2];  // residual words of the previous tile, written one iteration later
    float2* halfx = reinterpret_cast<float2*>(sm + kHalfX);
    const uint32_t xch_mine = smem_u32(&xch[(int)rank * 128 + row]);
    const uint32_t slot_stride = (uint32_t)(nclus * 128 * 8);
    const float4* cz4 = reinterpret_cast<const float4*>(c_lz + k0);
    const float4* cc4 = reinterpret_cast<const float4*>(c_c2 + k0);
    const float4* cm4 = reinterpret_cast<const float4*>(c_mpm + k0);  // spherical
    // this part's logits (log2 units) from S in place, and its four-way max:
    // diag min(lz - h S, c2) with h = log2(e)/2; tied lz - h S (without the
    // row's x^T P x, no clamp); spherical c2 - h_k max(S + |x|^2 + mpm_k, 0)
    auto logits = [&](float qn, float (&mx)[4]) {
#pragma unroll
      for (int k4 = 0; k4 < kPart / 4; ++k4) {
        const float4 vz = cz4[k4], vc = cc4[k4];
        const float lz[4] = {vz.x, vz.y, vz.z, vz.w}, cc[4] = {vc.x, vc.y, vc.z, vc.w};
        float mm[4] = {0.f, 0.f, 0.f, 0.f};
        if constexpr (kSph) {
          const float4 vm = cm4[k4];
          mm[0] = vm.x; mm[1] = vm.y; mm[2] = vm.z; mm[3] = vm.w;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int k = 4 * k4 + j;
          float l;
          if constexpr (kSph) l = fmaf(-cc[j], fmaxf(p[k] + (mm[j] + qn), 0.f), lz[j]);
          else if constexpr (kTied) l = fmaf(-kHalfLog2e, p[k], lz[j]);
          else l = fminf(fmaf(-kHalfLog2e, p[k], lz[j]), cc[j]);
          p[k] = l;
          mx[j] = fmaxf(mx[j], l);
        }
      }
    };
    // this row's |x|^2 for tile t (spherical; written by the prep warps)
    auto row_q = [&](int t, float& qn) -> bool {
      if constexpr (kSph) {
        if (!mbar_wait_warp(&bars->qfull[t & 1], (t >> 1) & 1, abort, lim)) return false;
        qn = qbuf[(t & 1) * 128 + row];
      }
      return true;
    };
    // kModeExtLse: the row's log-sum-exp over all K (log2 units), loaded one
    // tile ahead so that its latency hides behind the current tile
    auto ext_lse = [&](int u) -> float {
      const int64_t r = (cid + (int64_t)u * ncl) * kBM + row;
      return (u < T && r < a.N) ? __ldg(a.lse_in + r) : 0.f;
    };
    float lse_next = kNoXch ? ext_lse(0) : 0.f;
    // R holds two 64-component MN groups; this part's components are 16-byte
    // chunks rc0 .. rc0 + kPart / 8 - 1 of group k0 / 64
    char* rg = sm + kR + (k0 / 64) * kBlock;
    const int rc0 = (k0 % 64) / 8;
    auto store_r = [&](const uint32_t* w) {
#pragma unroll
      for (int c = 0; c < kPart / 8; ++c)
        *reinterpret_cast<uint4*>(rg + sw128((uint32_t)row, (uint32_t)((rc0 + c) * 8))) =
            make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->rfull);
    };
    bool ok = true;
    if constexpr (kEm) {
      for (int t = 0; t < T; ++t) {
        const int s = t & 1;
        const int64_t grow = (cid + (int64_t)t * ncl) * kBM + row;
        const bool valid = grow < a.N;
        if (!mbar_wait_warp(&bars->sfull[0], t & 1, abort, lim)) { ok = false; break; }
        tmem_fence_after();
        const uint32_t sc = tmem + lane_addr + kSCol + (uint32_t)k0;
  #pragma unroll
        for (int c = 0; c < kPart / 32; ++c) tmem_ld32(sc + 32 * c, p + 32 * c);
        float yv[16];  // tied: this part's piece of y = L^-1 x
        if (kTied && qc < ny) tmem_ld16(tmem + lane_addr + kSCol + kKC + 16 * qc, yv);
        const float lse_t = lse_next;
        if constexpr (kExt) lse_next = ext_lse(t + 1);
        float qn = 0.f;
        if (!row_q(t, qn)) { ok = false; break; }  // read before S(t) is released
        tmem_wait_ld();
        tmem_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->sfree[0]);
        float qy = 0.f;  // tied: the piece's share of |y|^2 = x^T P x
        if (kTied && qc < ny) {
  #pragma unroll
          for (int i = 0; i < 16; ++i) qy = fmaf(yv[i], yv[i], qy);
        }
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        logits(qn, mx);
        // residual part of the previous tile (the M-step's high part of t-1 ran meanwhile)
        if (t >= 1) {
          if (!mbar_wait_warp(&bars->rfree, 0u, abort, lim)) { ok = false; break; }  // M_hi(t-1)
          store_r(lo);
        }
        const float m = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        float f = 0.f, M = 0.f, S = 1.f;
        if constexpr (kExt) {  // r = 2^(l - lse): no row reduction, no exchange
  #pragma unroll
          for (int k = 0; k < kPart; ++k) p[k] = ex2_approx(p[k] - lse_t);
          f = valid ? 1.f : 0.f;
        } else {
        const float mref = (m == -INFINITY) ? 0.f : m;  // an all-padding part has p = 0
        float sm4[4] = {0.f, 0.f, 0.f, 0.f};
  #pragma unroll
        for (int k = 0; k < kPart; ++k) {
          p[k] = ex2_approx(p[k] - mref);
          sm4[k & 3] += p[k];
        }
        const float sum = (sm4[0] + sm4[1]) + (sm4[2] + sm4[3]);
        // combine the parts of the row (slot t & 1: a part writes the slot of
        // tile t+2 only after the barrier of tile t+1, which every other part
        // passes after reading its entries of tile t)
        float2* hxs = halfx + s * kSplit * 128;
        hxs[qc * 128 + row] = make_float2(m, sum);
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->hx[s]);
        if (!mbar_wait_warp(&bars->hx[s], (t >> 1) & 1, abort, lim)) { ok = false; break; }
        float2 o[kSplit];
  #pragma unroll
        for (int q = 0; q < kSplit; ++q) o[q] = q == qc ? make_float2(m, sum) : hxs[q * 128 + row];
        float mc = o[0].x;
  #pragma unroll
        for (int q = 1; q < kSplit; ++q) mc = fmaxf(mc, o[q].x);
        // exponents <= 0 here; ex2.approx (relative error ~2^-22) flushes results
        // below 2^-126, i.e. parts 2^126 times smaller than the row's largest.
        // Every CTA owns at least one live component, so mc is finite.
        float sc2 = 0.f;
  #pragma unroll
        for (int q = 0; q < kSplit; ++q) sc2 += o[q].y * ex2_approx(o[q].x - mc);
        // exchange (max, sum) of this CTA's components with the cluster (part 0 sends)
        if (qc == 0) {
          if (tid == kWarpSoftmax0 * 32) mbar_expect_tx(&bars->xch[s], (uint32_t)(nclus * 128 * 8));
  #pragma unroll
          for (int q = 0; q < kMaxCluster; ++q)
            if (q < nclus)
              st_async_f2(map_shared(xch_mine + s * slot_stride, q), mc, sc2, map_shared(smem_u32(&bars->xch[s]), q));
        }
        if (!mbar_wait_warp(&bars->xch[s], (t >> 1) & 1, abort, lim)) { ok = false; break; }
        float2 e[kMaxCluster];
  #pragma unroll
        for (int q = 0; q < kMaxCluster; ++q)
          e[q] = q < nclus ? xch[(s * nclus + q) * 128 + row] : make_float2(-INFINITY, 0.f);
        M = e[0].x;
  #pragma unroll
        for (int q = 1; q < kMaxCluster; ++q) M = fmaxf(M, e[q].x);
        S = 0.f;
  #pragma unroll
        for (int q = 0; q < kMaxCluster; ++q)
          if (q < nclus) S += e[q].y * ex2_approx(e[q].x - M);
        f = valid ? ex2_approx(m - M) * __frcp_rn(S) : 0.f;
        }
        // high part of tile t now (after the M-step's residual part of t-1);
        // the residual words stay in registers for the next iteration
        if (t >= 1 && !mbar_wait_warp(&bars->rfree, 1u, abort, lim)) { ok = false; break; }  // M_lo(t-1)
  #pragma unroll
        for (int c = 0; c < kPart / 8; ++c) {  // 8 components per 16-byte store
          uint32_t hw[4];
  #pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int k = 8 * c + 2 * i;
            const float r0 = p[k] * f, r1 = p[k + 1] * f;
            hw[i] = pack_bf16(r0, r1);
            lo[4 * c + i] = pack_bf16(r0 - bf16lo_to_f32(hw[i]), r1 - bf16hi_to_f32(hw[i]));
          }
          *reinterpret_cast<uint4*>(rg + sw128((uint32_t)row, (uint32_t)((rc0 + c) * 8))) =
              make_uint4(hw[0], hw[1], hw[2], hw[3]);
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->rfull);
        if (!kExt && valid && rank == 0 && qc == 0) ll_acc += (double)((M + log2f(S)) * kLn2);
        if (kTied && valid) ll_acc -= 0.5 * (double)qy;  // the row's -x^T P x / 2, piece by piece
        if (*abort) { ok = false; break; }
      }
      // the residual part of the last tile
      if (ok && T >= 1) {
        if (mbar_wait_warp(&bars->rfree, 0u, abort, lim)) store_r(lo);
        else ok = false;
      }
    } else {
      // responsibilities p[k] * f of tile t, fp32 [N][K]: the tile's rows are
      // staged in the (here unused) M-step stage and R buffer, [128 rows][128
      // components] with the 16-byte chunks of a row permuted by row & 7, then
      // every warp stores 8 whole rows of this CTA's components as 512-byte
      // runs (an unaligned output or K % 4 != 0: each thread its own values)
      auto store_proba = [&](int t, float f) -> bool {
        const int64_t grow = (cid + (int64_t)t * ncl) * kBM + row;
        const int comp0 = chunk * kKC + k0;
        if (!a.out_vec) {
          if (grow < a.N) {
            float* orow = a.out_f + grow * (int64_t)a.K + comp0;
#pragma unroll
            for (int k = 0; k < kPart; ++k)
              if (comp0 + k < a.K) orow[k] = p[k] * f;
          }
          return true;
        }
        float* stg = reinterpret_cast<float*>(sm + kMX);
        if (t >= 1 && !mbar_wait_warp(&bars->pfree, (t - 1) & 1, abort, lim)) return false;
#pragma unroll
        for (int c = 0; c < kPart / 4; ++c) {
          const int pos = ((k0 >> 2) + c) ^ (row & 7);
          *reinterpret_cast<float4*>(stg + row * kKC + pos * 4) =
              make_float4(p[4 * c] * f, p[4 * c + 1] * f, p[4 * c + 2] * f, p[4 * c + 3] * f);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->pfull);
        if (!mbar_wait_warp(&bars->pfull, t & 1, abort, lim)) return false;
        const int sw = warp - kWarpSoftmax0;
        const int comp = chunk * kKC + 4 * lane;
#pragma unroll 2
        for (int i = 0; i < kBM / kSoftWarps; ++i) {
          const int r = sw * (kBM / kSoftWarps) + i;
          const int64_t gr = (cid + (int64_t)t * ncl) * kBM + r;
          const float4 v = *reinterpret_cast<const float4*>(stg + r * kKC + ((lane ^ (r & 7)) * 4));
          if (gr < a.N) {
            float* o = a.out_f + gr * (int64_t)a.K + comp;
            if (comp + 3 < a.K) {
              *reinterpret_cast<float4*>(o) = v;
            } else {
              if (comp < a.K) o[0] = v.x;
              if (comp + 1 < a.K) o[1] = v.y;
              if (comp + 2 < a.K) o[2] = v.z;
            }
          }
        }
        // the staged values went into the stores above: the stage is free
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->pfree);
        return true;
      };
      // inference: the logits and the row's cluster-wide reduction only
      if constexpr (kMode == kModeRowStat) {
        // Software-pipelined over three tiles, so that the wait for the row's
        // other parts and the cluster exchange overlap the next tile's
        // logits.  Iteration t: A(t) this part's (max, sum) of tile t into
        // slot t % 4 of the part table; C(t - 2) the cluster's (max, sum) of
        // tile t - 2 into rowstat; B(t - 1) the row's four parts of tile t - 1
        // combined and sent to the cluster.  The part table lives in the R
        // buffer's second block (no M-step here; the first block is staging
        // slot 2).  Reuse: a part writes slot t % 4 once S(t) is complete,
        // i.e. after every warp loaded S(t - 2) (two S slots), which part 0
        // does only after its B(t - 4); the cluster writes exchange slot
        // (t + 1) & 1 of this CTA after its own C(t) (B after C within an
        // iteration), which follows this CTA's B(t) and so its C(t - 1).
        float2* parts = reinterpret_cast<float2*>(sm + kR + kBlock);  // [4][kSplit][128]
        static_assert(4 * kSplit * 128 * 8 <= kBlock, "part table in the R buffer's second block");
        for (int t = 0; t < T + 2; ++t) {
          if (t < T) {  // A(t)
            if (!mbar_wait_warp(&bars->sfull[t & 1], (t >> 1) & 1, abort, lim)) { ok = false; break; }
            tmem_fence_after();
            const uint32_t sc = tmem + lane_addr + kSCol + (uint32_t)((t & 1) * kS1Off + k0);
#pragma unroll
            for (int c = 0; c < kPart / 32; ++c) tmem_ld32(sc + 32 * c, p + 32 * c);
            float qn = 0.f;
            if (!row_q(t, qn)) { ok = false; break; }  // read before S(t) is released
            tmem_wait_ld();
            tmem_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->sfree[t & 1]);
            float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            logits(qn, mx);
            const float m = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
            const float mref = (m == -INFINITY) ? 0.f : m;
            float sm4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int k = 0; k < kPart; ++k) sm4[k & 3] += ex2_approx(p[k] - mref);
            parts[((t & 3) * kSplit + qc) * 128 + row] = make_float2(m, (sm4[0] + sm4[1]) + (sm4[2] + sm4[3]));
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->hx[t & 3]);
          }
          if (qc == 0 && t >= 2) {  // C(t - 2)
            const int u = t - 2, su = u & 1;
            if (!mbar_wait_warp(&bars->xch[su], (u >> 1) & 1, abort, lim)) { ok = false; break; }
            float2 e[kMaxCluster];
#pragma unroll
            for (int q = 0; q < kMaxCluster; ++q)
              e[q] = q < nclus ? xch[(su * nclus + q) * 128 + row] : make_float2(-INFINITY, 0.f);
            float M = e[0].x;
#pragma unroll
            for (int q = 1; q < kMaxCluster; ++q) M = fmaxf(M, e[q].x);
            float S = 0.f;
#pragma unroll
            for (int q = 0; q < kMaxCluster; ++q)
              if (q < nclus) S += e[q].y * ex2_approx(e[q].x - M);
            const int64_t gu = (cid + (int64_t)u * ncl) * kBM + row;
            if (gu < a.N && rank == 0) a.rowstat[gu] = make_float2(M, S);  // log2 units
          }
          if (qc == 0 && t >= 1 && t <= T) {  // B(t - 1)
            const int u = t - 1, hu = u & 3, su = u & 1;
            if (!mbar_wait_warp(&bars->hx[hu], (u >> 2) & 1, abort, lim)) { ok = false; break; }
            float2 o[kSplit];
#pragma unroll
            for (int q = 0; q < kSplit; ++q) o[q] = parts[(hu * kSplit + q) * 128 + row];
            float mc = o[0].x;
#pragma unroll
            for (int q = 1; q < kSplit; ++q) mc = fmaxf(mc, o[q].x);
            float sc2 = 0.f;
#pragma unroll
            for (int q = 0; q < kSplit; ++q) sc2 += o[q].y * ex2_approx(o[q].x - mc);
            if (tid == kWarpSoftmax0 * 32) mbar_expect_tx(&bars->xch[su], (uint32_t)(nclus * 128 * 8));
#pragma unroll
            for (int q = 0; q < kMaxCluster; ++q)
              if (q < nclus)
                st_async_f2(map_shared(xch_mine + su * slot_stride, q), mc, sc2,
                            map_shared(smem_u32(&bars->xch[su]), q));
          }
          if (*abort) { ok = false; break; }
        }
      } else
      for (int t = 0; t < T; ++t) {
        const int s = t & 1;
        const int64_t grow = (cid + (int64_t)t * ncl) * kBM + row;
        const bool valid = grow < a.N;
        if (!mbar_wait_warp(&bars->sfull[0], t & 1, abort, lim)) { ok = false; break; }
        tmem_fence_after();
        const uint32_t sc = tmem + lane_addr + kSCol + (uint32_t)k0;
#pragma unroll
        for (int c = 0; c < kPart / 32; ++c) tmem_ld32(sc + 32 * c, p + 32 * c);
        const float lse_t = lse_next;
        if constexpr (kNoXch) lse_next = ext_lse(t + 1);
        float qn = 0.f;
        if (!row_q(t, qn)) { ok = false; break; }  // read before S(t) is released
        tmem_wait_ld();
        tmem_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->sfree[0]);
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        logits(qn, mx);
        float2* hxs = halfx + s * kSplit * 128;
        const int comp0 = chunk * kKC + k0;  // global index of p[0]
        if constexpr (kMode == kModeProbaExt) {
          // r = 2^(l - lse) from the row's log-sum-exp over all K
#pragma unroll
          for (int k = 0; k < kPart; ++k) p[k] = ex2_approx(p[k] - lse_t);
          if (!store_proba(t, valid ? 1.f : 0.f)) { ok = false; break; }
          if (*abort) { ok = false; break; }
          continue;
        }
        float m = 0.f, sum = 0.f;
        float2 mine;
        if constexpr (kMode == kModeArgmax) {
          // this part's largest logit and its first component (increasing k)
          float bv = -INFINITY;
          int bi = 0x7fffffff;
#pragma unroll
          for (int k = 0; k < kPart; ++k)
            if (p[k] > bv) { bv = p[k]; bi = comp0 + k; }
          mine = make_float2(bv, __int_as_float(bi));
        } else {
          m = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
          const float mref = (m == -INFINITY) ? 0.f : m;
          float sm4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int k = 0; k < kPart; ++k) {
            p[k] = ex2_approx(p[k] - mref);
            sm4[k & 3] += p[k];
          }
          sum = (sm4[0] + sm4[1]) + (sm4[2] + sm4[3]);
          mine = make_float2(m, sum);
        }
        // combine the parts of the row (slot t & 1, as in the EM loop)
        hxs[qc * 128 + row] = mine;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->hx[s]);
        if (!mbar_wait_warp(&bars->hx[s], (t >> 1) & 1, abort, lim)) { ok = false; break; }
        float2 o[kSplit];
#pragma unroll
        for (int q = 0; q < kSplit; ++q) o[q] = q == qc ? mine : hxs[q * 128 + row];
        float2 cta;
        if constexpr (kMode == kModeArgmax) {
          cta = o[0];  // parts in increasing component order: strictly larger wins
#pragma unroll
          for (int q = 1; q < kSplit; ++q)
            if (o[q].x > cta.x) cta = o[q];
        } else {
          float mc = o[0].x;
#pragma unroll
          for (int q = 1; q < kSplit; ++q) mc = fmaxf(mc, o[q].x);
          float sc2 = 0.f;
#pragma unroll
          for (int q = 0; q < kSplit; ++q) sc2 += o[q].y * ex2_approx(o[q].x - mc);
          cta = make_float2(mc, sc2);
        }
        if (qc == 0) {
          if (tid == kWarpSoftmax0 * 32) mbar_expect_tx(&bars->xch[s], (uint32_t)(nclus * 128 * 8));
#pragma unroll
          for (int q = 0; q < kMaxCluster; ++q)
            if (q < nclus)
              st_async_f2(map_shared(xch_mine + s * slot_stride, q), cta.x, cta.y, map_shared(smem_u32(&bars->xch[s]), q));
        }
        if (!mbar_wait_warp(&bars->xch[s], (t >> 1) & 1, abort, lim)) { ok = false; break; }
        float2 e[kMaxCluster];
#pragma unroll
        for (int q = 0; q < kMaxCluster; ++q)
          e[q] = q < nclus ? xch[(s * nclus + q) * 128 + row] : make_float2(-INFINITY, 0.f);
        if constexpr (kMode == kModeArgmax) {
          float2 best = e[0];  // ranks in increasing component order: strictly larger wins
#pragma unroll
          for (int q = 1; q < kMaxCluster; ++q)
            if (q < nclus && e[q].x > best.x) best = e[q];
          if (valid && rank == 0 && qc == 0) {
            if (a.rowstat != nullptr) a.rowstat[grow] = best;  // grouped: (max, first component) of the group
            else a.out_i[grow] = (int64_t)__float_as_int(best.y);
          }
        } else {
          float M = e[0].x;
#pragma unroll
          for (int q = 1; q < kMaxCluster; ++q) M = fmaxf(M, e[q].x);
          float S = 0.f;
#pragma unroll
          for (int q = 0; q < kMaxCluster; ++q)
            if (q < nclus) S += e[q].y * ex2_approx(e[q].x - M);
          if constexpr (kMode == kModeRowStat) {
            // the row's (max, scaled sum) over this group's components (log2 units)
            if (valid && rank == 0 && qc == 0) a.rowstat[grow] = make_float2(M, S);
          } else if constexpr (kMode == kModeLse) {
            if (valid && rank == 0 && qc == 0) a.out_f[grow] = (M + log2f(S)) * kLn2;
          } else {
            if (!store_proba(t, valid ? ex2_approx(m - M) * __frcp_rn(S) : 0.f)) { ok = false; break; }
          }
        }
        if (*abort) { ok = false; break; }
      }
    }
    if (!ok) set_abort(bars, a.status);
    // ---------------- epilogue: statistics partials (all softmax warps) ----------------
    // the MMA thread always commits `mdone` (also after an abort): wait for it
    // without the abort shortcut before touching tensor memory again.  TMEM
    // lane = component; columns [x | s_hi | s_lo | 1].  Parts 0, 1 write the
    // sums of r x (32 features each), parts 2, 3 those of r x^2 = s_hi + s_lo
    // columns, part 0 also n_k.
    if (!mbar_wait_warp(&bars->mdone, 0, nullptr, 2 * lim)) set_abort(bars, a.status);
    tmem_fence_after();
    if constexpr (kEm) {
      static_assert(kSplit == 4, "epilogue column split");
      const int comp = (int)rank * kKC + row;
      float* out = a.part + ((int64_t)cid * a.Kp + comp) * a.F;
      const uint32_t dm = tmem + lane_addr + kDmCol;
      float v[32];
      if constexpr (kSph) {
        // columns [x (128) | 1 | |x|^2 in three terms]: part qc writes the
        // sums of r x for features 32 qc .. 32 qc + 31, part 0 also n_k and
        // sum r |x|^2
        tmem_ld32(dm + 32 * qc, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) out[1 + 32 * qc + j] = v[j];
        if (qc == 0) {
          tmem_ld16(dm + 128, v);
          tmem_wait_ld();
          out[0] = v[0];
          out[1 + 128] = v[1] + (v[2] + v[3]);
        }
      } else if constexpr (kTied) {
        // columns [x_hi | x_mid | x_lo | 1]: part qc sums features 16 qc .. 16 qc + 15
        float v1[16], v2[16];
        tmem_ld16(dm + 16 * qc, v);
        tmem_ld16(dm + 64 + 16 * qc, v1);
        tmem_ld16(dm + 128 + 16 * qc, v2);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) out[1 + 16 * qc + j] = v[j] + (v1[j] + v2[j]);
        if (qc == 0) {
          tmem_ld16(dm + 192, v);  // the first column is n_k
          tmem_wait_ld();
          out[0] = v[0];
        }
      } else if (qc < 2) {
        tmem_ld32(dm + 32 * qc, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) out[1 + 32 * qc + j] = v[j];
      } else {
        const int f0 = 32 * (qc - 2);
        float w2[16];
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // 16 features at a time: fewer live registers
          tmem_ld16(dm + 64 + f0 + 16 * h, v);
          tmem_ld16(dm + 128 + f0 + 16 * h, w2);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) out[1 + 64 + f0 + 16 * h + j] = v[j] + w2[j];
        }
      }
      if (kCov == GMMXX_DIAG && qc == 0) {
        tmem_ld32(dm + 192, v);  // 32 columns; the first is n_k
        tmem_wait_ld();
        out[0] = v[0];
      }
    }
    tmem_fence_before();
    if constexpr (kTied) {  // every part of every rank holds log-likelihood terms
      double* red = reinterpret_cast<double*>(sm + Y::red(nclus));
      double v = ll_acc;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[warp - kWarpSoftmax0] = v;
      asm volatile("bar.sync 2, %0;" ::"n"(kSoftWarps * 32) : "memory");
      if (tid == kWarpSoftmax0 * 32) {
        double t = 0.0;
#pragma unroll
        for (int i = 0; i < kSoftWarps; ++i) t += red[i];
        a.part_ll[(int64_t)cid * nclus + rank] = t;
      }
    } else if (kMode == kModeEm && qc == 0) {
      double* red = reinterpret_cast<double*>(sm + Y::red(nclus));
      double v = ll_acc;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[q4] = v;
      asm volatile("bar.sync 2, 128;" ::: "memory");
      if (tid == kWarpSoftmax0 * 32 && rank == 0) a.part_ll[cid] = red[0] + red[1] + red[2] + red[3];
    }
  }
  __syncthreads();
  if (warp == kWarpMma) {
    tmem_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  cluster_sync();  // no CTA exits while a peer may still write into its shared memory
}

// One clustered launch.  The grouped spherical passes cover chunks
// [chunk0, chunk0 + csize) of 128 components (csize < 0: the whole of L).
template <int kMode, int kCov = GMMXX_DIAG>
static int launch_mode(const TcLaunch& L0, const CUtensorMap& tmap, cudaStream_t st, int* ncl_out, int chunk0 = 0,
                       int csize = -1, const float* lse_in = nullptr, float2* rowstat = nullptr) {
  TcLaunch L = L0;
  if (csize > 0) {
    L.cluster_size = csize;
    L.Kp_part = (int64_t)csize * kKC;
  }
  auto kern = em_tc_diag_kernel<kMode, kCov>;
  const int smem = Lay<kCov>::total(L.cluster_size);
  // kModeExtLse and kModeProbaExt exchange nothing within a cluster: they run as virtual
  // clusters of single CTAs on every SM instead of the co-resident clusters
  const bool virt = (kMode == kModeExtLse || kMode == kModeProbaExt) && L.cluster_size > 1;
  TcLaunch Lq = L;
  if (virt) Lq.cluster_size = 1;
  int ncl = 0;
  if (int rc = clustered_launch((const void*)kern, kThreads, smem, Lq, &ncl)) return rc;
  if (virt) ncl /= L.cluster_size;  // whole virtual clusters
  if (ncl < 1) return set_error(GMMXX_ERR_UNSUPPORTED, "too few co-resident CTAs for %d-chunk groups", L.cluster_size);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = virt ? 1 : L.cluster_size;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3((unsigned)(ncl * L.cluster_size));
  TcArgs args{};
  args.N = L.N;
  args.Kp = L.Kp_part;
  args.F = L.F;
  args.cluster_size = L.cluster_size;
  args.params = L.params;
  args.consts = L.consts;
  args.part = L.part;
  args.part_ll = L.part_ll;
  args.status = L.status;
  args.wait_ns = L.wait_ns ? L.wait_ns : 2000000000ull;
  args.test_stall = L.test_stall;
  args.K = L.K;
  args.out_f = L.out_f;
  args.out_i = L.out_i;
  args.out_vec = ((reinterpret_cast<uintptr_t>(L.out_f) & 15u) == 0 && (L.K & 3) == 0) ? 1 : 0;
  args.chunk0 = chunk0;
  args.lse_in = lse_in;
  args.rowstat = rowstat;
  args.vcluster = virt ? L.cluster_size : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tmap, args);
  if (e != cudaSuccess)
    return set_error(GMMXX_ERR_CUDA, "em_tc_diag_kernel<%d, %d> launch: %s", kMode, kCov, cudaGetErrorString(e));
  *ncl_out = ncl;
  return GMMXX_OK;
}

}  // namespace

int launch_em_tc_diag(const TcLaunch& L, cudaStream_t st) {
  if (L.D != 64 || L.cluster_size < 1 || L.cluster_size > kMaxCluster)
    return set_error(GMMXX_ERR_UNSUPPORTED, "diag tensor-core kernel: D = 64, K <= %d", 128 * kMaxCluster);
  if (L.infer < 0 || L.infer > 3) return set_error(GMMXX_ERR_INVALID, "diag tensor-core kernel: mode %d", L.infer);
  if ((L.infer == kModeLse || L.infer == kModeProba) && L.out_f == nullptr)
    return set_error(GMMXX_ERR_INVALID, "diag tensor-core kernel: no output buffer");
  if (L.infer == kModeArgmax && L.out_i == nullptr)
    return set_error(GMMXX_ERR_INVALID, "diag tensor-core kernel: no label buffer");
  if (int rc = launch_tc_pack(GMMXX_DIAG, 1, L, st)) return rc;
  CUtensorMap tmap;
  if (int rc = make_x_tensor_map(L, &tmap)) return rc;
  int ncl = 0;
  int rc = GMMXX_OK;
  switch (L.infer) {
    case kModeEm: rc = launch_mode<kModeEm>(L, tmap, st, &ncl); break;
    case kModeLse: rc = launch_mode<kModeLse>(L, tmap, st, &ncl); break;
    case kModeArgmax: rc = launch_mode<kModeArgmax>(L, tmap, st, &ncl); break;
    default: rc = launch_mode<kModeProba>(L, tmap, st, &ncl); break;
  }
  if (rc != GMMXX_OK || L.infer != kModeEm) return rc;
  return launch_tc_reduce(L, ncl, st);
}

// Tied covariance, fp32 X, D = 64, K <= 512: EM statistics (no inference
// modes); the log-likelihood partials come one per cluster rank.
int launch_em_tc_tied(const TcLaunch& L, cudaStream_t st) {
  if (L.D != 64 || L.cluster_size < 1 || L.cluster_size > kMaxCluster || L.nchunks != L.cluster_size)
    return set_error(GMMXX_ERR_UNSUPPORTED, "tied tensor-core kernel: D = 64, K <= %d", 128 * kMaxCluster);
  if (L.infer != kModeEm) return set_error(GMMXX_ERR_UNSUPPORTED, "tied tensor-core kernel: EM statistics only");
  if (int rc = launch_tc_pack(GMMXX_TIED, 1, L, st)) return rc;
  CUtensorMap tmap;
  if (int rc = make_x_tensor_map(L, &tmap, true)) return rc;
  int ncl = 0;
  if (int rc = launch_mode<kModeEm, GMMXX_TIED>(L, tmap, st, &ncl)) return rc;
  return launch_tc_reduce(L, ncl, st, ncl * L.cluster_size);
}

// Spherical inference, one pass (K <= 512) or grouped: labels from each
// group's (max, first component), the log-sum-exp from each group's row
// statistics, the responsibilities of each group from the combined log2
// log-sum-exp (no cluster exchange).
static int sph128_infer(const TcLaunch& L, const CUtensorMap& tmap, bool one_pass, cudaStream_t st) {
  int ncl = 0;
  if (one_pass) {
    switch (L.infer) {
      case kModeLse: return launch_mode<kModeLse, GMMXX_SPHERICAL>(L, tmap, st, &ncl);
      case kModeArgmax: return launch_mode<kModeArgmax, GMMXX_SPHERICAL>(L, tmap, st, &ncl);
      default: return launch_mode<kModeProba, GMMXX_SPHERICAL>(L, tmap, st, &ncl);
    }
  }
  // per-row passes in groups of kRowStatChunks chunks (clusters of 2), the
  // responsibilities in groups of kGroupChunks (no clusters)
  const int nch = L.nchunks, g1 = kRowStatChunks, groups1 = (nch + g1 - 1) / g1;
  for (int g = 0; g < groups1; ++g) {
    const int csize = std::min(g1, nch - g * g1);
    float2* rs = L.rowstat + (int64_t)g * L.N;
    const int rc = L.infer == kModeArgmax
                       ? launch_mode<kModeArgmax, GMMXX_SPHERICAL>(L, tmap, st, &ncl, g * g1, csize, nullptr, rs)
                       : launch_mode<kModeRowStat, GMMXX_SPHERICAL>(L, tmap, st, &ncl, g * g1, csize, nullptr, rs);
    if (rc) return rc;
  }
  if (int rc = launch_infer_combine(L, groups1, L.infer, st)) return rc;
  if (L.infer != kModeProba) return GMMXX_OK;
  const int gc = kGroupChunks, groups = (nch + gc - 1) / gc;
  for (int g = 0; g < groups; ++g) {
    const int csize = std::min(gc, nch - g * gc);
    if (int rc = launch_mode<kModeProbaExt, GMMXX_SPHERICAL>(L, tmap, st, &ncl, g * gc, csize, L.lse, nullptr))
      return rc;
  }
  return GMMXX_OK;
}

// Spherical, bf16 X, D = 128, EM statistics: K <= 512 in one pass over a
// cluster of ceil(K / 128) CTAs; K > 1024 in two passes -- row statistics
// per group of 2 chunks (256 components, clusters of 2), their combination
// into each row's log-sum-exp and the log-likelihood, then per group of 4
// chunks the responsibilities from it and the M-step (no cluster exchange).
// Inference (TcLaunch::infer 1-3) runs on the same layouts.
int launch_em_tc_sph128(const TcLaunch& L, cudaStream_t st) {
  if (L.D != 128 || L.infer < 0 || L.infer > 3)
    return set_error(GMMXX_ERR_UNSUPPORTED, "spherical kernel: D = 128, mode %d", L.infer);
  const int nch = L.nchunks;
  const bool one_pass = nch <= kMaxCluster && L.cluster_size == nch;
  const bool grouped = nch > kMaxClusterSph && L.cluster_size == kGroupChunks;
  if (!one_pass && !grouped) return set_error(GMMXX_ERR_UNSUPPORTED, "spherical kernel: %d chunks", nch);
  if (grouped && (L.rowstat == nullptr || L.lse == nullptr))
    return set_error(GMMXX_ERR_WORKSPACE, "grouped pass buffers missing");
  if ((L.infer == kModeLse || L.infer == kModeProba) && L.out_f == nullptr)
    return set_error(GMMXX_ERR_INVALID, "spherical kernel: no output buffer");
  if (L.infer == kModeArgmax && L.out_i == nullptr)
    return set_error(GMMXX_ERR_INVALID, "spherical kernel: no label buffer");
  if (int rc = launch_tc_pack(GMMXX_SPHERICAL, 2, L, st)) return rc;
  CUtensorMap tmap;
  if (int rc = make_x_tensor_map(L, &tmap)) return rc;
  if (L.infer != kModeEm) return sph128_infer(L, tmap, one_pass, st);
  int ncl = 0;
  if (one_pass) {
    if (int rc = launch_mode<kModeEm, GMMXX_SPHERICAL>(L, tmap, st, &ncl)) return rc;
    return launch_tc_reduce(L, ncl, st);
  }
  // first pass in groups of kRowStatChunks chunks (clusters of 2), the
  // second in groups of kGroupChunks (no clusters)
  const int g1 = kRowStatChunks, groups1 = (nch + g1 - 1) / g1;
  for (int g = 0; g < groups1; ++g) {
    const int csize = std::min(g1, nch - g * g1);
    if (int rc = launch_mode<kModeRowStat, GMMXX_SPHERICAL>(L, tmap, st, &ncl, g * g1, csize, nullptr,
                                                            L.rowstat + (int64_t)g * L.N))
      return rc;
  }
  if (int rc = launch_rowstat_combine(L, groups1, st)) return rc;
  const int gc = kGroupChunks, groups = (nch + gc - 1) / gc;
  for (int g = 0; g < groups; ++g) {
    const int csize = std::min(gc, nch - g * gc);
    const int rc = sph_ext_enabled()
                       ? launch_sph_ext(L, tmap, g * gc, csize, st, &ncl)
                       : launch_mode<kModeExtLse, GMMXX_SPHERICAL>(L, tmap, st, &ncl, g * gc, csize, L.lse, nullptr);
    if (rc) return rc;
    TcLaunch Lg = L;  // statistics rows of this group's components
    const int k0 = g * gc * kKC;
    Lg.stats = L.stats + (int64_t)k0 * L.F;
    Lg.K = std::min(gc * kKC, L.K - k0);
    Lg.Kp_part = (int64_t)csize * kKC;
    Lg.ll = nullptr;
    if (int rc = launch_tc_reduce(Lg, ncl, st)) return rc;
  }
  return GMMXX_OK;
}

}  // namespace tc
}  // namespace gmmxx
