// em_tc.cu -- fused soft-EM statistics kernel on the 5th-generation tensor
// cores (tcgen05 + TMEM + TMA) for bf16 X with spherical covariance
// (D = 64 / 128; K <= 1024 in one pass, K <= 16384 in groups of 512
// components), B == 1, with E-step-only passes for inference (labels,
// score_samples, predict_proba); plus the host pieces every tensor-core
// kernel shares: the per-iteration weight-image packer, the tensor map of X,
// the clustered launch and the fixed-order reduction of the partials.  The
// diagonal-covariance kernel is em_tc_diag.cu.
//
// One thread-block cluster of C = ceil(K / 128) CTAs works on the same
// 128-row tile of X at a time; CTA `rank` owns components
// [128 rank, 128 rank + 128) whose split-bf16 logit weights stay resident in
// its shared memory for the whole launch.  Per row tile:
//
//   TMA          X tile (bf16, 128-byte swizzle) -> shared memory
//   prep warps   |x|^2 per row (the aux operand and the softmax's q)
//   MMA warp     E-step  S[128 rows, 128 comps] (TMEM, fp32) = x . W^T
//   softmax WG   logits from S, row max / exp / partial sum -> DSMEM exchange
//                of (max, sum) with the cluster peers -> r = exp(l - lse),
//                split r = r_hi + r_lo (two bf16) into shared memory
//   MMA warp     M-step  stats[128 comps, F] (TMEM, fp32) += R^T . [x | 1 | |x|^2]
//
// so the (N, K) responsibilities never leave the SM and X is read from HBM
// once per iteration.  Precision: X is exact in bf16; the logit weights are
// split into three bf16 terms (24 significant bits, fp32-equivalent); r into
// two (16 bits).  Products are exact and accumulate in fp32, so logits match
// the fp32 expanded-distance form.  Statistics leave the kernel once per
// cluster as partials that a second kernel reduces in a fixed order
// (run-to-run deterministic).
//
// Reference semantics: gmmxx/torch_fallback.py:2097-2291 (spherical E/M
// chunk loop), expanded-distance logits 337-354.
#include "gmm_common.cuh"
#include "tc_ptx.cuh"
#include "tc_api.cuh"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <type_traits>

namespace gmmxx {
namespace tc {

using namespace ptx;

constexpr int kBM = 128;          // rows per tile (UMMA M of the E-step)
constexpr int kKC = 128;          // components per CTA
constexpr int kNS = 3;            // bf16 terms of the split component weights (24 significant bits)
constexpr int kThreads = 384;     // 12 warps: TMA, MMA, 2 prep, 8 softmax
constexpr int kHalf = kKC / 2;    // components per softmax thread (two warps share a row)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kDmCol = 256;  // M-step accumulator columns [256, 256 + FDM)
constexpr int kBlock = 16384;     // one [128][64] bf16 swizzled block
constexpr int kAuxBytes = 4096;   // [16][128] K-major aux operand (1, |x|^2 hi / lo)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// 2^x on the SFU (ex2.approx.ftz: ~2^-22 relative error, subnormal results flushed)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

enum Warp { kWarpTma = 0, kWarpMma = 1, kWarpPrep0 = 2, kWarpSoftmax0 = 4 };

// Launch modes.  kModeFull: the whole of K in one cluster (K <= 1024).
// Large K runs as groups of kGroupChunks chunks (512 components) in two passes:
// kModeRowStat writes each row's (max, scaled sum) over the group's
// components, tc_lse_combine_kernel folds the groups into the row's
// log-sum-exp, and kModeExtLse turns that into responsibilities and the
// M-step statistics of the group's components.
//
// Inference (no M-step): kModeArgmax writes each row's (max logit, first
// component) over the group (TcArgs::row_out chooses rowstat or the label),
// kModeProba writes the responsibilities 2^(l - lse) of the group's
// components as fp32 rows of K, from the log-sum-exp of a row-statistics pass.
enum Mode { kModeFull = 0, kModeRowStat = 1, kModeExtLse = 2, kModeArgmax = 3, kModeProba = 4 };

// Weight images of both covariance types (built by tc_pack_kernel; the
// diagonal kernel em_tc_diag.cu reads the diag ones), and the shared-memory
// carve-up of em_tc_kernel (spherical), in byte offsets from a 1024-aligned
// base: weights (a_j) | stages {X, aux} x2 | R (two 64-component MN groups) |
// constants | q | row-half slots | exchange slots | barriers.
template <int COV, int DB>
struct Cfg {
  static constexpr int D = 64 * DB;
  static constexpr bool kDiag = (COV == GMMXX_DIAG);
  // weight blocks: a_j (x coefficient), for diag also v_j (x^2 coefficient)
  static constexpr int kParamBlocks = kDiag ? 2 * kNS * DB : kNS * DB;
  static constexpr int kParams = 0;
  __host__ __device__ static constexpr int a_blk(int j, int db) { return kParams + (j * DB + db) * kBlock; }
  __host__ __device__ static constexpr int v_blk(int j, int db) { return kParams + ((kNS + j) * DB + db) * kBlock; }
  // em_tc_kernel (spherical)
  static constexpr int kMaxCluster = 8;  // cluster ranks (128 components each)
  static constexpr int kStage0 = kParams + kParamBlocks * kBlock;
  static constexpr int kStageBytes = DB * kBlock + kAuxBytes;
  static constexpr int kR = kStage0 + 2 * kStageBytes;
  static constexpr int kConsts = kR + 2 * kBlock;  // mpm[128], h[128], c2[128]
  static constexpr int kQ = kConsts + 3 * 128 * 4; // q[2][128]
  static constexpr int kHalfX = kQ + 2 * 128 * 4;  // [tile parity][half][row] float2
  static constexpr int kXch = kHalfX + 2 * 2 * 128 * 8;
  __host__ __device__ static constexpr int xch_bytes(int C) { return 2 * C * 128 * 8; }
  __host__ __device__ static constexpr int bars(int C) { return kXch + xch_bytes(C); }
  // barriers (< 192 B) and the epilogue's 4-double reduction slot share the last 256 B
  __host__ __device__ static constexpr int red(int C) { return bars(C) + 192; }
  __host__ __device__ static constexpr int total(int C) { return bars(C) + 256; }
  // feature blocks of stage s (byte offsets)
  __host__ __device__ static constexpr int x_blk(int s, int db) { return kStage0 + s * kStageBytes + db * kBlock; }
  __host__ __device__ static constexpr int aux(int s) { return kStage0 + s * kStageBytes + DB * kBlock; }
  // M-step accumulator columns: [x (D) | aux (16)]
  static constexpr int kAuxCol = D;
  static constexpr int kFdm = kAuxCol + 16;
};

struct Bars {  // lives in dynamic shared memory; see Cfg::bars / Cfg::red
  uint64_t params;
  uint64_t xfull[2];   // TMA: X tile landed
  uint64_t fmain[2];   // prep: |x|^2 (aux operand and q) ready
  uint64_t fempty[2];  // MMA: stage free for the next TMA
  uint64_t sfull[2];   // MMA: S tile complete
  uint64_t sfree[2];   // softmax: S tile consumed
  uint64_t rfull;      // softmax: R part written
  uint64_t rfree;      // MMA: R part consumed
  uint64_t xch[2];     // cluster exchange of (row max, row sum)
  uint64_t hx[2];      // softmax: both component halves of the row wrote (max, sum)
  uint64_t mdone;      // MMA: all MMAs issued and complete
  uint32_t tmem_base;
  int abort;
};

static_assert(sizeof(Bars) <= 192, "barrier block overlaps the reduction slot");

__device__ __forceinline__ void set_abort(Bars* b, int* status) {
  b->abort = 1;
  atomicOr(status, 1 << GMMXX_ERR_TIMEOUT);
}

template <int COV, int DB, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    em_tc_kernel(const __grid_constant__ CUtensorMap tmap, TcArgs a) {
  // diagonal covariance has its own kernel (em_tc_diag.cu); Cfg<DIAG> only
  // describes the weight images that tc_pack_kernel builds for it
  static_assert(COV == GMMXX_SPHERICAL, "em_tc_kernel is the spherical kernel");
  // passes without an M-step: the stage is free after the E-step and the softmax
  constexpr bool kEOnly = MODE == kModeRowStat || MODE == kModeArgmax || MODE == kModeProba;
  using C = Cfg<COV, DB>;
  // The dynamic block is the kernel's only shared memory, declared 1024-byte
  // aligned (the 128-byte swizzle atoms need it).  All shared pointers derive
  // from it by constant offsets, so every access compiles to a shared-space
  // instruction rather than a generic one.
  extern __shared__ __align__(1024) char smem_raw[];
  char* sm = smem_raw;
  if ((smem_u32(smem_raw) & 1023u) != 0) {  // uniform across the grid: no CTA proceeds
    if (threadIdx.x == 0) atomicOr(a.status, 1 << GMMXX_ERR_UNSUPPORTED);
    return;
  }
  const int nclus = a.cluster_size;
  Bars* bars = reinterpret_cast<Bars*>(sm + C::bars(nclus));
  float* c_mpm = reinterpret_cast<float*>(sm + C::kConsts);
  float* c_h = c_mpm + 128;
  float* c_c2 = c_h + 128;
  float* qbuf = reinterpret_cast<float*>(sm + C::kQ);
  float2* xch = reinterpret_cast<float2*>(sm + C::kXch);
  volatile int* abort = &bars->abort;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const uint32_t cid = cluster_id_x();
  const uint32_t ncl = ncluster_x();
  const int64_t ntiles = (a.N + kBM - 1) / kBM;
  const int T = (int)((ntiles > (int64_t)cid) ? (ntiles - 1 - cid) / ncl + 1 : 0);

  if (tid == 0) {
    mbar_init(&bars->params, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->xfull[i], 1);
      mbar_init(&bars->fmain[i], 2);
      mbar_init(&bars->fempty[i], 1);
      mbar_init(&bars->sfull[i], 1);
      mbar_init(&bars->sfree[i], 8);
      mbar_init(&bars->xch[i], 1);
      mbar_init(&bars->hx[i], 8);
    }
    mbar_init(&bars->rfull, 8);
    mbar_init(&bars->rfree, 1);
    mbar_init(&bars->mdone, 1);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == kWarpMma) tmem_alloc(&bars->tmem_base, kTmemCols);
  // constants of this CTA's component chunk; constant rows of the aux operand(s)
  const int chunk = a.chunk0 + (int)rank;  // this CTA's 128-component chunk of K
  for (int i = tid; i < 3 * 128; i += kThreads) c_mpm[i] = a.consts[(int64_t)chunk * 3 * 128 + i];
  for (int s = 0; s < 2; ++s) {
    char* aux = sm + C::aux(s);
    for (int i = tid; i < 16 * 128; i += kThreads) {
      const int n = i >> 7, r = i & 127;
      *reinterpret_cast<__nv_bfloat16*>(aux + (r >> 6) * 2048 + sw128(n, r & 63)) =
          __float2bfloat16(n == 0 ? 1.f : 0.f);
    }
  }
  fence_proxy_async();
  tmem_fence_before();
  __syncthreads();
  cluster_sync();  // peers' barriers initialised before any DSMEM traffic
  tmem_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == kWarpTma) {
    // ---------------- producer: component weights once, then X tiles ----------------
    if (lane == 0) {
      prefetch_tmap(&tmap);
      mbar_expect_tx(&bars->params, C::kParamBlocks * kBlock);
      const char* src = a.params + (int64_t)chunk * C::kParamBlocks * kBlock;
      for (int i = 0; i < C::kParamBlocks; ++i)
        bulk_load(sm + C::kParams + i * kBlock, src + (int64_t)i * kBlock, kBlock, &bars->params);
      for (int t = 0; t < T; ++t) {
        const int s = t & 1;
        if (t >= 2 && !mbar_wait(&bars->fempty[s], ((t >> 1) - 1) & 1, abort)) { set_abort(bars, a.status); break; }
        // without an M-step the stage is free once the E-step read it; the
        // softmax must also have read the stage's |x|^2 entries (qbuf)
        if (kEOnly && t >= 2 && !mbar_wait(&bars->sfree[s], ((t >> 1) - 1) & 1, abort)) {
          set_abort(bars, a.status);
          break;
        }
        const int row0 = (int)((cid + (int64_t)t * ncl) * kBM);
        mbar_expect_tx(&bars->xfull[s], DB * kBlock);
        for (int db = 0; db < DB; ++db) tma_load_2d(sm + C::x_blk(s, db), &tmap, db * 64, row0, &bars->xfull[s]);
      }
    }
  } else if (warp == kWarpMma) {
    // ---------------- MMA issuer (one thread) ----------------
    if (lane == 0) {
      const uint32_t id_e = idesc_bf16(128, kKC, 0, 0);
      // the DB column blocks of x in one instruction
      const uint32_t id_m2 = idesc_bf16(128, 64 * DB, 1, 1);
      const uint32_t id_aux = idesc_bf16(128, 16, 1, 0);
      const uint32_t base = smem_u32(sm);
      const uint32_t r_base = base + C::kR;
      bool ok = mbar_wait(&bars->params, 0, abort);
      tmem_fence_after();
      // one K=64 feature block times one K=64 weight block (4 MMAs of K=16)
      auto block_mma = [&](uint32_t d, uint32_t fa, uint32_t wb, uint32_t& acc) {
        const uint64_t da = desc_kmajor(fa), dw = desc_kmajor(wb);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // +32 B along K per instruction
          mma_bf16(d, da + 2 * kk, dw + 2 * kk, id_e, acc);
          acc = 1;
        }
      };
      // E-step: x . a_j into S[t & 1]
      auto issue_e_main = [&](int t) -> bool {
        const int s = t & 1;
        if (!mbar_wait(&bars->fmain[s], (t >> 1) & 1, abort)) return false;
        if (t >= 2 && !mbar_wait(&bars->sfree[s], ((t >> 1) - 1) & 1, abort)) return false;
        tmem_fence_after();
        const uint32_t d = tmem + (uint32_t)(s * kKC);
        uint32_t acc = 0;
        for (int db = 0; db < DB; ++db) {
#pragma unroll
          for (int j = 0; j < kNS; ++j) block_mma(d, base + C::x_blk(s, db), base + C::a_blk(j, db), acc);
        }
        mma_commit(&bars->sfull[s]);
        return true;
      };
      // M-step of tile t with R part PART (0 = high bf16 terms, 1 = residual).
      // The DB column blocks of x are adjacent 16 KB blocks of the stage, so
      // one MN-major instruction covers them; PART is a template argument so
      // that the issue sequence carries no branches between instructions.
      auto issue_m = [&](int t, auto part_tag) -> bool {
        constexpr int part = decltype(part_tag)::value;
        const int s = t & 1;
        const int use = 2 * t + part;
        if (!mbar_wait(&bars->rfull, use & 1, abort)) return false;
        tmem_fence_after();
        const uint32_t acc0 = (t == 0 && part == 0) ? 0u : 1u;
        // descriptors at row 0; each 16-row step adds 2048 B (MN-major) or
        // 32 B / 2048 B per 4 steps (K-major aux)
        const uint64_t r0 = desc_mnmajor(r_base, kBlock);
        const uint64_t x0 = desc_mnmajor(base + C::x_blk(s, 0), kBlock);
        const uint64_t aux0 = desc_kmajor(base + C::aux(s));
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {  // 16 rows per instruction
          const uint64_t step = (uint64_t)(ks * 128);  // 2048 B >> 4
          const uint64_t ra = r0 + step;
          const uint32_t acc = ks == 0 ? acc0 : 1u;
          mma_bf16(tmem + kDmCol, ra, x0 + step, id_m2, acc);  // x
          mma_bf16(tmem + kDmCol + C::kAuxCol, ra, aux0 + (uint64_t)((ks >> 2) * 128 + (ks & 3) * 2), id_aux, acc);
        }
        mma_commit(&bars->rfree);
        if constexpr (part == 1) mma_commit(&bars->fempty[s]);
        return true;
      };
      using Hi = std::integral_constant<int, 0>;
      using Lo = std::integral_constant<int, 1>;
      if constexpr (kEOnly) {
        for (int t = 0; ok && t < T; ++t) {
          if (!issue_e_main(t)) { ok = false; break; }
          mma_commit(&bars->fempty[t & 1]);  // no M-step: the stage is free after E(t)
        }
      } else {
        if (ok && T > 0) ok = issue_e_main(0);
        for (int t = 0; ok && t < T; ++t) {
          if (t + 1 < T && !issue_e_main(t + 1)) { ok = false; break; }
          if (!issue_m(t, Hi{})) { ok = false; break; }
          if (!issue_m(t, Lo{})) { ok = false; break; }
        }
      }
      if (!ok) set_abort(bars, a.status);
      mma_commit(&bars->mdone);
    }
  } else if (warp < kWarpSoftmax0) {
    // ---------------- feature prep (2 warps) ----------------
    const int ptid = tid - kWarpPrep0 * 32;  // 0..63
    for (int t = 0; t < T; ++t) {
      const int s = t & 1;
      if (!mbar_wait_warp(&bars->xfull[s], (t >> 1) & 1, abort)) { set_abort(bars, a.status); break; }
      // |x|^2 per row (two threads per row), three bf16 terms q_0 + q_1 + q_2
      // (24 significant bits) into the aux operand
      char* aux = sm + C::aux(s);
      const int r = ptid >> 1, hf = ptid & 1;
      for (int rr = r; rr < kBM; rr += 32) {
        float acc = 0.f;
        for (int db = 0; db < DB; ++db)
          for (int c = hf * 4; c < hf * 4 + 4; ++c) {
            const uint4 v = *reinterpret_cast<const uint4*>(sm + C::x_blk(s, db) + rr * 128 + c * 16);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float x0 = bf16lo_to_f32(w[i]), x1 = bf16hi_to_f32(w[i]);
              acc = fmaf(x0, x0, acc);
              acc = fmaf(x1, x1, acc);
            }
          }
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        if (hf == 0) {
          qbuf[s * 128 + rr] = acc;
          char* blk = aux + (rr >> 6) * 2048;
          float rem = acc;
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            const __nv_bfloat16 qj = __float2bfloat16(rem);
            *reinterpret_cast<__nv_bfloat16*>(blk + sw128(1 + j, rr & 63)) = qj;
            rem -= __bfloat162float(qj);
          }
        }
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->fmain[s]);
    }
  } else {
    // ---------------- softmax: 8 warps, two per TMEM lane quarter ----------------
    // warp w handles rows 32*(w%4) .. +31 (its TMEM lane quarter) and the
    // component half hf = (w-4)/4, i.e. 64 logits per thread.
    const int q4 = warp & 3;
    const int hf = (warp - kWarpSoftmax0) >> 2;
    const int row = q4 * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q4 * 32) << 16;
    const int k0 = hf * kHalf;  // first component of this half
    double ll_acc = 0.0;
    float p[kHalf];
    float2* halfx = reinterpret_cast<float2*>(sm + C::kHalfX);  // [half][row]
    const uint32_t xch_mine = smem_u32(&xch[(int)rank * 128 + row]);  // slot 0 entry of (this rank, row)
    const uint32_t slot_stride = (uint32_t)(nclus * 128 * 8);
    const float4* cm4 = reinterpret_cast<const float4*>(c_mpm + k0);
    const float4* ch4 = reinterpret_cast<const float4*>(c_h + k0);
    const float4* cc4 = reinterpret_cast<const float4*>(c_c2 + k0);
    // passes from an external log-sum-exp: this row's value for the next tile
    // is loaded one tile ahead, so its latency hides behind the current tile
    constexpr bool kExt = MODE == kModeExtLse || MODE == kModeProba;
    auto ext_lse = [&](int u) -> float {
      const int64_t r = (cid + (int64_t)u * ncl) * kBM + row;
      return (u < T && r < a.N) ? __ldg(a.lse_in + r) : 0.f;
    };
    float lse_next = kExt ? ext_lse(0) : 0.f;
    for (int t = 0; t < T; ++t) {
      const int s = t & 1;
      const int64_t grow = (cid + (int64_t)t * ncl) * kBM + row;
      const bool valid = grow < a.N;
      const float lse_t = lse_next;
      if constexpr (kExt) lse_next = ext_lse(t + 1);
      if (!mbar_wait_warp(&bars->sfull[s], (t >> 1) & 1, abort)) { set_abort(bars, a.status); break; }
      tmem_fence_after();
      const uint32_t sc = tmem + lane_addr + (uint32_t)(s * kKC + k0);
      tmem_ld32(sc, p);
      tmem_ld32(sc + 32, p + 32);
      // |x|^2 of this row (signalled by the prep warps before S was issued)
      if (!mbar_wait_warp(&bars->fmain[s], (t >> 1) & 1, abort)) { set_abort(bars, a.status); break; }
      const float qn = qbuf[s * 128 + row];
      tmem_wait_ld();
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->sfree[s]);  // S(t) and this row's |x|^2 consumed
      // logits (log2 units) c2 - h max(|x|^2 + S + mpm, 0) and this half's row
      // max; four independent chains
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int k4 = 0; k4 < kHalf / 4; ++k4) {
        const float4 vm = cm4[k4], vc = cc4[k4];
        const float4 vh = ch4[k4];
        const float mm[4] = {vm.x, vm.y, vm.z, vm.w}, hh[4] = {vh.x, vh.y, vh.z, vh.w},
                    cc[4] = {vc.x, vc.y, vc.z, vc.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int k = 4 * k4 + j;
          const float dist = fmaxf(p[k] + (mm[j] + qn), 0.f);
          const float l = fmaf(-hh[j], dist, cc[j]);
          p[k] = l;
          mx[j] = fmaxf(mx[j], l);
        }
      }
      const float m = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      if constexpr (MODE == kModeArgmax) {
        // this half's largest logit and its first component, then the row's
        // over both halves and the cluster; halves and ranks are in increasing
        // component order and only a strictly larger logit replaces the best
        const int comp0 = chunk * kKC + k0;
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int k = 0; k < kHalf; ++k)
          if (p[k] > bv) { bv = p[k]; bi = comp0 + k; }
        float2* hxs = halfx + s * 2 * 128;
        hxs[hf * 128 + row] = make_float2(bv, __int_as_float(bi));
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->hx[s]);
        if (!mbar_wait_warp(&bars->hx[s], (t >> 1) & 1, abort)) { set_abort(bars, a.status); break; }
        float2 best = hxs[row];
        const float2 h1 = hxs[128 + row];
        if (h1.x > best.x) best = h1;
        if (hf == 0) {
          if (tid == kWarpSoftmax0 * 32) mbar_expect_tx(&bars->xch[s], (uint32_t)(nclus * 128 * 8));
#pragma unroll
          for (int q = 0; q < C::kMaxCluster; ++q)
            if (q < nclus)
              st_async_f2(map_shared(xch_mine + s * slot_stride, q), best.x, best.y,
                          map_shared(smem_u32(&bars->xch[s]), q));
        }
        if (!mbar_wait_warp(&bars->xch[s], (t >> 1) & 1, abort)) { set_abort(bars, a.status); break; }
        float2 g = xch[(s * nclus) * 128 + row];
#pragma unroll
        for (int q = 1; q < C::kMaxCluster; ++q)
          if (q < nclus) {
            const float2 e = xch[(s * nclus + q) * 128 + row];
            if (e.x > g.x) g = e;
          }
        if (valid && rank == 0 && hf == 0) {
          if (a.row_out == 3) a.out_i[grow] = (int64_t)__float_as_int(g.y);
          else a.rowstat[grow] = g;
        }
        if (*abort) break;
        continue;
      }
      if constexpr (MODE == kModeProba) {
        // responsibilities of this half's components from the row's
        // log-sum-exp over all K (log2 units), written as fp32 rows of K
        if (valid) {
          const float lse = lse_t;
          const int comp0 = chunk * kKC + k0;
          float* orow = a.out_f + grow * (int64_t)a.K + comp0;
          if (a.out_vec && comp0 + kHalf <= a.K) {
#pragma unroll
            for (int c = 0; c < kHalf / 4; ++c)
              reinterpret_cast<float4*>(orow)[c] =
                  make_float4(ex2_approx(p[4 * c] - lse), ex2_approx(p[4 * c + 1] - lse),
                              ex2_approx(p[4 * c + 2] - lse), ex2_approx(p[4 * c + 3] - lse));
          } else {
#pragma unroll
            for (int k = 0; k < kHalf; ++k)
              if (comp0 + k < a.K) orow[k] = ex2_approx(p[k] - lse);
          }
        }
        if (*abort) break;
        continue;
      }
      float M = 0.f, S = 1.f, f = 0.f;
      if constexpr (MODE == kModeExtLse) {
        // responsibilities from the row's log-sum-exp over all K (log2 units)
        const float lse = lse_t;
#pragma unroll
        for (int k = 0; k < kHalf; ++k) p[k] = ex2_approx(p[k] - lse);
        f = valid ? 1.f : 0.f;
      } else {
      // a half made only of padding components has m = -inf: its p must be 0
      const float mref = (m == -INFINITY) ? 0.f : m;
      float sm4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < kHalf; ++k) {
        p[k] = ex2_approx(p[k] - mref);
        sm4[k & 3] += p[k];
      }
      const float sum = (sm4[0] + sm4[1]) + (sm4[2] + sm4[3]);
      // combine the two halves of the row, one buffer per tile parity: a half
      // writes its entry for tile t+2 only after the hx barrier of tile t+1,
      // which the other half passes after reading this tile's entry.
      float2* hxs = halfx + s * 2 * 128;
      hxs[hf * 128 + row] = make_float2(m, sum);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->hx[s]);
      if (!mbar_wait_warp(&bars->hx[s], (t >> 1) & 1, abort)) { set_abort(bars, a.status); break; }
      const float2 o = hxs[(hf ^ 1) * 128 + row];
      const float mc = fmaxf(m, o.x);
      const float sc2 = sum * exp2f(m - mc) + o.y * exp2f(o.x - mc);
      // exchange (max, sum) of this CTA's components with the cluster (half 0 sends)
      if (hf == 0) {
        if (tid == kWarpSoftmax0 * 32) mbar_expect_tx(&bars->xch[s], (uint32_t)(nclus * 128 * 8));
#pragma unroll
        for (int q = 0; q < C::kMaxCluster; ++q)
          if (q < nclus)
            st_async_f2(map_shared(xch_mine + s * slot_stride, q), mc, sc2, map_shared(smem_u32(&bars->xch[s]), q));
      }
      if (!mbar_wait_warp(&bars->xch[s], (t >> 1) & 1, abort)) { set_abort(bars, a.status); break; }
      // all ranks' (max, sum) of this row: loads issued together, then combined
      float2 e[C::kMaxCluster];
#pragma unroll
      for (int q = 0; q < C::kMaxCluster; ++q)
        e[q] = q < nclus ? xch[(s * nclus + q) * 128 + row] : make_float2(-INFINITY, 0.f);
      M = e[0].x;
#pragma unroll
      for (int q = 1; q < C::kMaxCluster; ++q) M = fmaxf(M, e[q].x);
      S = 0.f;
#pragma unroll
      for (int q = 0; q < C::kMaxCluster; ++q)
        if (q < nclus) S += e[q].y * exp2f(e[q].x - M);
      if constexpr (MODE == kModeRowStat) {
        // the row's (max, scaled sum) over this group's components; no R, no M-step
        if (valid && rank == 0 && hf == 0) {
          if (a.row_out == 0) a.rowstat[grow] = make_float2(M, S);
          else a.out_f[grow] = a.row_out == 1 ? (M + log2f(S)) * kLn2 : M + log2f(S);
        }
        if (*abort) break;
        continue;
      }
      f = valid ? exp2f(m - M) / S : 0.f;
      }
      // responsibilities -> R in two passes (bf16 high part, then the residual);
      // this half's 64 components are exactly R's MN group hf.  Both parts are
      // formed now; the residual words wait in registers for the second pass.
      char* rg = sm + C::kR + hf * kBlock;
      if (t >= 1 && !mbar_wait_warp(&bars->rfree, 1u, abort)) { set_abort(bars, a.status); break; }  // M_lo(t-1)
      uint32_t lo[kHalf / 2];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int kk = c * 8 + 2 * i;
          const float r0 = p[kk] * f, r1 = p[kk + 1] * f;
          w[i] = pack_bf16(r0, r1);
          lo[4 * c + i] = pack_bf16(r0 - bf16lo_to_f32(w[i]), r1 - bf16hi_to_f32(w[i]));
        }
        *reinterpret_cast<uint4*>(rg + sw128((uint32_t)row, (uint32_t)(c * 8))) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->rfull);
      if (!mbar_wait_warp(&bars->rfree, 0u, abort)) { set_abort(bars, a.status); break; }  // M_hi(t)
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(rg + sw128((uint32_t)row, (uint32_t)(c * 8))) =
            make_uint4(lo[4 * c], lo[4 * c + 1], lo[4 * c + 2], lo[4 * c + 3]);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->rfull);
      // log-likelihood of the row, off the R critical path (rank 0 holds it)
      if (MODE == kModeFull && valid && rank == 0 && hf == 0) ll_acc += (double)((M + log2f(S)) * kLn2);
      if (*abort) break;
    }
    // ---------------- epilogue: statistics partials (half-0 warps) ----------------
    // drain: the MMA thread always commits `mdone` (also after an abort), so
    // wait for it without the abort shortcut before touching TMEM again
    if (hf == 0) {
      if (!mbar_wait_warp(&bars->mdone, 0, nullptr, 4000000000ull)) set_abort(bars, a.status);
      tmem_fence_after();
    }
    if (hf == 0 && !kEOnly) {
      const int comp = (int)rank * kKC + row;  // this thread's TMEM lane = component
      float* out = a.part + ((int64_t)cid * a.Kp + comp) * a.F;
      for (int c0 = 0; c0 < C::kFdm; c0 += 16) {
        float v[32];
        tmem_ld32(tmem + lane_addr + kDmCol + c0, v);  // 32 columns; 16 used per step
        tmem_wait_ld();
        for (int j = 0; j < 16 && c0 + j < C::kFdm; ++j) {
          const int col = c0 + j;
          if (col < C::D) out[1 + col] = v[j];                                  // sum r x
          else if (col == C::kAuxCol) out[0] = v[j];                            // n_k
          else if (col == C::kAuxCol + 1) out[1 + C::D] = v[j] + v[j + 1] + v[j + 2];  // sum r |x|^2
        }
      }
      tmem_fence_before();
      // log-likelihood partial of this cluster (rank 0 holds it)
      double* red = reinterpret_cast<double*>(sm + C::red(nclus));
      double v = ll_acc;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[q4] = v;
      asm volatile("bar.sync 2, 128;" ::: "memory");
      if (MODE == kModeFull && tid == kWarpSoftmax0 * 32 && rank == 0)
        a.part_ll[cid] = red[0] + red[1] + red[2] + red[3];
    }
  }
  __syncthreads();
  if (warp == kWarpMma) {
    tmem_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  cluster_sync();  // no CTA exits while a peer may still write into its shared memory
}

// Pack the per-iteration component table into this kernel's shared-memory
// images: split-bf16 weight blocks (128-byte swizzle) + epilogue constants.
template <int COV, int DB>
__global__ void tc_pack_kernel(int K, int64_t Kp_table, const float* wt, const CompConst* cc, char* params,
                               float* consts) {
  using C = Cfg<COV, DB>;
  const int k = blockIdx.x;  // padded component index
  const int chunk = k / kKC, kl = k % kKC;
  char* img = params + (int64_t)chunk * C::kParamBlocks * kBlock;
  const bool live = k < K;
  for (int d = threadIdx.x; d < C::D; d += blockDim.x) {
    const int db = d >> 6, c = d & 63;
    // x coefficient: -2 mu (spherical) | -2 mu / var (diag, table rows D..2D)
    float ra = live ? wt[(int64_t)(C::kDiag ? C::D + d : d) * Kp_table + k] : 0.f;
    // x^2 coefficient (diag): 1 / var
    float rv = (live && C::kDiag) ? wt[(int64_t)d * Kp_table + k] : 0.f;
#pragma unroll
    for (int j = 0; j < kNS; ++j) {  // w = w_0 + w_1 + w_2, each bf16
      const __nv_bfloat16 ha = __float2bfloat16(ra);
      *reinterpret_cast<__nv_bfloat16*>(img + C::a_blk(j, db) + sw128(kl, c)) = ha;
      ra -= __bfloat162float(ha);
      if (C::kDiag) {
        const __nv_bfloat16 hv = __float2bfloat16(rv);
        *reinterpret_cast<__nv_bfloat16*>(img + C::v_blk(j, db) + sw128(kl, c)) = hv;
        rv -= __bfloat162float(hv);
      }
    }
  }
  if (threadIdx.x == 0) {
    float* cs = consts + (int64_t)chunk * 3 * 128;
    if (live) {
      const CompConst q = cc[k];
      cs[kl] = q.mpm;
      cs[128 + kl] = 0.5f * kLog2e * q.s;
      cs[256 + kl] = kLog2e * (q.lw - 0.5f * q.ln);
    } else {  // padding component: logit -inf, no contribution anywhere
      cs[kl] = 0.f;
      cs[128 + kl] = 0.f;
      cs[256 + kl] = -INFINITY;
    }
  }
}

// Tied covariance (em_tc_diag.cu, tied mode): per chunk three term blocks of
// [192 rows][64 features] bf16 with 128-byte swizzle -- rows 0-127 the
// chunk's components' x coefficient -2 (P mu)_d, rows 128 + i row
// 16 p0 + i of L^-1 for the pieces [p0, p1) of y = L^-1 x that this chunk's
// cluster rank computes (the 4 pieces of 16 rows spread over the C ranks),
// each value split into three bf16 terms; then the epilogue constants.
__global__ void tc_pack_tied_kernel(int K, int64_t Kp_table, int csize, const float* wt, const float* linv,
                                    const CompConst* cc, char* params, float* consts) {
  const int row = blockIdx.x % 192, chunk = blockIdx.x / 192;
  char* img = params + (int64_t)chunk * 3 * kTiedTermBytes;
  const int p0 = 4 * chunk / csize, p1 = 4 * (chunk + 1) / csize;
  const int k = chunk * kKC + row;
  for (int d = threadIdx.x; d < 64; d += blockDim.x) {
    float v = 0.f;
    if (row < kKC) {
      if (k < K) v = wt[(int64_t)d * Kp_table + k];
    } else if (row - kKC < 16 * (p1 - p0)) {
      v = linv[(16 * p0 + (row - kKC)) * 64 + d];
    }
#pragma unroll
    for (int j = 0; j < kNS; ++j) {
      const __nv_bfloat16 h = __float2bfloat16(v);
      *reinterpret_cast<__nv_bfloat16*>(img + j * kTiedTermBytes + sw128(row, d)) = h;
      v -= __bfloat162float(h);
    }
  }
  if (threadIdx.x == 0 && row < kKC) {
    float* cs = consts + (int64_t)chunk * 3 * 128;
    if (k < K) {
      const CompConst q = cc[k];
      cs[row] = q.mpm;
      cs[128 + row] = 0.5f * kLog2e * q.s;
      cs[256 + row] = kLog2e * (q.lw - 0.5f * q.ln);
    } else {
      cs[row] = 0.f;
      cs[128 + row] = 0.f;
      cs[256 + row] = -INFINITY;
    }
  }
}

// stats[k][f] += sum over clusters of part[cl][k][f] (fixed order), ll += sum part_ll
__global__ void tc_reduce_kernel(const float* part, const double* part_ll, int ncl, int K, int64_t Kp, int F,
                                 float* stats, double* ll, int n_ll) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < (int64_t)K * F) {
    const int64_t k = i / F, f = i - k * F;
    float s = 0.f;
    for (int c = 0; c < ncl; ++c) s += part[((int64_t)c * Kp + k) * F + f];
    stats[i] += s;
  }
  if (i == 0 && ll != nullptr) {
    double s = 0.0;
    for (int c = 0; c < n_ll; ++c) s += part_ll[c];
    *ll += s;
  }
}

// Grouped large-K path: each row's log-sum-exp over all groups (log2 units)
// from the per-group (max, scaled sum), and one fixed-order log-likelihood
// partial per block.
__global__ void tc_lse_combine_kernel(const float2* rowstat, int groups, int64_t N, float* lse, double* ll_part,
                                      float scale = 1.f) {
  double acc = 0.0;
  for (int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; n < N; n += (int64_t)gridDim.x * blockDim.x) {
    // the groups' partials in blocks of 8 independent loads (the second
    // sweep re-reads them from cache), summed in group order
    float M = -INFINITY;
    int g = 0;
    for (; g + 8 <= groups; g += 8) {
      float x[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = __ldg(&rowstat[(int64_t)(g + i) * N + n].x);
#pragma unroll
      for (int i = 0; i < 8; ++i) M = fmaxf(M, x[i]);
    }
    for (; g < groups; ++g) M = fmaxf(M, __ldg(&rowstat[(int64_t)g * N + n].x));
    float S = 0.f;
    g = 0;
    for (; g + 8 <= groups; g += 8) {
      float2 e[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) e[i] = __ldg(&rowstat[(int64_t)(g + i) * N + n]);
#pragma unroll
      for (int i = 0; i < 8; ++i) S += e[i].y * exp2f(e[i].x - M);
    }
    for (; g < groups; ++g) {
      const float2 e = __ldg(&rowstat[(int64_t)g * N + n]);
      S += e.y * exp2f(e.x - M);
    }
    const float l2 = M + log2f(S);
    lse[n] = scale == 1.f ? l2 : l2 * scale;
    acc += (double)l2 * (double)kLn2;
  }
  if (ll_part == nullptr) return;
  __shared__ double red[32];
  acc = warp_sum_d(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
    ll_part[blockIdx.x] = s;
  }
}

// blocks of the per-row combine kernels: four per SM (their log-likelihood
// partials, one per block, fit the kTcMaxClusters * kMaxClusterSph slots)
constexpr int kCombineBlocks = 4 * 148;
static_assert(kCombineBlocks <= kTcMaxClusters * kMaxClusterSph, "log-likelihood partial slots");

// Grouped inference: each row's label from the per-group (max logit, first
// component), groups in increasing component order, strictly larger wins.
__global__ void tc_argmax_combine_kernel(const float2* rowstat, int groups, int64_t N, int64_t* labels) {
  for (int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; n < N; n += (int64_t)gridDim.x * blockDim.x) {
    float2 best = rowstat[n];
    for (int g = 1; g < groups; ++g) {
      const float2 e = rowstat[(int64_t)g * N + n];
      if (e.x > best.x) best = e;
    }
    labels[n] = (int64_t)__float_as_int(best.y);
  }
}

__global__ void tc_ll_sum_kernel(const double* ll_part, int n, double* ll) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += ll_part[i];
    *ll += s;
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

// GMMXX_B200_SPH_KERNEL=legacy keeps spherical D = 128 EM on em_tc_kernel
// (the A/B switch of the two tensor-core layouts); anything else uses the
// diag-kernel layout where it applies.
bool sph128_enabled() {
  const char* e = getenv("GMMXX_B200_SPH_KERNEL");
  return !(e != nullptr && strcmp(e, "legacy") == 0);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int launch_tc_pack(int cov, int db, const TcLaunch& L, cudaStream_t st) {
  const unsigned grid = (unsigned)(L.nchunks * kKC);
  if (cov == GMMXX_TIED && db == 1) {
    if (L.linv == nullptr) return set_error(GMMXX_ERR_WORKSPACE, "tied tensor-core pack: no L^-1 in the workspace");
    tc_pack_tied_kernel<<<(unsigned)(L.nchunks * 192), 64, 0, st>>>(L.K, L.Kp_table, L.cluster_size, L.wt, L.linv,
                                                                    L.cc, L.params, L.consts);
  } else if (cov == GMMXX_DIAG && db == 1)
    tc_pack_kernel<GMMXX_DIAG, 1><<<grid, 64, 0, st>>>(L.K, L.Kp_table, L.wt, L.cc, L.params, L.consts);
  else if (cov == GMMXX_SPHERICAL && db == 1)
    tc_pack_kernel<GMMXX_SPHERICAL, 1><<<grid, 64, 0, st>>>(L.K, L.Kp_table, L.wt, L.cc, L.params, L.consts);
  else if (cov == GMMXX_SPHERICAL && db == 2)
    tc_pack_kernel<GMMXX_SPHERICAL, 2><<<grid, 64, 0, st>>>(L.K, L.Kp_table, L.wt, L.cc, L.params, L.consts);
  else
    return set_error(GMMXX_ERR_UNSUPPORTED, "no weight image layout for this shape");
  return check_launch("tc_pack_kernel");
}

int make_x_tensor_map(const TcLaunch& L, CUtensorMap* tmap, bool fp32) {
  // X (N rows x D), 128-row boxes of 128 bytes per row (64 bf16 or 32 fp32
  // columns), 128-byte swizzle
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return set_error(GMMXX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t esz = fp32 ? 4 : 2;
  cuuint64_t dims[2] = {(cuuint64_t)L.D, (cuuint64_t)L.N};
  cuuint64_t strides[1] = {(cuuint64_t)L.D * esz};
  cuuint32_t box[2] = {(cuuint32_t)(128 / esz), (cuuint32_t)kBM};
  cuuint32_t es[2] = {1, 1};
  CUresult cr = enc(tmap, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                    const_cast<void*>(L.x), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return set_error(GMMXX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)cr);
  return GMMXX_OK;
}

int launch_tc_reduce(const TcLaunch& L, int ncl, cudaStream_t st, int n_ll) {
  const int64_t n = (int64_t)L.K * L.F;
  tc_reduce_kernel<<<(unsigned)ceil_div(std::max<int64_t>(n, 1), 256), 256, 0, st>>>(
      L.part, L.part_ll, ncl, L.K, L.Kp_part, L.F, L.stats, L.ll, n_ll < 0 ? ncl : n_ll);
  return check_launch("tc_reduce_kernel");
}

int clustered_launch(const void* kern, int threads, int smem, const TcLaunch& L, int* ncl_out) {
  const int nclus = L.cluster_size;
  {  // test hook: GMMXX_B200_TEST_NO_CLUSTER=1 answers as a device with no co-resident cluster would
    const char* e = getenv("GMMXX_B200_TEST_NO_CLUSTER");
    if (e != nullptr && strcmp(e, "1") == 0)
      return set_error(GMMXX_ERR_UNSUPPORTED, "no co-resident cluster of %d CTAs (GMMXX_B200_TEST_NO_CLUSTER)", nclus);
  }
  if (smem > 232448) return set_error(GMMXX_ERR_UNSUPPORTED, "tensor-core kernel shared memory over budget");
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return set_error(GMMXX_ERR_CUDA, "tensor-core kernel attributes: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = nclus;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3((unsigned)nclus);
  int max_clusters = 0;
  e = cudaOccupancyMaxActiveClusters(&max_clusters, kern, &cfg);
  if (e != cudaSuccess || max_clusters <= 0) {
    cudaGetLastError();
    return set_error(GMMXX_ERR_UNSUPPORTED, "no co-resident cluster of %d CTAs (%s)", nclus, cudaGetErrorString(e));
  }
  const int64_t ntiles = (L.N + kBM - 1) / kBM;
  const int ncl = (int)std::min<int64_t>(std::min<int64_t>(max_clusters, kMaxClusters), ntiles);
  *ncl_out = ncl;
  return GMMXX_OK;
}

// One clustered launch of em_tc_kernel over chunks [chunk0, chunk0 + csize).
template <int COV, int DB, int MODE>
static int launch_mode(const TcLaunch& L, int chunk0, int csize, const float* lse_in, float2* rowstat, int* ncl_out,
                       cudaStream_t st, int row_out = 0) {
  using C = Cfg<COV, DB>;
  // the dynamic block is the kernel's only shared memory: <= 227 KB per CTA
  static_assert(C::total(C::kMaxCluster) <= 232448, "shared memory budget");
  CUtensorMap tmap;
  if (int rc = make_x_tensor_map(L, &tmap)) return rc;
  auto kern = em_tc_kernel<COV, DB, MODE>;
  const int smem = C::total(csize);
  TcLaunch Lc = L;
  Lc.cluster_size = csize;
  int ncl = 0;
  if (int rc = clustered_launch((const void*)kern, kThreads, smem, Lc, &ncl)) return rc;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3((unsigned)(ncl * csize));
  TcArgs args{};
  args.N = L.N;
  args.Kp = (int64_t)csize * kKC;
  args.F = L.F;
  args.cluster_size = csize;
  args.params = L.params;
  args.consts = L.consts;
  args.part = L.part;
  args.part_ll = L.part_ll;
  args.status = L.status;
  args.chunk0 = chunk0;
  args.lse_in = lse_in;
  args.rowstat = rowstat;
  args.K = L.K;
  args.out_f = L.out_f;
  args.out_i = L.out_i;
  args.out_vec = ((reinterpret_cast<uintptr_t>(L.out_f) & 15u) == 0 && (L.K & 3) == 0) ? 1 : 0;
  args.row_out = row_out;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tmap, args);
  if (e != cudaSuccess) return set_error(GMMXX_ERR_CUDA, "em_tc_kernel launch: %s", cudaGetErrorString(e));
  *ncl_out = ncl;
  return GMMXX_OK;
}

// K <= 1024: one launch over the whole of K, then the fixed-order reduction.
template <int COV, int DB>
static int launch_t(const TcLaunch& L, cudaStream_t st) {
  if (int rc = launch_tc_pack(COV, DB, L, st)) return rc;
  int ncl = 0;
  if (int rc = launch_mode<COV, DB, kModeFull>(L, 0, L.cluster_size, nullptr, nullptr, &ncl, st)) return rc;
  return launch_tc_reduce(L, ncl, st);
}

// Spherical K > 1024: groups of kGroupChunks chunks (512 components).  Pass 1 writes
// each row's (max, sum) per group; the combine folds them into the row's
// log-sum-exp and the log-likelihood; pass 2 forms the responsibilities of
// each group's components from it and accumulates their statistics.
template <int DB>
static int launch_grouped(const TcLaunch& L, cudaStream_t st) {
  if (int rc = launch_tc_pack(GMMXX_SPHERICAL, DB, L, st)) return rc;
  const int gc = tc_group_chunks(L.K);
  const int groups = (L.nchunks + gc - 1) / gc;
  int ncl = 0;
  for (int g = 0; g < groups; ++g) {
    const int csize = std::min(gc, L.nchunks - g * gc);
    if (int rc = launch_mode<GMMXX_SPHERICAL, DB, kModeRowStat>(L, g * gc, csize, nullptr,
                                                                 L.rowstat + (int64_t)g * L.N, &ncl, st))
      return rc;
  }
  if (int rc = launch_rowstat_combine(L, groups, st)) return rc;
  for (int g = 0; g < groups; ++g) {
    const int csize = std::min(gc, L.nchunks - g * gc);
    if (int rc = launch_mode<GMMXX_SPHERICAL, DB, kModeExtLse>(L, g * gc, csize, L.lse, nullptr, &ncl, st))
      return rc;
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

// Spherical inference (TcLaunch::infer = 1 log-sum-exp, 2 labels, 3
// responsibilities) in groups of up to 8 chunks: per-row passes without an
// M-step, folded over the groups by the combine kernels.  One group writes
// its rows' results directly (the label, the natural-log log-sum-exp, or
// the log2 log-sum-exp that the responsibilities pass reads from L.lse).
template <int DB>
static int launch_sph_infer(const TcLaunch& L, cudaStream_t st) {
  if (L.infer < 1 || L.infer > 3) return set_error(GMMXX_ERR_INVALID, "tensor-core inference mode %d", L.infer);
  if ((L.infer == 2 && L.out_i == nullptr) || (L.infer != 2 && L.out_f == nullptr))
    return set_error(GMMXX_ERR_INVALID, "tensor-core inference: no output buffer");
  const int gc = tc_group_chunks(L.K);
  const int groups = (L.nchunks + gc - 1) / gc;
  if (groups > 1 && L.rowstat == nullptr) return set_error(GMMXX_ERR_WORKSPACE, "grouped pass buffers missing");
  if (L.infer == 3 && L.lse == nullptr) return set_error(GMMXX_ERR_WORKSPACE, "per-row log-sum-exp buffer missing");
  if (int rc = launch_tc_pack(GMMXX_SPHERICAL, DB, L, st)) return rc;
  auto csz = [&](int g) { return std::min(gc, L.nchunks - g * gc); };
  const int nb = kCombineBlocks;
  int ncl = 0;
  if (L.infer == 2) {  // labels
    if (groups == 1) return launch_mode<GMMXX_SPHERICAL, DB, kModeArgmax>(L, 0, csz(0), nullptr, nullptr, &ncl, st, 3);
    for (int g = 0; g < groups; ++g)
      if (int rc = launch_mode<GMMXX_SPHERICAL, DB, kModeArgmax>(L, g * gc, csz(g), nullptr,
                                                                  L.rowstat + (int64_t)g * L.N, &ncl, st))
        return rc;
    tc_argmax_combine_kernel<<<nb, 256, 0, st>>>(L.rowstat, groups, L.N, L.out_i);
    return check_launch("tc_argmax_combine_kernel");
  }
  // each row's log-sum-exp over all K: natural log into out_f (score_samples),
  // or log2 units into L.lse for the responsibilities pass
  if (groups == 1) {
    if (L.infer == 1) return launch_mode<GMMXX_SPHERICAL, DB, kModeRowStat>(L, 0, csz(0), nullptr, nullptr, &ncl, st, 1);
    TcLaunch Lq = L;
    Lq.out_f = L.lse;
    if (int rc = launch_mode<GMMXX_SPHERICAL, DB, kModeRowStat>(Lq, 0, csz(0), nullptr, nullptr, &ncl, st, 2)) return rc;
  } else {
    for (int g = 0; g < groups; ++g)
      if (int rc = launch_mode<GMMXX_SPHERICAL, DB, kModeRowStat>(L, g * gc, csz(g), nullptr,
                                                                   L.rowstat + (int64_t)g * L.N, &ncl, st))
        return rc;
    if (L.infer == 1) {
      tc_lse_combine_kernel<<<nb, 256, 0, st>>>(L.rowstat, groups, L.N, L.out_f, nullptr, kLn2);
      return check_launch("tc_lse_combine_kernel");
    }
    tc_lse_combine_kernel<<<nb, 256, 0, st>>>(L.rowstat, groups, L.N, L.lse, nullptr, 1.f);
    if (int rc = check_launch("tc_lse_combine_kernel")) return rc;
  }
  for (int g = 0; g < groups; ++g)
    if (int rc = launch_mode<GMMXX_SPHERICAL, DB, kModeProba>(L, g * gc, csz(g), L.lse, nullptr, &ncl, st))
      return rc;
  return GMMXX_OK;
}

int launch_infer_combine(const TcLaunch& L, int groups, int infer, cudaStream_t st) {
  const int nb = kCombineBlocks;
  if (infer == 2) {
    tc_argmax_combine_kernel<<<nb, 256, 0, st>>>(L.rowstat, groups, L.N, L.out_i);
    return check_launch("tc_argmax_combine_kernel");
  }
  if (infer == 1) tc_lse_combine_kernel<<<nb, 256, 0, st>>>(L.rowstat, groups, L.N, L.out_f, nullptr, kLn2);
  else tc_lse_combine_kernel<<<nb, 256, 0, st>>>(L.rowstat, groups, L.N, L.lse, nullptr, 1.f);
  return check_launch("tc_lse_combine_kernel");
}

int launch_rowstat_combine(const TcLaunch& L, int groups, cudaStream_t st) {
  const int nb = kCombineBlocks;
  tc_lse_combine_kernel<<<nb, 256, 0, st>>>(L.rowstat, groups, L.N, L.lse, L.part_ll);
  if (int rc = check_launch("tc_lse_combine_kernel")) return rc;
  tc_ll_sum_kernel<<<1, 32, 0, st>>>(L.part_ll, nb, L.ll);
  return check_launch("tc_ll_sum_kernel");
}

int launch_em_tc(int cov, const TcLaunch& L, cudaStream_t st) {
  if (cov == GMMXX_DIAG && L.D == 64 && L.cluster_size <= kMaxClusterDiag) return launch_em_tc_diag(L, st);
  if (cov == GMMXX_TIED) return launch_em_tc_tied(L, st);
  // spherical D = 128 EM and inference (K <= 512 in one pass, K > 1024 in
  // groups of 512): the diag kernel's layout; 512 < K <= 1024 takes em_tc_kernel
  if (cov == GMMXX_SPHERICAL && L.D == 128 && sph128_enabled() &&
      (L.nchunks <= kMaxClusterDiag || L.nchunks > kMaxClusterSph))
    return launch_em_tc_sph128(L, st);
  if (L.infer != 0) {
    if (cov == GMMXX_SPHERICAL && L.D == 64) return launch_sph_infer<1>(L, st);
    if (cov == GMMXX_SPHERICAL && L.D == 128) return launch_sph_infer<2>(L, st);
    return set_error(GMMXX_ERR_UNSUPPORTED, "no tensor-core inference kernel for this shape");
  }
  if (cov == GMMXX_SPHERICAL && L.nchunks > kMaxClusterSph) {
    if (L.rowstat == nullptr || L.lse == nullptr) return set_error(GMMXX_ERR_WORKSPACE, "grouped pass buffers missing");
    if (L.D == 64) return launch_grouped<1>(L, st);
    if (L.D == 128) return launch_grouped<2>(L, st);
  }
  if (cov == GMMXX_SPHERICAL && L.D == 64) return launch_t<GMMXX_SPHERICAL, 1>(L, st);
  if (cov == GMMXX_SPHERICAL && L.D == 128) return launch_t<GMMXX_SPHERICAL, 2>(L, st);
  return set_error(GMMXX_ERR_UNSUPPORTED, "no tensor-core kernel for this shape");
}

}  // namespace tc
}  // namespace gmmxx
