// em_tc_sph_ext.cu -- the second pass of the grouped spherical EM (bf16 X,
// D = 128, K > 1024): each row's responsibilities over one group's
// components from the row's log-sum-exp over all K (written by the first
// pass), and those components' M-step statistics.
//
// The pass has no row reduction, so the components can sit on the MMA's M
// dimension and X passes through shared memory once:
//
//   TMA      X(t) -> one of four slots (two [128 rows][64 features] bf16
//            boxes, 128-byte swizzle); the weights (three bf16 terms) once
//   MMA      E-step S^T(t)[comp][row] = W[comp][feat] . X(t)^T: A = the
//            weights (K-major), B = the X slot as TMA left it (K-major,
//            rows x features); 24 instructions of N = 128 rows
//   prep     (4 warps, thread = row) |x|^2 of the row in fp32, and the row's
//            log-sum-exp, into a two-slot table
//   softmax  (16 warps, thread = component, four parts of 32 rows)
//            r = 2^(l - lse_row), l = c2 - h max(S + |x|^2 + |mu|^2, 0),
//            written back over its own S^T columns as r_hi, r_lo (bf16
//            pairs of rows): the M-step's A operand, in tensor memory;
//            n_k and sum r |x|^2 accumulate per thread (fp32 per tile,
//            fp64 across tiles)
//   MMA      M-step stats[comp][feat] += R^T(t) . X(t): A = r_hi then r_lo
//            from tensor memory, B = the same X slot read MN-major (rows x
//            64-feature groups); 16 instructions of N = 128 features
//
// Tensor memory holds three S^T / R^T buffers of 128 columns and the M-step
// accumulator (128), so the E-steps run up to three tiles ahead of the
// M-steps and the tensor pipe does not wait for the softmax; four X slots
// give each TMA load about two tile periods.  Shared memory: weights 96 KB
// + X slots 128 KB + the row tables.
//
// The logits repeat the first pass's arithmetic (em_tc_diag.cu, spherical
// layout): the same E-step instruction order over the weight terms and
// feature halves, |x|^2 summed over the features in order with fmaf, the
// same logit expression, so r sums to 1 over K up to the rounding of the
// two passes' tensor-core accumulation.
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

namespace gmmxx {
namespace tc {
namespace {

using namespace ptx;

constexpr int kBM = 128;      // rows per tile
constexpr int kKC = 128;      // components per CTA
constexpr int kNS = 3;        // bf16 terms of the split weights
constexpr int kBlock = 16384; // one [128][64] bf16 swizzled block
constexpr int kXSlots = 4;    // X tiles in flight
constexpr int kSR = 3;        // S^T / R^T buffers in tensor memory
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kDmCol = kSR * 128;  // M-step accumulator [comp][feature]

// The E-steps and the M-steps are issued by threads of two warps on
// different SM sub-partitions (warp % 4): each sub-partition also runs four
// softmax warps, and one issuing thread there for all MMAs of a tile was
// measured to hold the tensor pipe at about half its rate while the softmax
// ran.
enum Warp { kWarpTma = 0, kWarpMma = 1, kWarpPrep0 = 2, kWarpSoft0 = 6, kWarpMmaM = 22 };
constexpr int kSoftWarps = 16;
constexpr int kThreads = (kWarpMmaM + 1) * 32;  // 23 warps

// shared memory (byte offsets from the 1024-aligned dynamic block)
constexpr int kW = 0;                              // term j, features 64h.. at (2j + h) * kBlock
constexpr int kX = kW + 2 * kNS * kBlock;          // slot s: [box 0 | box 1] at kX + 2 s kBlock
constexpr int kQ = kX + kXSlots * 2 * kBlock;      // |x|^2 [2 slots][128 rows]
constexpr int kLse = kQ + 2 * 128 * 4;             // log-sum-exp (log2 units) [2 slots][128 rows]
constexpr int kBars = kLse + 2 * 128 * 4;
constexpr int kTotal = kBars + 256;
static_assert(kTotal <= 232448, "shared memory budget");
static_assert(kSR * 128 + 128 <= (int)kTmemCols, "tensor memory budget");

struct Bars {
  uint64_t params;            // TMA: weights landed
  uint64_t xfull[kXSlots];    // TMA: X tile landed in the slot
  uint64_t xfree[kXSlots];    // MMA: the M-step of the slot's tile is done
  uint64_t qfull[2];          // prep: |x|^2 and lse of the tile written (4 warps)
  uint64_t qfree[2];          // softmax: the slot's rows read (16 warps)
  uint64_t sfull[kSR];        // MMA: S^T(t) complete
  uint64_t rfull[kSR];        // softmax: R^T(t) written (16 warps)
  uint64_t mfree[kSR];        // MMA: the M-step read R^T(t): the buffer is free
  uint64_t mdone;             // MMA: every MMA complete (both issuing threads)
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

__device__ __forceinline__ void set_abort(Bars* b, int* status) {
  b->abort = 1;
  atomicOr(status, 1 << GMMXX_ERR_TIMEOUT);
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kThreads, 1)
    em_tc_sph_ext_kernel(const __grid_constant__ CUtensorMap tmap, TcArgs a) {
  extern __shared__ __align__(1024) char smem_raw[];
  char* sm = smem_raw;
  if ((smem_u32(smem_raw) & 1023u) != 0) {  // uniform across the grid: no CTA proceeds
    if (threadIdx.x == 0) atomicOr(a.status, 1 << GMMXX_ERR_UNSUPPORTED);
    return;
  }
  Bars* bars = reinterpret_cast<Bars*>(sm + kBars);
  float* qbuf = reinterpret_cast<float*>(sm + kQ);
  float* lbuf = reinterpret_cast<float*>(sm + kLse);
  volatile int* abort = &bars->abort;
  const uint64_t lim = a.wait_ns;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // a cluster-free launch: CTA i acts as chunk i % vcluster of the group for
  // the row tiles of virtual cluster i / vcluster
  const int vc = a.vcluster;
  const uint32_t rank = blockIdx.x % (uint32_t)vc;
  const uint32_t cid = blockIdx.x / (uint32_t)vc;
  const uint32_t ncl = gridDim.x / (uint32_t)vc;
  const int64_t ntiles = (a.N + kBM - 1) / kBM;
  const int T = (int)((ntiles > (int64_t)cid) ? (ntiles - 1 - cid) / ncl + 1 : 0);
  const int chunk = a.chunk0 + (int)rank;
  auto row0 = [&](int t) { return ((int64_t)cid + (int64_t)t * ncl) * kBM; };

  if (tid == 0) {
    mbar_init(&bars->params, 1);
    for (int i = 0; i < kXSlots; ++i) {
      mbar_init(&bars->xfull[i], 1);
      mbar_init(&bars->xfree[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->qfull[i], 4);
      mbar_init(&bars->qfree[i], kSoftWarps);
    }
    for (int i = 0; i < kSR; ++i) {
      mbar_init(&bars->sfull[i], 1);
      mbar_init(&bars->rfull[i], kSoftWarps);
      mbar_init(&bars->mfree[i], 1);
    }
    mbar_init(&bars->mdone, 2);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == kWarpMma) tmem_alloc(&bars->tmem_base, kTmemCols);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == kWarpTma) {
    // ---------------- producer: weights once, then X tiles ----------------
    if (lane == 0) {
      prefetch_tmap(&tmap);
      mbar_expect_tx(&bars->params, 2 * kNS * kBlock);
      const char* src = a.params + (int64_t)chunk * 2 * kNS * kBlock;
      for (int i = 0; i < 2 * kNS; ++i)
        bulk_load(sm + kW + i * kBlock, src + (int64_t)i * kBlock, kBlock, &bars->params);
      bool ok = true;
      int issued = 0;
      for (int t = 0; t < T; ++t) {
        const int s = t % kXSlots;
        if (t >= kXSlots && !mbar_wait(&bars->xfree[s], ((t / kXSlots) - 1) & 1, abort, lim)) { ok = false; break; }
        if (a.test_stall) break;  // test hook: no X tile ever lands, every wait on it runs out
        mbar_expect_tx(&bars->xfull[s], 2 * kBlock);
        char* dst = sm + kX + s * 2 * kBlock;
        tma_load_2d(dst, &tmap, 0, (int)row0(t), &bars->xfull[s]);
        tma_load_2d(dst + kBlock, &tmap, 64, (int)row0(t), &bars->xfull[s]);
        issued = t + 1;
      }
      if (!ok) set_abort(bars, a.status);
      // before the CTA can exit, every copy it started has landed (bounded,
      // also after an abort)
      mbar_wait(&bars->params, 0, nullptr, lim);
      for (int u = std::max(0, issued - kXSlots); u < issued; ++u)
        mbar_wait(&bars->xfull[u % kXSlots], (u / kXSlots) & 1, nullptr, lim);
    }
  } else if (warp == kWarpMma || warp == kWarpMmaM) {
    // ---------------- MMA issuers: E-steps (warp kWarpMma), M-steps (warp kWarpMmaM) ----------------
    if (lane == 0) {
      const uint32_t base = smem_u32(sm);
      bool ok = true;
      if (warp == kWarpMma) {
        const uint32_t id_e = idesc_bf16(128, 128, 0, 0);  // W (K-major) x X^T (K-major)
        ok = mbar_wait(&bars->params, 0, abort, lim);
        tmem_fence_after();
        uint64_t wd[kNS][2];
#pragma unroll
        for (int j = 0; j < kNS; ++j)
#pragma unroll
          for (int h = 0; h < 2; ++h) wd[j][h] = desc_kmajor(base + kW + (2 * j + h) * kBlock);
        // E-step of tile t into buffer t % 3 once the M-step of t - 3 has read
        // it, in the first pass's order: the weight terms over features 0-63,
        // then over features 64-127
        for (int t = 0; ok && t < T; ++t) {
          const int s = t % kXSlots, b = t % kSR;
          if (!mbar_wait(&bars->xfull[s], (t / kXSlots) & 1, abort, lim)) { ok = false; break; }
          if (t >= kSR && !mbar_wait(&bars->mfree[b], ((t / kSR) - 1) & 1, abort, lim)) { ok = false; break; }
          tmem_fence_after();
          const uint32_t d = tmem + (uint32_t)(b * 128);
          const uint32_t xs = base + kX + s * 2 * kBlock;
          uint32_t acc = 0;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint64_t xd = desc_kmajor(xs + h * kBlock);
#pragma unroll
            for (int j = 0; j < kNS; ++j)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {  // 16 features per instruction: +32 B
                mma_bf16(d, wd[j][h] + 2 * kk, xd + 2 * kk, id_e, acc);
                acc = 1;
              }
          }
          mma_commit(&bars->sfull[b]);
        }
      } else {
        // M-step of tile t: A = R^T(t) in the buffer's columns, part p of 32
        // rows at columns 32 p (r_hi, 16 columns of row pairs) and 32 p + 16
        // (r_lo); 16 rows per instruction
        const uint32_t id_m = idesc_bf16(128, 128, 0, 1);  // R^T (tensor memory) x X (MN-major)
        for (int t = 0; ok && t < T; ++t) {
          const int s = t % kXSlots, b = t % kSR;
          if (!mbar_wait(&bars->rfull[b], (t / kSR) & 1, abort, lim)) { ok = false; break; }
          tmem_fence_after();
          const uint64_t xm = desc_mnmajor(base + kX + s * 2 * kBlock, kBlock);
          const uint32_t rb = tmem + (uint32_t)(b * 128);
#pragma unroll
          for (int part = 0; part < 2; ++part)
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {  // rows 16 ks .. 16 ks + 15: +2048 B (MN-major)
              const uint32_t acol = (uint32_t)(32 * (ks >> 1) + 8 * (ks & 1) + 16 * part);
              mma_bf16_ts(tmem + kDmCol, rb + acol, xm + (uint64_t)(ks * 128), id_m,
                          (t == 0 && part == 0 && ks == 0) ? 0u : 1u);
            }
          mma_commit(&bars->mfree[b]);
          mma_commit(&bars->xfree[s]);
        }
      }
      if (!ok) set_abort(bars, a.status);
      mma_commit(&bars->mdone);
    }
  } else if (warp < kWarpSoft0) {
    // ---------------- prep: 4 warps, thread = row ----------------
    const int r = (warp - kWarpPrep0) * 32 + lane;
    const uint32_t swz = (uint32_t)(r & 7);
    auto lse_of = [&](int u) -> float {
      const int64_t g = row0(u) + r;
      return (u < T && g < a.N) ? __ldg(a.lse_in + g) : INFINITY;  // rows past N: r = 0
    };
    float lse_next = lse_of(0);
    bool ok = true;
    for (int t = 0; t < T; ++t) {
      const int s = t % kXSlots, qs = t & 1;
      if (!mbar_wait_warp(&bars->xfull[s], (t / kXSlots) & 1, abort, lim)) { ok = false; break; }
      const float lv = lse_next;
      lse_next = lse_of(t + 1);
      // |x|^2 over features 0 .. 127 in order (the first pass's sum)
      float q = 0.f;
      const char* xr = sm + kX + s * 2 * kBlock + r * 128;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = *reinterpret_cast<const uint4*>(xr + h * kBlock + ((c ^ swz) << 4));
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float x0 = bf16lo_to_f32(w[i]), x1 = bf16hi_to_f32(w[i]);
            q = fmaf(x0, x0, q);
            q = fmaf(x1, x1, q);
          }
        }
      if (t >= 2 && !mbar_wait_warp(&bars->qfree[qs], ((t >> 1) - 1) & 1, abort, lim)) { ok = false; break; }
      qbuf[qs * 128 + r] = q;
      lbuf[qs * 128 + r] = lv;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->qfull[qs]);
      if (*abort) { ok = false; break; }
    }
    if (!ok) set_abort(bars, a.status);
  } else {
    // ---------------- softmax: 16 warps (6 .. 21), thread = component ----------------
    // warp w reads lanes 32 (w % 4) .. + 31 (the tensor-memory access rule):
    // components 32 (w % 4) + lane; part p owns rows 32 p .. 32 p + 31
    const int q4 = warp & 3;
    const int p = (warp - kWarpSoft0) >> 2;
    const int kl = q4 * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q4 * 32) << 16;
    const float* cs = a.consts + (int64_t)chunk * 3 * 128;
    const float mpm = cs[kl], hh = cs[128 + kl], c2 = cs[256 + kl];  // padding: c2 = -inf
    double n_acc = 0.0, q_acc = 0.0;
    bool ok = true;
    for (int t = 0; t < T; ++t) {
      const int b = t % kSR, qs = t & 1;
      if (!mbar_wait_warp(&bars->sfull[b], (t / kSR) & 1, abort, lim)) { ok = false; break; }
      tmem_fence_after();
      const uint32_t col = tmem + lane_addr + (uint32_t)(b * 128 + 32 * p);
      float v[32];
      tmem_ld32(col, v);
      if (!mbar_wait_warp(&bars->qfull[qs], (t >> 1) & 1, abort, lim)) { ok = false; break; }
      tmem_wait_ld();
      const float4* q4p = reinterpret_cast<const float4*>(qbuf + qs * 128 + 32 * p);
      const float4* l4p = reinterpret_cast<const float4*>(lbuf + qs * 128 + 32 * p);
      float ns = 0.f, qsum = 0.f;
      uint32_t hw[16], lw[16];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 qq = q4p[c], ll = l4p[c];
        const float qv[4] = {qq.x, qq.y, qq.z, qq.w}, lv[4] = {ll.x, ll.y, ll.z, ll.w};
        float rv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float l = fmaf(-hh, fmaxf(v[4 * c + e] + (mpm + qv[e]), 0.f), c2);
          rv[e] = ex2_approx(l - lv[e]);
          ns += rv[e];
          qsum = fmaf(rv[e], qv[e], qsum);
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const uint32_t h2 = pack_bf16(rv[2 * e], rv[2 * e + 1]);
          hw[2 * c + e] = h2;
          lw[2 * c + e] = pack_bf16(rv[2 * e] - bf16lo_to_f32(h2), rv[2 * e + 1] - bf16hi_to_f32(h2));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->qfree[qs]);  // the tile's rows of the table are read
      tmem_st16(col, hw);
      tmem_st16(col + 16, lw);
      tmem_wait_st();
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->rfull[b]);
      n_acc += (double)ns;
      q_acc += (double)qsum;
      if (*abort) { ok = false; break; }
    }
    if (!ok) set_abort(bars, a.status);
    // ---------------- epilogue: statistics partials ----------------
    // the MMA thread always commits `mdone` (also after an abort): wait for it
    // without the abort shortcut before reading tensor memory.  Layout of a
    // component's partial row: [n_k | sum r x (128) | sum r |x|^2].
    if (!mbar_wait_warp(&bars->mdone, 0, nullptr, 2 * lim)) set_abort(bars, a.status);
    tmem_fence_after();
    const int comp = (int)rank * kKC + kl;
    float* out = a.part + ((int64_t)cid * a.Kp + comp) * a.F;
    float dv[32];
    tmem_ld32(tmem + lane_addr + kDmCol + (uint32_t)(32 * p), dv);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) out[1 + 32 * p + j] = T > 0 ? dv[j] : 0.f;
    // n_k and sum r |x|^2: the four parts' sums in part order (the X slots
    // are idle once every MMA is complete)
    double* red = reinterpret_cast<double*>(sm + kX);
    red[(p * 128 + kl) * 2] = n_acc;
    red[(p * 128 + kl) * 2 + 1] = q_acc;
    asm volatile("bar.sync 1, %0;" ::"n"(kSoftWarps * 32) : "memory");
    if (p == 0) {
      double n = 0.0, qq = 0.0;
#pragma unroll
      for (int pp = 0; pp < 4; ++pp) {
        n += red[(pp * 128 + kl) * 2];
        qq += red[(pp * 128 + kl) * 2 + 1];
      }
      out[0] = (float)n;
      out[1 + 128] = (float)qq;
    }
    tmem_fence_before();
  }
  __syncthreads();
  if (warp == kWarpMma) {
    tmem_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

// GMMXX_B200_SPH_PASS2=diag keeps the second pass on em_tc_diag_kernel's
// external-log-sum-exp mode (the A/B switch of the two layouts).
bool sph_ext_enabled() {
  const char* e = getenv("GMMXX_B200_SPH_PASS2");
  return !(e != nullptr && strcmp(e, "diag") == 0);
}

int launch_sph_ext(const TcLaunch& L, const CUtensorMap& tmap, int chunk0, int csize, cudaStream_t st,
                   int* ncl_out) {
  if (L.D != 128 || csize < 1 || L.lse == nullptr)
    return set_error(GMMXX_ERR_UNSUPPORTED, "spherical second pass: D = 128 with a log-sum-exp buffer");
  TcLaunch Lq = L;
  Lq.cluster_size = 1;
  int nctas = 0;
  if (int rc = clustered_launch((const void*)em_tc_sph_ext_kernel, kThreads, kTotal, Lq, &nctas)) return rc;
  const int ncl = nctas / csize;  // whole virtual clusters
  if (ncl < 1) return set_error(GMMXX_ERR_UNSUPPORTED, "too few co-resident CTAs for %d-chunk groups", csize);
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
  args.wait_ns = L.wait_ns ? L.wait_ns : 2000000000ull;
  args.test_stall = L.test_stall;
  args.K = L.K;
  args.chunk0 = chunk0;
  args.lse_in = L.lse;
  args.vcluster = csize;
  em_tc_sph_ext_kernel<<<(unsigned)(ncl * csize), kThreads, kTotal, st>>>(tmap, args);
  if (int rc = check_launch("em_tc_sph_ext_kernel")) return rc;
  *ncl_out = ncl;
  return GMMXX_OK;
}

}  // namespace tc
}  // namespace gmmxx
