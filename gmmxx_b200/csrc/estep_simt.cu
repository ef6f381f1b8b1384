// estep_simt.cu -- SIMT fp32 E-step / M-step statistics kernels (all four
// covariance types, any x dtype).
//
// These are the engine's exact-fp32 kernels: the logits, the streaming
// per-row logsumexp, responsibilities and the sufficient statistics are all
// computed in fp32 on the CUDA cores, in the same expanded-distance form as the
// reference's torch path (gmmxx/torch_fallback.py:337-465, 468-596,
// 2255-2291).  Tile: 64 rows x 64 components per CTA, 256 threads with 4x4
// register micro-tiles; features and component weights are staged through
// shared memory in chunks of 32.
//
//   rows_kernel   one pass over all K per row tile: logsumexp (+ sum for the
//                 log-likelihood), argmax (labels) or exp(logit - lse)
//                 (responsibilities / predict_proba).
//   mstep_kernel  grid (row blocks, K tiles, B): recomputes the logits of its
//                 64-component slice, r = exp(logit - lse), and accumulates
//                 sum_n r_nk psi(x_n) in registers over many row tiles; one
//                 flush per CTA into its own partial slot.  (N, K) is never
//                 materialised.
//   em_small_kernel  K <= 64 (one component tile): the two passes above in
//                 one -- logits, the row's logsumexp, r and the statistics per
//                 row tile, the log-likelihood summed per CTA.
//   topk_rows_kernel / topk_mstep_kernel  approximate top-k EM: each row's
//                 top_k components and responsibilities, then the statistics
//                 from those lists.
#include "rows_api.cuh"

#include <float.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>

namespace gmmxx {



template <int COV>
__device__ __forceinline__ float feat_e(const float* xr, int f, int D, const uint16_t* pairs) {
  if (COV == GMMXX_SPHERICAL || COV == GMMXX_TIED) return xr[f];
  if (COV == GMMXX_DIAG) return f < D ? xr[f] * xr[f] : xr[f - D];
  if (f < D) return xr[f];
  const uint16_t p = pairs[f - D];
  return xr[p & 0xff] * xr[p >> 8];
}

template <int COV>
__device__ __forceinline__ float feat_m(const float* xr, float q, int f, int D, int FM, const uint16_t* pairs) {
  if (f >= FM) return 0.f;
  if (f == 0) return 1.f;
  if (f <= D) return xr[f - 1];
  const int g = f - 1 - D;
  if (COV == GMMXX_SPHERICAL) return q;
  if (COV == GMMXX_DIAG) return xr[g] * xr[g];
  if (COV == GMMXX_FULL) {
    const uint16_t p = pairs[g];
    return xr[p & 0xff] * xr[p >> 8];
  }
  return 0.f;
}

// Shared-memory carve-up common to both kernels.
struct Smem {
  float* xs;        // [kBN][D+1]
  float* q;         // [kBN]
  float* phic;      // [kFC][kBN]
  float* wc;        // [kFC][kBK]
  float* prec;      // [D][D] (tied)
  uint16_t* pairs;  // [D(D+1)/2] (full)
  float* R;         // [kBN][kBK]      (mstep)
  float* phim;      // [kBN][64]       (mstep)
};

__host__ __device__ inline int64_t smem_bytes(int cov, int D, bool mstep) {
  int64_t b = 0;
  b += (int64_t)kBN * (D + 1) * 4;
  b += kBN * 4;
  b += kFC * kBN * 4 + kFC * kBK * 4;
  if (cov == GMMXX_TIED) b += (int64_t)D * D * 4;
  if (mstep) b += kBN * kBK * 4 + kBN * 64 * 4;
  if (cov == GMMXX_FULL) b += round_up((int64_t)D * (D + 1) / 2 * 2, 16);
  return b;
}

template <int COV>
__device__ __forceinline__ Smem carve(char* base, int D, bool mstep) {
  Smem s;
  float* p = reinterpret_cast<float*>(base);
  s.phic = p; p += kFC * kBN;
  s.wc = p; p += kFC * kBK;
  s.R = nullptr; s.phim = nullptr;
  if (mstep) { s.R = p; p += kBN * kBK; s.phim = p; p += kBN * 64; }
  s.q = p; p += kBN;
  s.prec = nullptr;
  if (COV == GMMXX_TIED) { s.prec = p; p += D * D; }
  s.xs = p; p += kBN * (D + 1);
  s.pairs = reinterpret_cast<uint16_t*>(p);
  return s;
}

// Stage one row tile of x (fp32 in smem, zero beyond N) and its q_n.
template <int COV>
__device__ __forceinline__ void load_rows(const RowArgs& a, const Smem& s, int b, int64_t row0) {
  const int D = a.D, xst = D + 1;
  const int64_t base = ((int64_t)b * a.N + row0) * D;
  const int64_t nrows = min((int64_t)kBN, a.N - row0);
  for (int e = threadIdx.x; e < kBN * D; e += kThreads) {
    const int r = e / D, d = e - r * D;
    s.xs[r * xst + d] = (r < nrows) ? load_x(a.x, base + e, a.dt) : 0.f;
  }
  __syncthreads();
  if (COV == GMMXX_SPHERICAL) {
    // |x|^2 (torch_fallback.py:1992, x_sq_all)
    if (threadIdx.x < kBN) {
      const float* xr = s.xs + threadIdx.x * xst;
      float acc = 0.f;
      for (int d = 0; d < D; ++d) acc = fmaf(xr[d], xr[d], acc);
      s.q[threadIdx.x] = acc;
    }
  } else if (COV == GMMXX_TIED) {
    if (a.q_in != nullptr) {  // computed by the LSE pass of this iteration
      if (threadIdx.x < kBN) {
        const int64_t row = row0 + threadIdx.x;
        s.q[threadIdx.x] = row < a.N ? a.q_in[(int64_t)b * a.N + row] : 0.f;
      }
    } else {
      // x^T P x (torch_fallback.py:452) as Y = X P on 4x4 register tiles
      // (thread: rows 4 ty.., columns 4 tx.. of each 64-column block), then
      // q = sum_j Y_j x_j reduced over the 16 threads of a row group
      const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
      float qp[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c0 = 0; c0 < D; c0 += 64) {
        const int col = c0 + tx * 4;
        float y[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) y[i][j] = 0.f;
        if (col < D) {
          for (int d = 0; d < D; ++d) {
            float xv[4], pv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) xv[i] = s.xs[(ty * 4 + i) * xst + d];
#pragma unroll
            for (int j = 0; j < 4; ++j) pv[j] = (col + j < D) ? s.prec[d * D + col + j] : 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int j = 0; j < 4; ++j) y[i][j] = fmaf(xv[i], pv[j], y[i][j]);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j)
              if (col + j < D) qp[i] = fmaf(y[i][j], s.xs[(ty * 4 + i) * xst + col + j], qp[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) qp[i] += __shfl_xor_sync(0xffffffffu, qp[i], o);
      if (tx == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          s.q[ty * 4 + i] = qp[i];
          const int64_t row = row0 + ty * 4 + i;
          if (a.q_out != nullptr && row < a.N) a.q_out[(int64_t)b * a.N + row] = qp[i];
        }
      }
    }
  } else {
    if (threadIdx.x < kBN) s.q[threadIdx.x] = 0.f;
  }
  __syncthreads();
}

// 64x64 dot products of the row tile's features with one component tile.
template <int COV>
__device__ __forceinline__ void tile_dots(const RowArgs& a, const Smem& s, int b, int kt, float acc[4][4]) {
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int D = a.D, xst = D + 1, FE = a.FE;
  const float* wtb = a.wt + (int64_t)b * FE * a.Kp + (int64_t)kt * kBK;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int f0 = 0; f0 < FE; f0 += kFC) {
    __syncthreads();
    for (int e = threadIdx.x; e < kFC * kBN; e += kThreads) {
      const int r = e & (kBN - 1), f = e / kBN;
      s.phic[e] = (f0 + f < FE) ? feat_e<COV>(s.xs + r * xst, f0 + f, D, s.pairs) : 0.f;
    }
    for (int e = threadIdx.x; e < kFC * kBK; e += kThreads) {
      const int k = e & (kBK - 1), f = e / kBK;
      s.wc[e] = (f0 + f < FE) ? __ldg(wtb + (int64_t)(f0 + f) * a.Kp + k) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int f = 0; f < kFC; ++f) {
      const float4 xv = *reinterpret_cast<const float4*>(s.phic + f * kBN + ty * 4);
      const float4 wv = *reinterpret_cast<const float4*>(s.wc + f * kBK + tx * 4);
      const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
      const float wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wa[j], acc[i][j]);
    }
  }
}

// acc -> logits in place (invalid components -> -inf).
__device__ __forceinline__ void to_logits(const RowArgs& a, const Smem& s, int b, int kt, float acc[4][4]) {
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int k = kt * kBK + tx * 4 + j;
    if (k < a.K) {
      const CompConst c = a.cc[(int64_t)b * a.K + k];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float dist = s.q[ty * 4 + i] + acc[i][j] + c.mpm;
        dist = fmaxf(dist, 0.f);
        acc[i][j] = c.lw - 0.5f * (c.s * dist + c.ln);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i][j] = -INFINITY;
    }
  }
}

__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) { m = m2; s = s2; return; }
  const float nm = fmaxf(m, m2);
  s = s * expf(m - nm) + s2 * expf(m2 - nm);
  m = nm;
}

// sum_n r_nk psi(x_n) for one row tile (R in s.R): n_k, the statistic of the
// constant feature 0, as a column sum of R; the other FM - 1 features in
// 64-wide chunks (thread: components 4 kg.., features 4 fg.. of a chunk)
template <int COV, int NCH>
__device__ __forceinline__ void mstep_tile(const RowArgs& a, const Smem& s, float (&macc)[NCH][4][4],
                                           float (&nk)[4]) {
  const int kg = threadIdx.x >> 4, fg = threadIdx.x & 15;
  const int D = a.D, xst = D + 1;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    __syncthreads();
    for (int e = threadIdx.x; e < kBN * 64; e += kThreads) {
      const int r = e >> 6, f = e & 63;
      s.phim[e] = feat_m<COV>(s.xs + r * xst, s.q[r], 1 + c * 64 + f, D, a.FM, s.pairs);
    }
    __syncthreads();
#pragma unroll 4
    for (int r = 0; r < kBN; ++r) {
      const float4 rv = *reinterpret_cast<const float4*>(s.R + r * kBK + kg * 4);
      const float4 pv = *reinterpret_cast<const float4*>(s.phim + r * 64 + fg * 4);
      const float ra[4] = {rv.x, rv.y, rv.z, rv.w};
      const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
      if (c == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) nk[i] += ra[i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) macc[c][i][j] = fmaf(ra[i], pa[j], macc[c][i][j]);
    }
  }
}

// one CTA's statistics into its partial slot st[Kp][FM] (component tile kt)
template <int NCH>
__device__ __forceinline__ void mstep_flush(const RowArgs& a, float* st, int kt, const float (&macc)[NCH][4][4],
                                            const float (&nk)[4]) {
  const int kg = threadIdx.x >> 4, fg = threadIdx.x & 15;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int k = kt * kBK + kg * 4 + i;
    if (k >= a.K) continue;
    if (fg == 0) st[(int64_t)k * a.FM] = nk[i];
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int f = 1 + c * 64 + fg * 4 + j;
        if (f < a.FM) st[(int64_t)k * a.FM + f] = macc[c][i][j];
      }
  }
}

template <int COV, int MODE>
__global__ void __launch_bounds__(kThreads) rows_kernel(RowArgs a) {
  extern __shared__ __align__(16) char smem_raw[];
  const Smem s = carve<COV>(smem_raw, a.D, false);
  const int b = blockIdx.y;
  const int64_t row0 = (int64_t)blockIdx.x * kBN;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  if (COV == GMMXX_TIED) {
    const float* pb = a.prec + (int64_t)b * a.D * a.D;
    for (int e = threadIdx.x; e < a.D * a.D; e += kThreads) s.prec[e] = pb[e];
  }
  if (COV == GMMXX_FULL) {
    for (int i = threadIdx.x; i < a.D; i += kThreads) {
      int p = i * a.D - i * (i - 1) / 2;  // index of (i, i) in the packed i<=j order
      for (int j = i; j < a.D; ++j) s.pairs[p++] = (uint16_t)(i | (j << 8));
    }
  }
  __syncthreads();
  load_rows<COV>(a, s, b, row0);

  float run_m[4], run_s[4], lse_row[4];
  float best_v[4];
  int best_k[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    run_m[i] = -INFINITY; run_s[i] = 0.f; best_v[i] = -INFINITY; best_k[i] = 0;
    const int64_t row = row0 + ty * 4 + i;
    lse_row[i] = (MODE == MODE_RESP && row < a.N) ? a.lse_in[(int64_t)b * a.N + row] : 0.f;
  }
  const int ktiles = (int)(a.Kp / kBK);
  float acc[4][4];
  for (int kt = 0; kt < ktiles; ++kt) {
    tile_dots<COV>(a, s, b, kt, acc);
    to_logits(a, s, b, kt, acc);
    if (MODE == MODE_LSE) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float m = fmaxf(fmaxf(acc[i][0], acc[i][1]), fmaxf(acc[i][2], acc[i][3]));
        float sm = 0.f;
        if (m != -INFINITY) {
#pragma unroll
          for (int j = 0; j < 4; ++j) sm += expf(acc[i][j] - m);
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) {
          const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
          const float s2 = __shfl_xor_sync(0xffffffffu, sm, o);
          lse_merge(m, sm, m2, s2);
        }
        lse_merge(run_m[i], run_s[i], m, sm);
      }
    } else if (MODE == MODE_ARGMAX) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float v = best_v[i];
        int kk = best_k[i];
        float tv = -INFINITY;
        int tk = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (acc[i][j] > tv) { tv = acc[i][j]; tk = kt * kBK + tx * 4 + j; }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) {
          const float v2 = __shfl_xor_sync(0xffffffffu, tv, o);
          const int k2 = __shfl_xor_sync(0xffffffffu, tk, o);
          if (v2 > tv || (v2 == tv && k2 < tk)) { tv = v2; tk = k2; }
        }
        if (tv > v) { v = tv; kk = tk; }  // later tiles replace only on strictly larger
        best_v[i] = v; best_k[i] = kk;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t row = row0 + ty * 4 + i;
        if (row >= a.N) continue;
        float* orow = a.out + ((int64_t)b * a.N + row) * a.K;
        const int k0 = kt * kBK + tx * 4;
        float p[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) p[j] = expf(acc[i][j] - lse_row[i]);
        if ((a.K & 3) == 0 && k0 + 3 < a.K) {
          *reinterpret_cast<float4*>(orow + k0) = make_float4(p[0], p[1], p[2], p[3]);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (k0 + j < a.K) orow[k0 + j] = p[j];
        }
      }
    }
  }

  if (MODE == MODE_LSE) {
    double part = 0.0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t row = row0 + ty * 4 + i;
      const float l = run_m[i] + logf(run_s[i]);
      if (row < a.N && tx == 0) {
        a.lse_out[(int64_t)b * a.N + row] = l;
        part += (double)l;
      }
    }
    if (a.ll_part != nullptr) {
      __shared__ double red[kThreads / 32];
      const double tot = block_sum<double>(part, red);
      if (threadIdx.x == 0) a.ll_part[(int64_t)b * gridDim.x + blockIdx.x] = tot;
    }
  } else if (MODE == MODE_ARGMAX) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t row = row0 + ty * 4 + i;
      if (row < a.N && tx == 0) a.labels[(int64_t)b * a.N + row] = best_k[i];
    }
  }
}

template <int COV, int NCH>
__global__ void __launch_bounds__(kThreads) mstep_kernel(RowArgs a) {
  extern __shared__ __align__(16) char smem_raw[];
  const Smem s = carve<COV>(smem_raw, a.D, true);
  const int b = blockIdx.z, kt = blockIdx.y;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int D = a.D;
  if (COV == GMMXX_TIED) {
    const float* pb = a.prec + (int64_t)b * D * D;
    for (int e = threadIdx.x; e < D * D; e += kThreads) s.prec[e] = pb[e];
  }
  if (COV == GMMXX_FULL) {
    for (int i = threadIdx.x; i < D; i += kThreads) {
      int p = i * D - i * (i - 1) / 2;
      for (int j = i; j < D; ++j) s.pairs[p++] = (uint16_t)(i | (j << 8));
    }
  }
  float macc[NCH][4][4];
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) macc[c][i][j] = 0.f;
  float nk[4] = {0.f, 0.f, 0.f, 0.f};

  const int64_t rstart = (int64_t)blockIdx.x * a.rows_per_cta;
  const int64_t rend = min(rstart + a.rows_per_cta, a.N);
  const float* lse_b = a.lse_in + (int64_t)b * a.N;
  float acc[4][4];
  for (int64_t row0 = rstart; row0 < rend; row0 += kBN) {
    __syncthreads();
    load_rows<COV>(a, s, b, row0);
    tile_dots<COV>(a, s, b, kt, acc);
    to_logits(a, s, b, kt, acc);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t row = row0 + ty * 4 + i;
      const bool ok = row < rend;
      const float l = ok ? lse_b[row] : 0.f;
      float r[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = ok ? expf(acc[i][j] - l) : 0.f;  // -inf -> 0
      *reinterpret_cast<float4*>(s.R + (ty * 4 + i) * kBK + tx * 4) = make_float4(r[0], r[1], r[2], r[3]);
    }
    mstep_tile<COV, NCH>(a, s, macc, nk);
  }
  // one flush per CTA into its own partial slot (reduced in a fixed order later)
  mstep_flush<NCH>(a, a.part + ((int64_t)b * a.part_blocks + blockIdx.x) * a.Kp * a.FM, kt, macc, nk);
}

// One pass for K <= 64: every component of a row is in this CTA's tile, so
// the row's logsumexp is complete after one tile_dots.  Same arithmetic, in
// the same order, as rows_kernel<MODE_LSE> followed by mstep_kernel (the
// statistics are bitwise identical; the log-likelihood is summed per CTA).
template <int COV, int NCH>
__global__ void __launch_bounds__(kThreads) em_small_kernel(RowArgs a) {
  extern __shared__ __align__(16) char smem_raw[];
  const Smem s = carve<COV>(smem_raw, a.D, true);
  const int b = blockIdx.z;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int D = a.D;
  if (COV == GMMXX_TIED) {
    const float* pb = a.prec + (int64_t)b * D * D;
    for (int e = threadIdx.x; e < D * D; e += kThreads) s.prec[e] = pb[e];
  }
  if (COV == GMMXX_FULL) {
    for (int i = threadIdx.x; i < D; i += kThreads) {
      int p = i * D - i * (i - 1) / 2;
      for (int j = i; j < D; ++j) s.pairs[p++] = (uint16_t)(i | (j << 8));
    }
  }
  float macc[NCH][4][4];
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) macc[c][i][j] = 0.f;
  float nk[4] = {0.f, 0.f, 0.f, 0.f};
  double ll = 0.0;

  const int64_t rstart = (int64_t)blockIdx.x * a.rows_per_cta;
  const int64_t rend = min(rstart + a.rows_per_cta, a.N);
  float acc[4][4];
  for (int64_t row0 = rstart; row0 < rend; row0 += kBN) {
    __syncthreads();
    load_rows<COV>(a, s, b, row0);
    tile_dots<COV>(a, s, b, 0, acc);
    to_logits(a, s, b, 0, acc);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // the row's logsumexp over its 16 threads (as rows_kernel<MODE_LSE>)
      float m = fmaxf(fmaxf(acc[i][0], acc[i][1]), fmaxf(acc[i][2], acc[i][3]));
      float sm = 0.f;
      if (m != -INFINITY) {
#pragma unroll
        for (int j = 0; j < 4; ++j) sm += expf(acc[i][j] - m);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, sm, o);
        lse_merge(m, sm, m2, s2);
      }
      float run_m = -INFINITY, run_s = 0.f;
      lse_merge(run_m, run_s, m, sm);
      const float l = run_m + logf(run_s);
      const int64_t row = row0 + ty * 4 + i;
      const bool ok = row < rend;
      if (ok && tx == 0) ll += (double)l;
      float r[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = ok ? expf(acc[i][j] - l) : 0.f;  // -inf -> 0
      *reinterpret_cast<float4*>(s.R + (ty * 4 + i) * kBK + tx * 4) = make_float4(r[0], r[1], r[2], r[3]);
    }
    mstep_tile<COV, NCH>(a, s, macc, nk);
  }
  mstep_flush<NCH>(a, a.part + ((int64_t)b * a.part_blocks + blockIdx.x) * a.Kp * a.FM, 0, macc, nk);
  if (a.ll_part != nullptr) {
    __shared__ double red[kThreads / 32];
    const double tot = block_sum<double>(ll, red);
    if (threadIdx.x == 0) a.ll_part[(int64_t)b * gridDim.x + blockIdx.x] = tot;
  }
}

// Full covariance, K <= 32: the one-pass kernel on a 128-row x 32-component
// tile.  The 64 x 64 tile above pads K = 32 to 64 components, so half of its
// E-step and M-step products are spent on padding; here each one counts.
// E-step thread: rows 4 ty.., components 4 tx.. (8 x 32 threads), the same
// feature order as tile_dots; the row's log-sum-exp over its 8 threads,
// merged in the order the 64-wide tile merges its non-empty lanes.  M-step
// thread: components 4 kg.., features 4 fg.. of a 64-feature chunk, over one
// half (rh) of the tile's rows; the halves are added (half 0 + half 1) at
// the flush, so the statistics are deterministic.
constexpr int kNR = 128;  // rows per tile
constexpr int kNK = 32;   // components

__host__ __device__ inline int64_t smem_bytes_narrow(int D) {
  return (int64_t)(kFC * kNR + kFC * kNK + kNR * kNK + kNR * 64 + kNR * (D + 1)) * 4 +
         round_up((int64_t)D * (D + 1) / 2 * 2, 16);
}

template <int NCH>
__global__ void __launch_bounds__(kThreads) em_small_narrow_kernel(RowArgs a) {
  static_assert(kThreads == 256 && NCH <= 3, "thread maps and the flush buffer");
  extern __shared__ __align__(16) char smem_raw[];
  const int D = a.D, xst = D + 1, FE = a.FE;
  float* phic = reinterpret_cast<float*>(smem_raw);  // [kFC][kNR]
  float* wc = phic + kFC * kNR;                        // [kFC][kNK]
  float* R = wc + kFC * kNK;                           // [kNR][kNK]
  float* phim = R + kNR * kNK;                         // [kNR][64]
  float* xs = phim + kNR * 64;                         // [kNR][D + 1]
  uint16_t* pairs = reinterpret_cast<uint16_t*>(xs + kNR * xst);
  const int b = blockIdx.z;
  const int tx = threadIdx.x & 7, ty = threadIdx.x >> 3;                                // E-step 8 x 32
  const int kg = threadIdx.x & 7, fg = (threadIdx.x >> 3) & 15, rh = threadIdx.x >> 7;  // M-step 8 x 16 x 2
  for (int i = threadIdx.x; i < D; i += kThreads) {
    int p = i * D - i * (i - 1) / 2;
    for (int j = i; j < D; ++j) pairs[p++] = (uint16_t)(i | (j << 8));
  }
  float macc[NCH][4][4];
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) macc[c][i][j] = 0.f;
  float nk[4] = {0.f, 0.f, 0.f, 0.f};
  double ll = 0.0;
  const float* wtb = a.wt + (int64_t)b * FE * a.Kp;

  const int64_t rstart = (int64_t)blockIdx.x * a.rows_per_cta;
  const int64_t rend = min(rstart + a.rows_per_cta, a.N);
  float acc[4][4];
  for (int64_t row0 = rstart; row0 < rend; row0 += kNR) {
    __syncthreads();  // the previous tile's reads of xs, R and phim are done
    {
      const int64_t base = ((int64_t)b * a.N + row0) * D;
      const int64_t nrows = min((int64_t)kNR, a.N - row0);
      for (int e = threadIdx.x; e < kNR * D; e += kThreads) {
        const int r = e / D, d = e - r * D;
        xs[r * xst + d] = (r < nrows) ? load_x(a.x, base + e, a.dt) : 0.f;
      }
    }
    // E-step: the tile's features against the 32 components, kFC at a time
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    for (int f0 = 0; f0 < FE; f0 += kFC) {
      __syncthreads();
      for (int e = threadIdx.x; e < kFC * kNR; e += kThreads) {
        const int r = e & (kNR - 1), f = e / kNR;
        phic[e] = (f0 + f < FE) ? feat_e<GMMXX_FULL>(xs + r * xst, f0 + f, D, pairs) : 0.f;
      }
      for (int e = threadIdx.x; e < kFC * kNK; e += kThreads) {
        const int k = e & (kNK - 1), f = e / kNK;
        wc[e] = (f0 + f < FE) ? __ldg(wtb + (int64_t)(f0 + f) * a.Kp + k) : 0.f;
      }
      __syncthreads();
#pragma unroll 8
      for (int f = 0; f < kFC; ++f) {
        const float4 xv = *reinterpret_cast<const float4*>(phic + f * kNR + ty * 4);
        const float4 wv = *reinterpret_cast<const float4*>(wc + f * kNK + tx * 4);
        const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
        const float wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wa[j], acc[i][j]);
      }
    }
    // logits (full covariance: no per-row term), invalid components -> -inf
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = tx * 4 + j;
      if (k < a.K) {
        const CompConst c = a.cc[(int64_t)b * a.K + k];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float dist = acc[i][j] + c.mpm;
          dist = fmaxf(dist, 0.f);
          acc[i][j] = c.lw - 0.5f * (c.s * dist + c.ln);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i][j] = -INFINITY;
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float m = fmaxf(fmaxf(acc[i][0], acc[i][1]), fmaxf(acc[i][2], acc[i][3]));
      float sm = 0.f;
      if (m != -INFINITY) {
#pragma unroll
        for (int j = 0; j < 4; ++j) sm += expf(acc[i][j] - m);
      }
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, sm, o);
        lse_merge(m, sm, m2, s2);
      }
      float run_m = -INFINITY, run_s = 0.f;
      lse_merge(run_m, run_s, m, sm);
      const float l = run_m + logf(run_s);
      const int64_t row = row0 + ty * 4 + i;
      const bool ok = row < rend;
      if (ok && tx == 0) ll += (double)l;
      float r[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = ok ? expf(acc[i][j] - l) : 0.f;  // -inf -> 0
      *reinterpret_cast<float4*>(R + (ty * 4 + i) * kNK + tx * 4) = make_float4(r[0], r[1], r[2], r[3]);
    }
    // M-step: sum over this half's rows of r_nk psi(x_n), 64 features at a time
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      __syncthreads();  // R written; the previous chunk's reads of phim are done
      for (int e = threadIdx.x; e < kNR * 64; e += kThreads) {
        const int r = e >> 6, f = e & 63;
        phim[e] = feat_m<GMMXX_FULL>(xs + r * xst, 0.f, 1 + c * 64 + f, D, a.FM, pairs);
      }
      __syncthreads();
#pragma unroll 4
      for (int rr = 0; rr < kNR / 2; ++rr) {
        const int r = rh * (kNR / 2) + rr;
        const float4 rv = *reinterpret_cast<const float4*>(R + r * kNK + kg * 4);
        const float4 pv = *reinterpret_cast<const float4*>(phim + r * 64 + fg * 4);
        const float ra[4] = {rv.x, rv.y, rv.z, rv.w};
        const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
        if (c == 0) {
#pragma unroll
          for (int i = 0; i < 4; ++i) nk[i] += ra[i];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) macc[c][i][j] = fmaf(ra[i], pa[j], macc[c][i][j]);
      }
    }
  }
  // flush: half 1 hands its sums to half 0 through shared memory (phim, idle
  // now), half 0 adds them and writes this CTA's partial slot
  constexpr int kW = NCH * 16 + 4;
  static_assert(128 * kW <= kNR * 64, "flush buffer inside phim");
  __syncthreads();
  float* red = phim + (threadIdx.x & 127) * kW;
  if (rh == 1) {
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) red[c * 16 + i * 4 + j] = macc[c][i][j];
#pragma unroll
    for (int i = 0; i < 4; ++i) red[NCH * 16 + i] = nk[i];
  }
  __syncthreads();
  if (rh == 0) {
    float* st = a.part + ((int64_t)b * a.part_blocks + blockIdx.x) * a.Kp * a.FM;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = kg * 4 + i;
      if (k >= a.K) continue;
      if (fg == 0) st[(int64_t)k * a.FM] = nk[i] + red[NCH * 16 + i];
#pragma unroll
      for (int c = 0; c < NCH; ++c)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int f = 1 + c * 64 + fg * 4 + j;
          if (f < a.FM) st[(int64_t)k * a.FM + f] = macc[c][i][j] + red[c * 16 + i * 4 + j];
        }
    }
  }
  if (a.ll_part != nullptr) {
    __shared__ double red_ll[kThreads / 32];
    const double tot = block_sum<double>(ll, red_ll);
    if (threadIdx.x == 0) a.ll_part[(int64_t)b * gridDim.x + blockIdx.x] = tot;
  }
}

// Approximate top-k EM (torch_fallback.py:667-767 _topk_logits_for_chunk /
// _accumulate_topk_stats; _cuda.py:783-889): a row's responsibilities are
// the softmax of its top_k logits, zero for every other component.
//
// Selection pass, grid (row tiles, B): the logits of each 64-component tile
// go through shared memory, and one thread per row merges them into the
// row's list, sorted by logit (descending) with the lower component index
// first among equal logits (a candidate enters only when strictly larger than
// the list's last entry, and moves up only past strictly smaller entries).
// After the last tile: the list's log-sum-exp (summed per CTA into the
// log-likelihood partials, as rows_kernel<MODE_LSE> does), and the lists of
// (component, r = exp(logit - lse)) to scratch.
__host__ __device__ inline int64_t topk_rows_smem(int cov, int D, int top_k) {
  return smem_bytes(cov, D, false) + (int64_t)kBN * (kBK + 1) * 4 + (int64_t)top_k * kBN * 8;
}

template <int COV>
__global__ void __launch_bounds__(kThreads) topk_rows_kernel(RowArgs a) {
  extern __shared__ __align__(16) char smem_raw[];
  const Smem s = carve<COV>(smem_raw, a.D, false);
  float* lt = reinterpret_cast<float*>(smem_raw + smem_bytes(COV, a.D, false));  // [kBN][kBK + 1]
  const int T = a.top_k;
  float* lv = lt + kBN * (kBK + 1);                       // [T][kBN] list logits
  int* li = reinterpret_cast<int*>(lv + T * kBN);         // [T][kBN] list components
  const int b = blockIdx.y;
  const int64_t row0 = (int64_t)blockIdx.x * kBN;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  if (COV == GMMXX_TIED) {
    const float* pb = a.prec + (int64_t)b * a.D * a.D;
    for (int e = threadIdx.x; e < a.D * a.D; e += kThreads) s.prec[e] = pb[e];
  }
  if (COV == GMMXX_FULL) {
    for (int i = threadIdx.x; i < a.D; i += kThreads) {
      int p = i * a.D - i * (i - 1) / 2;
      for (int j = i; j < a.D; ++j) s.pairs[p++] = (uint16_t)(i | (j << 8));
    }
  }
  for (int e = threadIdx.x; e < T * kBN; e += kThreads) {
    lv[e] = -INFINITY;
    li[e] = -1;
  }
  __syncthreads();
  load_rows<COV>(a, s, b, row0);

  const int ktiles = (int)(a.Kp / kBK);
  float acc[4][4];
  for (int kt = 0; kt < ktiles; ++kt) {
    tile_dots<COV>(a, s, b, kt, acc);
    to_logits(a, s, b, kt, acc);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) lt[(ty * 4 + i) * (kBK + 1) + tx * 4 + j] = acc[i][j];
    __syncthreads();
    if (threadIdx.x < kBN) {
      const int r = threadIdx.x;
      const int kn = min(kBK, a.K - kt * kBK);
      float vmin = lv[(T - 1) * kBN + r];
      for (int c = 0; c < kn; ++c) {
        const float v = lt[r * (kBK + 1) + c];
        if (!(v > vmin)) continue;
        int t = T - 1;
        while (t > 0 && v > lv[(t - 1) * kBN + r]) {
          lv[t * kBN + r] = lv[(t - 1) * kBN + r];
          li[t * kBN + r] = li[(t - 1) * kBN + r];
          --t;
        }
        lv[t * kBN + r] = v;
        li[t * kBN + r] = kt * kBK + c;
        vmin = lv[(T - 1) * kBN + r];
      }
    }
    __syncthreads();  // the next tile's logits overwrite lt
  }

  double part = 0.0;
  if (threadIdx.x < kBN) {
    const int r = threadIdx.x;
    const int64_t row = row0 + r;
    if (row < a.N) {
      const float m = lv[r];
      float sm = 0.f;
      if (m != -INFINITY) {
        for (int t = 0; t < T; ++t) sm += expf(lv[t * kBN + r] - m);
      }
      const float l = (m == -INFINITY) ? -INFINITY : m + logf(sm);
      const int64_t o = ((int64_t)b * a.N + row) * T;
      for (int t = 0; t < T; ++t) {
        a.topk_idx[o + t] = li[t * kBN + r];
        a.topk_r[o + t] = (m == -INFINITY) ? 0.f : expf(lv[t * kBN + r] - l);
      }
      part = (double)l;
    }
  }
  if (a.ll_part != nullptr) {
    __shared__ double red[kThreads / 32];
    const double tot = block_sum<double>(part, red);
    if (threadIdx.x == 0) a.ll_part[(int64_t)b * gridDim.x + blockIdx.x] = tot;
  }
}

// M-step over the top-k lists, grid (row blocks, component tiles, B) like
// mstep_kernel: a row tile's R block (64 rows x this CTA's 64 components) is
// filled from the lists instead of recomputed logits, and tiles where no row
// has a listed component in this slice are skipped.
template <int COV, int NCH>
__global__ void __launch_bounds__(kThreads) topk_mstep_kernel(RowArgs a) {
  extern __shared__ __align__(16) char smem_raw[];
  const Smem s = carve<COV>(smem_raw, a.D, true);
  const int b = blockIdx.z, kt = blockIdx.y;
  const int D = a.D, T = a.top_k;
  if (COV == GMMXX_TIED) {
    const float* pb = a.prec + (int64_t)b * D * D;
    for (int e = threadIdx.x; e < D * D; e += kThreads) s.prec[e] = pb[e];
  }
  if (COV == GMMXX_FULL) {
    for (int i = threadIdx.x; i < D; i += kThreads) {
      int p = i * D - i * (i - 1) / 2;
      for (int j = i; j < D; ++j) s.pairs[p++] = (uint16_t)(i | (j << 8));
    }
  }
  float macc[NCH][4][4];
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) macc[c][i][j] = 0.f;
  float nk[4] = {0.f, 0.f, 0.f, 0.f};

  const int64_t rstart = (int64_t)blockIdx.x * a.rows_per_cta;
  const int64_t rend = min(rstart + a.rows_per_cta, a.N);
  const int k0 = kt * kBK;
  for (int64_t row0 = rstart; row0 < rend; row0 += kBN) {
    __syncthreads();  // the previous tile's reads of R are done
    for (int e = threadIdx.x; e < kBN * kBK; e += kThreads) s.R[e] = 0.f;
    __syncthreads();
    int has = 0;
    if (threadIdx.x < kBN) {
      const int64_t row = row0 + threadIdx.x;
      if (row < rend) {
        const int64_t o = ((int64_t)b * a.N + row) * T;
        for (int t = 0; t < T; ++t) {
          const int c = a.topk_idx[o + t] - k0;  // -1 entries fall outside every slice
          if (c >= 0 && c < kBK) {
            s.R[threadIdx.x * kBK + c] = a.topk_r[o + t];
            has = 1;
          }
        }
      }
    }
    if (__syncthreads_or(has) == 0) continue;
    load_rows<COV>(a, s, b, row0);
    mstep_tile<COV, NCH>(a, s, macc, nk);
  }
  mstep_flush<NCH>(a, a.part + ((int64_t)b * a.part_blocks + blockIdx.x) * a.Kp * a.FM, kt, macc, nk);
}

__global__ void stats_reduce_kernel(const float* part, int64_t nblk, int64_t stride, int64_t Kp, int K, int FM,
                                    int B, float* stats, const double* ll_part, int64_t nll, double* ll) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per_b = (int64_t)K * FM;
  if (i < per_b * B) {
    const int64_t b = i / per_b, r = i - b * per_b;
    const int64_t k = r / FM, f = r - k * FM;
    const float* p = part + (b * stride) * Kp * FM + k * FM + f;
    float s = 0.f;
    for (int64_t c = 0; c < nblk; ++c) s += p[c * Kp * FM];
    stats[i] += s;
  }
  if (i == 0 && ll != nullptr) {
    double s = 0.0;
    for (int64_t c = 0; c < nll * B; ++c) s += ll_part[c];
    *ll += s;
  }
}

// xx (B, D, D) += sum_n x_n x_n^T  (tied covariance; torch_fallback.py:2856-2862)
__global__ void __launch_bounds__(kThreads) xx_total_kernel(const void* x, int dt, int64_t N, int D,
                                                            int64_t rows_per_cta, float* xx) {
  extern __shared__ __align__(16) char smem_raw[];
  float* xs = reinterpret_cast<float*>(smem_raw);  // [kBN][D+1]
  const int b = blockIdx.y;
  const int xst = D + 1;
  const int64_t rstart = (int64_t)blockIdx.x * rows_per_cta;
  const int64_t rend = min(rstart + rows_per_cta, N);
  constexpr int kPer = (kMaxD * kMaxD) / kThreads;  // 64
  float acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) acc[i] = 0.f;
  for (int64_t row0 = rstart; row0 < rend; row0 += kBN) {
    __syncthreads();
    const int64_t nrows = min((int64_t)kBN, rend - row0);
    const int64_t base = ((int64_t)b * N + row0) * D;
    for (int e = threadIdx.x; e < kBN * D; e += kThreads) {
      const int r = e / D, d = e - r * D;
      xs[r * xst + d] = (r < nrows) ? load_x(x, base + e, dt) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = threadIdx.x + i * kThreads;
      if (e < D * D) {
        const int di = e / D, de = e - di * D;
        float t = acc[i];
        for (int r = 0; r < kBN; ++r) t = fmaf(xs[r * xst + di], xs[r * xst + de], t);
        acc[i] = t;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = threadIdx.x + i * kThreads;
    if (e < D * D) xx[((int64_t)b * gridDim.x + blockIdx.x) * D * D + e] = acc[i];  // this CTA's partial
  }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------

static int sm_count() {
  static int cached = 0;
  if (cached == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&cached, cudaDevAttrMultiProcessorCount, dev);
    if (cached <= 0) cached = 148;
  }
  return cached;
}

// Row blocks of a (row blocks, component tiles, B) statistics grid: as many
// as fill one wave of co-resident CTAs (a partly filled second or third
// wave would cost a whole wave), at most the partial slots the workspace
// reserves (mstep_blocks) and at most one per row tile.
template <typename KernelT>
static int64_t wave_blocks(KernelT k, int64_t smem, int64_t ktiles, int64_t B, int64_t nblk_max, int64_t tiles) {
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kThreads, (size_t)smem) != cudaSuccess || occ < 1) {
    cudaGetLastError();
    occ = 1;
  }
  int64_t nblk = (int64_t)sm_count() * occ / (ktiles * B);
  nblk = std::min(std::max<int64_t>(nblk, 1), nblk_max);
  return std::min(nblk, std::max<int64_t>(tiles, 1));
}

template <typename KernelT>
static int prep_smem(KernelT k, int64_t bytes) {
  if (bytes > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return set_error(GMMXX_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  }
  return GMMXX_OK;
}

template <int COV, int MODE>
static int launch_rows_t(const RowArgs& a, int B, cudaStream_t st) {
  const int64_t sm = smem_bytes(COV, a.D, false);
  auto k = rows_kernel<COV, MODE>;
  if (int rc = prep_smem(k, sm)) return rc;
  dim3 grid((unsigned)ceil_div(a.N, kBN), (unsigned)B);
  k<<<grid, kThreads, sm, st>>>(a);
  return check_launch("rows_kernel");
}

int launch_rows(int cov, int mode, const RowArgs& a, int B, cudaStream_t st) {
  if (a.N == 0) return GMMXX_OK;
#define GMMXX_ROWS_CASE(C)                                                    \
  case C:                                                                     \
    if (mode == MODE_LSE) return launch_rows_t<C, MODE_LSE>(a, B, st);        \
    if (mode == MODE_ARGMAX) return launch_rows_t<C, MODE_ARGMAX>(a, B, st);  \
    return launch_rows_t<C, MODE_RESP>(a, B, st);
  switch (cov) {
    GMMXX_ROWS_CASE(GMMXX_SPHERICAL)
    GMMXX_ROWS_CASE(GMMXX_DIAG)
    GMMXX_ROWS_CASE(GMMXX_TIED)
    GMMXX_ROWS_CASE(GMMXX_FULL)
  }
#undef GMMXX_ROWS_CASE
  return set_error(GMMXX_ERR_INVALID, "bad covariance type %d", cov);
}

template <int COV, int NCH>
static int launch_mstep_t(RowArgs& a, int B, cudaStream_t st) {
  const int64_t sm = smem_bytes(COV, a.D, true);
  auto k = mstep_kernel<COV, NCH>;
  if (int rc = prep_smem(k, sm)) return rc;
  const int ktiles = (int)(a.Kp / kBK);
  const int64_t tiles = ceil_div(a.N, kBN);
  const int64_t nblk_max = mstep_blocks(B, a.N, a.Kp);  // partial slots reserved in the workspace
  a.rows_per_cta = ceil_div(tiles, wave_blocks(k, sm, ktiles, B, nblk_max, tiles)) * kBN;
  const int64_t nblk = ceil_div(a.N, a.rows_per_cta);
  a.part_blocks = nblk_max;
  dim3 grid((unsigned)nblk, (unsigned)ktiles, (unsigned)B);
  k<<<grid, kThreads, sm, st>>>(a);
  return check_launch("mstep_kernel");
}

template <int COV>
static int launch_mstep_c(RowArgs& a, int B, cudaStream_t st) {
  const int nch = (int)ceil_div(a.FM - 1, 64);  // n_k is a column sum of R, outside the chunks
  switch (nch) {
    case 1: return launch_mstep_t<COV, 1>(a, B, st);
    case 2: return launch_mstep_t<COV, 2>(a, B, st);
    case 3: return launch_mstep_t<COV, 3>(a, B, st);
    case 4: return launch_mstep_t<COV, 4>(a, B, st);
    case 5: return launch_mstep_t<COV, 5>(a, B, st);
    case 6: return launch_mstep_t<COV, 6>(a, B, st);
  }
  return set_error(GMMXX_ERR_UNSUPPORTED, "statistics width %d exceeds the SIMT window", a.FM);
}

int launch_mstep(int cov, RowArgs& a, int B, cudaStream_t st) {
  if (a.N == 0) return GMMXX_OK;
  switch (cov) {
    case GMMXX_SPHERICAL: return launch_mstep_c<GMMXX_SPHERICAL>(a, B, st);
    case GMMXX_DIAG: return launch_mstep_c<GMMXX_DIAG>(a, B, st);
    case GMMXX_TIED: return launch_mstep_c<GMMXX_TIED>(a, B, st);
    case GMMXX_FULL: return launch_mstep_c<GMMXX_FULL>(a, B, st);
  }
  return set_error(GMMXX_ERR_INVALID, "bad covariance type %d", cov);
}

template <int COV, int NCH>
static int launch_small_t(RowArgs a, int B, cudaStream_t st) {
  const int64_t sm = smem_bytes(COV, a.D, true);
  auto k = em_small_kernel<COV, NCH>;
  if (int rc = prep_smem(k, sm)) return rc;
  const int64_t tiles = ceil_div(a.N, kBN);
  const int64_t nblk_max = mstep_blocks(B, a.N, a.Kp);
  a.rows_per_cta = ceil_div(tiles, wave_blocks(k, sm, 1, B, nblk_max, tiles)) * kBN;
  const int64_t nblk = ceil_div(a.N, a.rows_per_cta);
  a.part_blocks = nblk_max;
  dim3 grid((unsigned)nblk, 1u, (unsigned)B);
  k<<<grid, kThreads, sm, st>>>(a);
  if (int rc = check_launch("em_small_kernel")) return rc;
  // statistics: the first nblk of nblk_max slots; log-likelihood: nblk per problem, packed
  const int64_t n = (int64_t)B * a.K * a.FM;
  stats_reduce_kernel<<<(unsigned)ceil_div(std::max<int64_t>(n, 1), 256), 256, 0, st>>>(
      a.part, nblk, nblk_max, a.Kp, a.K, a.FM, B, a.stats, a.ll_part, nblk, a.ll);
  return check_launch("stats_reduce_kernel");
}

template <int COV>
static int launch_small_c(const RowArgs& a, int B, cudaStream_t st) {
  switch ((int)ceil_div(a.FM - 1, 64)) {  // n_k is a column sum of R, outside the chunks
    case 1: return launch_small_t<COV, 1>(a, B, st);
    case 2: return launch_small_t<COV, 2>(a, B, st);
    case 3: return launch_small_t<COV, 3>(a, B, st);
    case 4: return launch_small_t<COV, 4>(a, B, st);
    case 5: return launch_small_t<COV, 5>(a, B, st);
    case 6: return launch_small_t<COV, 6>(a, B, st);
  }
  return set_error(GMMXX_ERR_UNSUPPORTED, "statistics width %d exceeds the SIMT window", a.FM);
}

template <int NCH>
static int launch_small_narrow_t(RowArgs a, int B, cudaStream_t st) {
  const int64_t sm = smem_bytes_narrow(a.D);
  auto k = em_small_narrow_kernel<NCH>;
  if (int rc = prep_smem(k, sm)) return rc;
  const int64_t tiles = ceil_div(a.N, kNR);
  const int64_t nblk_max = mstep_blocks(B, a.N, a.Kp);
  a.rows_per_cta = ceil_div(tiles, wave_blocks(k, sm, 1, B, nblk_max, tiles)) * kNR;
  const int64_t nblk = ceil_div(a.N, a.rows_per_cta);
  a.part_blocks = nblk_max;
  dim3 grid((unsigned)nblk, 1u, (unsigned)B);
  k<<<grid, kThreads, sm, st>>>(a);
  if (int rc = check_launch("em_small_narrow_kernel")) return rc;
  const int64_t n = (int64_t)B * a.K * a.FM;
  stats_reduce_kernel<<<(unsigned)ceil_div(std::max<int64_t>(n, 1), 256), 256, 0, st>>>(
      a.part, nblk, nblk_max, a.Kp, a.K, a.FM, B, a.stats, a.ll_part, nblk, a.ll);
  return check_launch("stats_reduce_kernel");
}

// GMMXX_B200_SMALL_TILE=wide keeps full covariance with K <= 32 on the 64 x 64
// tile (the A/B switch of the two tilings)
static bool narrow_enabled() {
  const char* e = getenv("GMMXX_B200_SMALL_TILE");
  return !(e != nullptr && strcmp(e, "wide") == 0);
}

int launch_em_small(int cov, const RowArgs& a, int B, cudaStream_t st) {
  if (a.N == 0) return GMMXX_OK;
  if (a.Kp != kBK) return set_error(GMMXX_ERR_UNSUPPORTED, "one-pass statistics need K <= %d", kBK);
  if (cov == GMMXX_FULL && a.K <= kNK && narrow_enabled()) {
    switch ((int)ceil_div(a.FM - 1, 64)) {
      case 1: return launch_small_narrow_t<1>(a, B, st);
      case 2: return launch_small_narrow_t<2>(a, B, st);
      case 3: return launch_small_narrow_t<3>(a, B, st);
      default: break;  // wider statistics: the 64 x 64 tile
    }
  }
  switch (cov) {
    case GMMXX_SPHERICAL: return launch_small_c<GMMXX_SPHERICAL>(a, B, st);
    case GMMXX_DIAG: return launch_small_c<GMMXX_DIAG>(a, B, st);
    case GMMXX_TIED: return launch_small_c<GMMXX_TIED>(a, B, st);
    case GMMXX_FULL: return launch_small_c<GMMXX_FULL>(a, B, st);
  }
  return set_error(GMMXX_ERR_INVALID, "bad covariance type %d", cov);
}

template <int COV>
static int launch_topk_rows_t(const RowArgs& a, int B, cudaStream_t st) {
  const int64_t sm = topk_rows_smem(COV, a.D, a.top_k);
  auto k = topk_rows_kernel<COV>;
  if (int rc = prep_smem(k, sm)) return rc;
  dim3 grid((unsigned)ceil_div(a.N, kBN), (unsigned)B);  // the LSE pass's grid: same partial layout
  k<<<grid, kThreads, sm, st>>>(a);
  return check_launch("topk_rows_kernel");
}

int launch_topk_rows(int cov, const RowArgs& a, int B, cudaStream_t st) {
  if (a.N == 0) return GMMXX_OK;
  if (a.top_k < 1 || a.top_k > kMaxTopK || a.top_k >= a.K)
    return set_error(GMMXX_ERR_INVALID, "top_k=%d outside [1, min(K - 1, %d)]", a.top_k, kMaxTopK);
  switch (cov) {
    case GMMXX_SPHERICAL: return launch_topk_rows_t<GMMXX_SPHERICAL>(a, B, st);
    case GMMXX_DIAG: return launch_topk_rows_t<GMMXX_DIAG>(a, B, st);
    case GMMXX_TIED: return launch_topk_rows_t<GMMXX_TIED>(a, B, st);
    case GMMXX_FULL: return launch_topk_rows_t<GMMXX_FULL>(a, B, st);
  }
  return set_error(GMMXX_ERR_INVALID, "bad covariance type %d", cov);
}

template <int COV, int NCH>
static int launch_topk_mstep_t(RowArgs& a, int B, cudaStream_t st) {
  const int64_t sm = smem_bytes(COV, a.D, true);
  auto k = topk_mstep_kernel<COV, NCH>;
  if (int rc = prep_smem(k, sm)) return rc;
  const int ktiles = (int)(a.Kp / kBK);
  const int64_t tiles = ceil_div(a.N, kBN);
  const int64_t nblk_max = mstep_blocks(B, a.N, a.Kp);
  a.rows_per_cta = ceil_div(tiles, wave_blocks(k, sm, ktiles, B, nblk_max, tiles)) * kBN;
  const int64_t nblk = ceil_div(a.N, a.rows_per_cta);
  a.part_blocks = nblk_max;
  dim3 grid((unsigned)nblk, (unsigned)ktiles, (unsigned)B);
  k<<<grid, kThreads, sm, st>>>(a);
  return check_launch("topk_mstep_kernel");
}

template <int COV>
static int launch_topk_mstep_c(RowArgs& a, int B, cudaStream_t st) {
  switch ((int)ceil_div(a.FM - 1, 64)) {  // n_k is a column sum of R, outside the chunks
    case 1: return launch_topk_mstep_t<COV, 1>(a, B, st);
    case 2: return launch_topk_mstep_t<COV, 2>(a, B, st);
    case 3: return launch_topk_mstep_t<COV, 3>(a, B, st);
    case 4: return launch_topk_mstep_t<COV, 4>(a, B, st);
    case 5: return launch_topk_mstep_t<COV, 5>(a, B, st);
    case 6: return launch_topk_mstep_t<COV, 6>(a, B, st);
  }
  return set_error(GMMXX_ERR_UNSUPPORTED, "statistics width %d exceeds the SIMT window", a.FM);
}

int launch_topk_mstep(int cov, RowArgs& a, int B, cudaStream_t st) {
  if (a.N == 0) return GMMXX_OK;
  switch (cov) {
    case GMMXX_SPHERICAL: return launch_topk_mstep_c<GMMXX_SPHERICAL>(a, B, st);
    case GMMXX_DIAG: return launch_topk_mstep_c<GMMXX_DIAG>(a, B, st);
    case GMMXX_TIED: return launch_topk_mstep_c<GMMXX_TIED>(a, B, st);
    case GMMXX_FULL: return launch_topk_mstep_c<GMMXX_FULL>(a, B, st);
  }
  return set_error(GMMXX_ERR_INVALID, "bad covariance type %d", cov);
}

int launch_stats_reduce(const RowArgs& a, int B, cudaStream_t st) {
  if (a.N == 0) return GMMXX_OK;
  const int64_t tiles = ceil_div(a.N, kBN);
  const int64_t nblk_max = mstep_blocks(B, a.N, a.Kp);
  // slots the M-step filled (launch_mstep recorded its rows per CTA)
  const int64_t rpc = a.rows_per_cta > 0 ? a.rows_per_cta : ceil_div(tiles, nblk_max) * kBN;
  const int64_t nblk = ceil_div(a.N, rpc);
  const int64_t n = (int64_t)B * a.K * a.FM;
  // partial slots are strided by nblk_max; only the first nblk are written
  stats_reduce_kernel<<<(unsigned)ceil_div(std::max<int64_t>(n, 1), 256), 256, 0, st>>>(
      a.part, nblk, nblk_max, a.Kp, a.K, a.FM, B, a.stats, a.ll_part, tiles, a.ll);
  return check_launch("stats_reduce_kernel");
}

int launch_xx_total(const void* x, int dt, int64_t B, int64_t N, int D, float* xx, float* part, cudaStream_t st) {
  if (N == 0) return GMMXX_OK;
  const int64_t sm = (int64_t)kBN * (D + 1) * 4;
  if (int rc = prep_smem(xx_total_kernel, sm)) return rc;
  const int64_t tiles = ceil_div(N, kBN);
  const int64_t nmax = xx_blocks(B, N);
  const int64_t rpc = ceil_div(tiles, nmax) * kBN;
  const int64_t nblk = ceil_div(N, rpc);
  // partial slots of problem b start at (b * nblk) and are packed, so the
  // reduction below uses stride nblk
  dim3 grid((unsigned)nblk, (unsigned)B);
  xx_total_kernel<<<grid, kThreads, sm, st>>>(x, dt, N, D, rpc, part);
  if (int rc = check_launch("xx_total_kernel")) return rc;
  const int64_t n = B * (int64_t)D * D;
  stats_reduce_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(part, nblk, nblk, D, D, D, (int)B, xx, nullptr, 0,
                                                                  nullptr);
  return check_launch("stats_reduce_kernel");
}

}  // namespace gmmxx
