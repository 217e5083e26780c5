// vmscan_conv.cuh — depthwise causal conv1d along a scan direction, fused
// with SiLU, and its VJP.
//
// Reference: MambaBlock applies `nn.Conv1d(d_inner, d_inner, kernel_size=K,
// padding=K-1, groups=d_inner)` to the (possibly permuted / reversed)
// sequence, keeps the first L outputs and applies SiLU
// (mlx_vision_mamba/mamba_block.py:129-132,170-171; permutations :443-534):
//   out[p] = silu(bias + sum_{k<K} w[c, k] * x[p - K + 1 + k])   (zero for p-K+1+k < 0)
// where p runs over scan positions.  Here p is mapped to its token through the
// direction, so the permuted copy of the reference never exists.
//
// Layout: a CTA covers CONV_THREADS float4 channel groups x CONV_CHUNK scan
// positions of one batch row; the tokens of those positions are computed
// once into shared memory; every thread slides a register window along the
// chunk, so each x element is read once (plus a K-1 halo per chunk).  The
// loads of CONV_FWD_U (forward) / CONV_BWD_U (VJP) positions are issued
// together ahead of their use, so each thread keeps that many HBM reads in
// flight instead of one.
#pragma once

#include "vmscan_common.cuh"

namespace vmscan {

constexpr int CONV_CHUNK = 32;
constexpr int CONV_KMAX = 8;
constexpr int CONV_THREADS = 64;  // float4 channel groups per CTA (768 and 1536 channels fill whole CTAs)
constexpr int CONV_RGROUPS = 16;  // row groups of the first dw/dbias reduction level
// Loads issued together, measured on (64, 196, 768): forward 8 positions
// (16: slower), VJP 4 (8 or 16: slower; 164 registers already limit the VJP
// to 6 CTAs per SM).
constexpr int CONV_FWD_U = 8;  // positions whose x loads are issued together (forward)
constexpr int CONV_BWD_U = 4;  // positions whose x and dout loads are issued together (VJP)

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ void fma4(float4& a, float w, const float4& x) {
  a.x = fmaf(w, x.x, a.x);
  a.y = fmaf(w, x.y, a.y);
  a.z = fmaf(w, x.z, a.z);
  a.w = fmaf(w, x.w, a.w);
}

__device__ __forceinline__ float dsilu_f(float pre) {
  const float sig = __fdividef(1.0f, 1.0f + ex2_approx(-kLog2e * pre));
  return sig * fmaf(pre, 1.0f - sig, 1.0f);
}

// Window KW (4 or 8) >= K; the K real taps sit at the newest end of the window.
template <int KW, bool SPLIT>
__global__ void __launch_bounds__(CONV_THREADS)
    conv_silu_fwd_kernel(const float* __restrict__ x, int64_t sxb, int64_t sxs, const float* __restrict__ w,
                         const float* __restrict__ bias, float* __restrict__ out, int64_t sob, int64_t sos,
                         float* __restrict__ out_hi, float* __restrict__ out_lo, int C, int K, const ScanGeom g) {
  __shared__ int64_t tok[CONV_CHUNK + CONV_KMAX];
  const int p0 = blockIdx.y * CONV_CHUNK;
  const int b = blockIdx.z;
  const int L = g.seqlen;
  const int span = CONV_CHUNK + K - 1;
  for (int t = threadIdx.x; t < span; t += blockDim.x) {
    const int p = p0 - (K - 1) + t;
    tok[t] = (p >= 0 && p < L) ? scan_pos_token(g, p) : int64_t(-1);
  }
  __syncthreads();
  const int c4 = blockIdx.x * CONV_THREADS + threadIdx.x;
  if (c4 * 4 >= C) return;
  float wv[KW][4];
#pragma unroll
  for (int m = 0; m < KW; ++m) {
    const int k = m - (KW - K);  // tap index of window slot m
#pragma unroll
    for (int q = 0; q < 4; ++q) wv[m][q] = (k >= 0) ? w[size_t(c4 * 4 + q) * K + k] : 0.f;
  }
  const float4 bv = ldg4(bias + c4 * 4);
  float4 win[KW];
#pragma unroll
  for (int m = 0; m < KW; ++m) win[m] = make_float4(0.f, 0.f, 0.f, 0.f);
  const float* xb = x + b * sxb + c4 * 4;
  float* ob = out + b * sob + c4 * 4;
  for (int t0 = 0; t0 < span; t0 += CONV_FWD_U) {
    float4 xs[CONV_FWD_U];
#pragma unroll
    for (int u = 0; u < CONV_FWD_U; ++u) {
      const int64_t tk = (t0 + u < span) ? tok[t0 + u] : int64_t(-1);
      xs[u] = (tk >= 0) ? ldg4(xb + tk * sxs) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < CONV_FWD_U; ++u) {
      const int t = t0 + u;
      if (t < span) {
        const int64_t tk = tok[t];
#pragma unroll
        for (int m = 0; m < KW - 1; ++m) win[m] = win[m + 1];
        win[KW - 1] = xs[u];
        if (t >= K - 1 && tk >= 0) {
          float4 acc = bv;
#pragma unroll
          for (int m = 0; m < KW; ++m) {
            acc.x = fmaf(wv[m][0], win[m].x, acc.x);
            acc.y = fmaf(wv[m][1], win[m].y, acc.y);
            acc.z = fmaf(wv[m][2], win[m].z, acc.z);
            acc.w = fmaf(wv[m][3], win[m].w, acc.w);
          }
          float4 o;
          o.x = silu_f(acc.x);
          o.y = silu_f(acc.y);
          o.z = silu_f(acc.z);
          o.w = silu_f(acc.w);
          *reinterpret_cast<float4*>(ob + tk * sos) = o;
          if constexpr (SPLIT) {
            // TF32 parts for the x_proj GEMM, same layout as out (a separate
            // instantiation: the plain path carries no per-position test)
            float4 hi, lo;
            split_tf32_4(o, hi, lo);
            const int64_t off = b * sob + c4 * 4 + tk * sos;
            *reinterpret_cast<float4*>(out_hi + off) = hi;
            *reinterpret_cast<float4*>(out_lo + off) = lo;
          }
        }
      }
    }
  }
}

// VJP.  For the chunk [p0, p0+CHUNK) it recomputes the pre-activation on
// [p0, p0+CHUNK+K-1), forms dpre = dout * silu'(pre), emits
//   dx[p'] = sum_k w[k] dpre[p' + K - 1 - k]
// and per-thread partial sums of dw[k] = sum_p dpre[p] x[p-K+1+k] and
// dbias = sum_p dpre[p] over the chunk, written slot-major to
// wpart[b][chunk][slot][c] (slot k < K: dw[k], slot KMAX: dbias) as float4.
template <int KW, bool SPLIT>
__global__ void __launch_bounds__(CONV_THREADS)
    conv_silu_bwd_kernel(const float* __restrict__ x, int64_t sxb, int64_t sxs, const float* __restrict__ w,
                         const float* __restrict__ bias, const float* __restrict__ dout, int64_t sdb, int64_t sds,
                         float* __restrict__ dx, int64_t sxgb, int64_t sxgs, float* __restrict__ dx_lo,
                         float* __restrict__ wpart, int C, int K, const ScanGeom g) {
  __shared__ int64_t tok[CONV_CHUNK + 2 * CONV_KMAX];
  const int p0 = blockIdx.y * CONV_CHUNK;
  const int nchunk = gridDim.y;
  const int b = blockIdx.z;
  const int L = g.seqlen;
  const int span = CONV_CHUNK + 2 * K - 2;
  for (int t = threadIdx.x; t < span; t += blockDim.x) {
    const int p = p0 - (K - 1) + t;
    tok[t] = (p >= 0 && p < L) ? scan_pos_token(g, p) : int64_t(-1);
  }
  __syncthreads();
  const int c4 = blockIdx.x * CONV_THREADS + threadIdx.x;
  if (c4 * 4 >= C) return;
  float wv[KW][4];
#pragma unroll
  for (int m = 0; m < KW; ++m) {
    const int k = m - (KW - K);
#pragma unroll
    for (int q = 0; q < 4; ++q) wv[m][q] = (k >= 0) ? w[size_t(c4 * 4 + q) * K + k] : 0.f;
  }
  // wr[j] multiplies dpre window slot j (tap KW - 1 - j; zero past K), so the
  // dx sum below indexes registers with compile-time slots only
  float wr[KW][4];
#pragma unroll
  for (int j = 0; j < KW; ++j) {
    const int k = KW - 1 - j;
#pragma unroll
    for (int q = 0; q < 4; ++q) wr[j][q] = (k < K) ? w[size_t(c4 * 4 + q) * K + k] : 0.f;
  }
  const float4 bv = ldg4(bias + c4 * 4);
  float4 xw[KW], dw_acc[KW], dpw[KW];
#pragma unroll
  for (int m = 0; m < KW; ++m) {
    xw[m] = make_float4(0.f, 0.f, 0.f, 0.f);
    dw_acc[m] = make_float4(0.f, 0.f, 0.f, 0.f);
    dpw[m] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float4 db_acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const float* xb = x + b * sxb + c4 * 4;
  const float* gb = dout + b * sdb + c4 * 4;
  float* dxb = dx + b * sxgb + c4 * 4;
  for (int t0 = 0; t0 < span; t0 += CONV_BWD_U) {
    float4 xs[CONV_BWD_U], gs[CONV_BWD_U];
#pragma unroll
    for (int u = 0; u < CONV_BWD_U; ++u) {
      const int64_t tk = (t0 + u < span) ? tok[t0 + u] : int64_t(-1);
      xs[u] = (tk >= 0) ? ldg4(xb + tk * sxs) : make_float4(0.f, 0.f, 0.f, 0.f);
      gs[u] = (tk >= 0 && t0 + u >= K - 1) ? ldg4(gb + tk * sds) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < CONV_BWD_U; ++u) {
      const int t = t0 + u;
      if (t < span) {
        const int p = p0 - (K - 1) + t;
        const int64_t tk = tok[t];
#pragma unroll
        for (int m = 0; m < KW - 1; ++m) xw[m] = xw[m + 1];
        xw[KW - 1] = xs[u];
        float4 dp = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p >= p0 && tk >= 0) {
          float4 pre = bv;
#pragma unroll
          for (int m = 0; m < KW; ++m) {
            pre.x = fmaf(wv[m][0], xw[m].x, pre.x);
            pre.y = fmaf(wv[m][1], xw[m].y, pre.y);
            pre.z = fmaf(wv[m][2], xw[m].z, pre.z);
            pre.w = fmaf(wv[m][3], xw[m].w, pre.w);
          }
          const float4 go = gs[u];
          dp.x = go.x * dsilu_f(pre.x);
          dp.y = go.y * dsilu_f(pre.y);
          dp.z = go.z * dsilu_f(pre.z);
          dp.w = go.w * dsilu_f(pre.w);
          if (p < p0 + CONV_CHUNK) {
#pragma unroll
            for (int m = 0; m < KW; ++m) {
              dw_acc[m].x = fmaf(dp.x, xw[m].x, dw_acc[m].x);
              dw_acc[m].y = fmaf(dp.y, xw[m].y, dw_acc[m].y);
              dw_acc[m].z = fmaf(dp.z, xw[m].z, dw_acc[m].z);
              dw_acc[m].w = fmaf(dp.w, xw[m].w, dw_acc[m].w);
            }
            db_acc.x += dp.x;
            db_acc.y += dp.y;
            db_acc.z += dp.z;
            db_acc.w += dp.w;
          }
        }
#pragma unroll
        for (int m = 0; m < KW - 1; ++m) dpw[m] = dpw[m + 1];
        dpw[KW - 1] = dp;
        // dx at p' = p - (K - 1): taps k read dpre[p - k] = dpw[KW - 1 - k]
        const int pp = p - (K - 1);
        if (pp >= p0 && pp < p0 + CONV_CHUNK && pp < L) {
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          // taps k = 0 .. K-1 in order: slot j = KW - 1 - k
#pragma unroll
          for (int j = KW - 1; j >= 0; --j) {
            acc.x = fmaf(wr[j][0], dpw[j].x, acc.x);
            acc.y = fmaf(wr[j][1], dpw[j].y, acc.y);
            acc.z = fmaf(wr[j][2], dpw[j].z, acc.z);
            acc.w = fmaf(wr[j][3], dpw[j].w, acc.w);
          }
          const int64_t tkp = tok[t - (K - 1)];
          if constexpr (SPLIT) {
            // the TF32 parts of dx (for the in_proj gradient GEMMs) instead of dx
            // (a separate instantiation: the plain path carries no per-position test)
            float4 hi, lo;
            split_tf32_4(acc, hi, lo);
            *reinterpret_cast<float4*>(dxb + tkp * sxgs) = hi;
            *reinterpret_cast<float4*>(dx_lo + b * sxgb + c4 * 4 + tkp * sxgs) = lo;
          } else {
            *reinterpret_cast<float4*>(dxb + tkp * sxgs) = acc;
          }
        }
      }
    }
  }
  // partials: slot k < K holds dw[k] (window slot KW-K+k), slot CONV_KMAX holds dbias
  float* wp = wpart + (size_t(b) * nchunk + blockIdx.y) * (CONV_KMAX + 1) * C + c4 * 4;
  // window slot m holds tap k = m - (KW - K); compile-time slots keep dw_acc in registers
#pragma unroll
  for (int m = 0; m < KW; ++m) {
    const int k = m - (KW - K);
    if (k >= 0) *reinterpret_cast<float4*>(wp + size_t(k) * C) = dw_acc[m];
  }
  *reinterpret_cast<float4*>(wp + size_t(CONV_KMAX) * C) = db_acc;
}

// dweight (C, K) and dbias (C) from the (batch, chunk) partials, in two
// fixed-order levels: conv_reduce_kernel sums row group blockIdx.y (rows
// r = y, y + G, ...) of every (slot, channel) column into gpart[y]; then
// conv_reduce2_kernel sums the G group partials in order.  Columns are
// contiguous in the slot-major layout, so every load is coalesced.
// Rows are loaded CONV_RED_U at a time before they are added (in row order),
// so a thread keeps that many reads in flight.
constexpr int CONV_RED_U = 8;

__global__ void conv_reduce_kernel(const float* __restrict__ wpart, float* __restrict__ gpart, int nrows, int C,
                                   int K) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;  // slot * C + c over the K + 1 used slots
  if (col >= (K + 1) * C) return;
  const int sl = col / C, c = col % C;
  const int slot = sl < K ? sl : CONV_KMAX;
  const size_t stride = size_t(CONV_KMAX + 1) * C;
  const float* src = wpart + size_t(slot) * C + c;
  const int G = gridDim.y;
  float acc = 0.f;
  for (int r0 = blockIdx.y; r0 < nrows; r0 += CONV_RED_U * G) {
    float v[CONV_RED_U];
#pragma unroll
    for (int u = 0; u < CONV_RED_U; ++u) {
      const int r = r0 + u * G;
      v[u] = r < nrows ? src[size_t(r) * stride] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < CONV_RED_U; ++u) acc += v[u];
  }
  gpart[size_t(blockIdx.y) * (K + 1) * C + col] = acc;
}

__global__ void conv_reduce2_kernel(const float* __restrict__ gpart, float* __restrict__ dw, float* __restrict__ db,
                                    int ngroups, int C, int K) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= (K + 1) * C) return;
  float acc = 0.f;
  for (int g0 = 0; g0 < ngroups; g0 += CONV_RED_U) {
    float v[CONV_RED_U];
#pragma unroll
    for (int u = 0; u < CONV_RED_U; ++u)
      v[u] = g0 + u < ngroups ? gpart[size_t(g0 + u) * (K + 1) * C + col] : 0.f;
#pragma unroll
    for (int u = 0; u < CONV_RED_U; ++u) acc += v[u];
  }
  const int sl = col / C, c = col % C;
  if (sl < K)
    dw[size_t(c) * K + sl] = acc;
  else
    db[c] = acc;
}

}  // namespace vmscan
