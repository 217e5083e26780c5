// vmscan_norm.cuh — LayerNorm over the last dimension, forward and VJP, for
// the residual blocks and the encoder's final norm (MLX nn.LayerNorm in the
// reference: mamba_block.py:201,222,401, vision_mamba.py:192; eps 1e-5, affine).
//
//   y = (x - mean) * rstd * w + b,   rstd = 1 / sqrt(var + eps),
//   var the biased variance over the row.
//   VJP, with xhat = (x - mean) rstd and g = dy w:
//   dx = rstd (g - mean(g) - xhat mean(g xhat)),  dw = sum_rows dy xhat,
//   db = sum_rows dy.
//
// One warp per row: lane l holds the row's float4 chunks l, l + 32, ...
// (NC chunks per lane, dim % 4 == 0, dim <= 1024), so the sums over the row
// are warp shuffles and every access is a coalesced 16-byte load or store.
// The VJP kernel writes one dw / db partial row per CTA (its warps' rows
// summed in warp order); sum_rows_kernel (vmscan_dt.cuh) adds those rows in a
// fixed order, so dw and db are deterministic.
#pragma once

#include "vmscan_common.cuh"

namespace vmscan {

constexpr int LN_WARPS = 8;           // warps per CTA
constexpr int LN_ROWS_PER_WARP = 2;   // rows a VJP warp handles (loads of both in flight together)
constexpr int LN_MAX_DIM = 1024;      // NC <= 8 chunks of 4 per lane

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

template <int NC>
__global__ void __launch_bounds__(LN_WARPS * 32)
    layernorm_fwd_kernel(const float* __restrict__ x, int64_t ldx, const float* __restrict__ w,
                         const float* __restrict__ b, float eps, float* __restrict__ y, int64_t ldy,
                         float* __restrict__ mean_out, float* __restrict__ rstd_out, int rows, int dim) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * LN_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nq = dim >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + int64_t(row) * ldx);
  float4 v[NC];
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int q = lane + 32 * c;
    v[c] = q < nq ? xr[q] : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (v[c].x + v[c].y) + (v[c].z + v[c].w);
  }
  const float mean = warp_sum(s) / float(dim);
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    if (lane + 32 * c < nq) {
      const float a0 = v[c].x - mean, a1 = v[c].y - mean, a2 = v[c].z - mean, a3 = v[c].w - mean;
      ss += (a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3);
    }
  }
  const float rstd = 1.0f / sqrtf(warp_sum(ss) / float(dim) + eps);
  float4* yr = reinterpret_cast<float4*>(y + int64_t(row) * ldy);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int q = lane + 32 * c;
    if (q < nq) {
      const float4 wv = w4[q], bv = b4[q];
      float4 o;
      o.x = fmaf((v[c].x - mean) * rstd, wv.x, bv.x);
      o.y = fmaf((v[c].y - mean) * rstd, wv.y, bv.y);
      o.z = fmaf((v[c].z - mean) * rstd, wv.z, bv.z);
      o.w = fmaf((v[c].w - mean) * rstd, wv.w, bv.w);
      yr[q] = o;
    }
  }
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// VJP: CTA blk handles rows [blk * R, (blk + 1) * R), R = LN_WARPS *
// LN_ROWS_PER_WARP, warp w rows blk * R + w * LN_ROWS_PER_WARP + i.  part:
// (gridDim.x, 2 dim) row-major, dw partials then db partials.  Dynamic shared
// memory: LN_WARPS * 2 * dim floats.
template <int NC>
__global__ void __launch_bounds__(LN_WARPS * 32)
    layernorm_bwd_kernel(const float* __restrict__ x, int64_t ldx, const float* __restrict__ w,
                         const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                         const float* __restrict__ dy, int64_t lddy, float* __restrict__ dx, int64_t lddx,
                         float* __restrict__ part, int rows, int dim) {
  extern __shared__ float ln_sm[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nq = dim >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4 wv[NC], dwa[NC], dba[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int q = lane + 32 * c;
    wv[c] = q < nq ? w4[q] : make_float4(0.f, 0.f, 0.f, 0.f);
    dwa[c] = dba[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float inv_dim = 1.0f / float(dim);
  const int row0 = (blockIdx.x * LN_WARPS + warp) * LN_ROWS_PER_WARP;
  // the warp's rows in pairs, both rows' loads issued before either is used
  for (int i = 0; i < LN_ROWS_PER_WARP; i += 2) {
    float4 xv[2][NC], dv[2][NC];
    float mean[2], rstd[2];
    bool live[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = row0 + i + h;
      live[h] = row < rows;
      mean[h] = live[h] ? mean_in[row] : 0.f;
      rstd[h] = live[h] ? rstd_in[row] : 0.f;
      const float4* xr = reinterpret_cast<const float4*>(x + int64_t(live[h] ? row : 0) * ldx);
      const float4* gr = reinterpret_cast<const float4*>(dy + int64_t(live[h] ? row : 0) * lddy);
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int q = lane + 32 * c;
        const bool ok = live[h] && q < nq;
        xv[h][c] = ok ? xr[q] : make_float4(0.f, 0.f, 0.f, 0.f);
        dv[h][c] = ok ? gr[q] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (!live[h]) break;  // warp-uniform: the row index does not depend on the lane
      const int row = row0 + i + h;
      float4 xh[NC], g[NC];
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const float4 a = xv[h][c], d = dv[h][c];
        const float m = mean[h], r = rstd[h];
        // chunks past the row end are zero in x and dy: their terms vanish
        xh[c] = lane + 32 * c < nq ? make_float4((a.x - m) * r, (a.y - m) * r, (a.z - m) * r, (a.w - m) * r)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
        g[c] = make_float4(d.x * wv[c].x, d.y * wv[c].y, d.z * wv[c].z, d.w * wv[c].w);
        s1 += (g[c].x + g[c].y) + (g[c].z + g[c].w);
        s2 += (g[c].x * xh[c].x + g[c].y * xh[c].y) + (g[c].z * xh[c].z + g[c].w * xh[c].w);
        dwa[c].x = fmaf(d.x, xh[c].x, dwa[c].x);
        dwa[c].y = fmaf(d.y, xh[c].y, dwa[c].y);
        dwa[c].z = fmaf(d.z, xh[c].z, dwa[c].z);
        dwa[c].w = fmaf(d.w, xh[c].w, dwa[c].w);
        dba[c].x += d.x;
        dba[c].y += d.y;
        dba[c].z += d.z;
        dba[c].w += d.w;
      }
      const float m1 = warp_sum(s1) * inv_dim, m2 = warp_sum(s2) * inv_dim;
      const float r = rstd[h];
      float4* dxr = reinterpret_cast<float4*>(dx + int64_t(row) * lddx);
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int q = lane + 32 * c;
        if (q < nq) {
          float4 o;
          o.x = r * (g[c].x - m1 - xh[c].x * m2);
          o.y = r * (g[c].y - m1 - xh[c].y * m2);
          o.z = r * (g[c].z - m1 - xh[c].z * m2);
          o.w = r * (g[c].w - m1 - xh[c].w * m2);
          dxr[q] = o;
        }
      }
    }
  }
  // the CTA's partial rows: its warps' sums added in warp order
  float4* sw = reinterpret_cast<float4*>(ln_sm);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int q = lane + 32 * c;
    if (q < nq) {
      sw[warp * 2 * nq + q] = dwa[c];
      sw[warp * 2 * nq + nq + q] = dba[c];
    }
  }
  __syncthreads();
  float4* pr = reinterpret_cast<float4*>(part + int64_t(blockIdx.x) * 2 * dim);
  for (int q = threadIdx.x; q < 2 * nq; q += LN_WARPS * 32) {
    float4 acc = sw[q];
    for (int k = 1; k < LN_WARPS; ++k) {
      const float4 t = sw[k * 2 * nq + q];
      acc.x += t.x;
      acc.y += t.y;
      acc.z += t.z;
      acc.w += t.w;
    }
    pr[q] = acc;
  }
}

}  // namespace vmscan
