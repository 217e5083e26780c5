// vmscan_dt.cuh — dt_proj + bias + softplus producing the scan's delta, and
// the softplus part of its VJP.
//
// Reference (mlx_vision_mamba/mamba_block.py:177-181): dt = x_dbc[..., :dt_rank],
// delta = dt_proj(dt) with dt_proj = nn.Linear(dt_rank, d_inner, bias=True),
// then delta = log(1 + exp(delta)).  Per token t and channel d:
//   pre[t, d]   = bias[d] + sum_r x[t, r] W[d, r]
//   delta[t, d] = log(1 + exp(pre[t, d]))
//   dpre[t, d]  = ddelta[t, d] * sigmoid(pre[t, d])      (VJP; pre recomputed)
// The remaining gradients (dx = dpre W, dW = dpre^T x, dbias = column sums of
// dpre) are plain GEMMs / reductions done by the caller.
//
// Layout: a CTA owns DTP_THREADS x (1 or 2) channels x DTP_TOKENS tokens;
// the tokens' x rows (dt_rank floats, zero-padded to RP) are staged once in
// shared memory (transposed) and read as broadcasts; each thread keeps its
// channels' weight rows in registers and forms 4 tokens' dot products as two
// packed pairs per channel, so a token costs dt_rank / 2 packed FMAs per
// channel and no global loads.  delta / dpre rows are written coalesced
// (consecutive channels per warp).
#pragma once

#include "vmscan_common.cuh"

namespace vmscan {

constexpr int DTP_THREADS = 128;
constexpr int DTP_TOKENS = 64;
constexpr int DTP_RMAX = 64;
constexpr int DTP_U = 4;  // tokens per iteration (two packed pairs)
static_assert(DTP_TOKENS % DTP_U == 0, "xs holds whole token groups");

// Channels per thread for a rank bucket: two (d and d + DTP_THREADS, so each
// shared-memory load of x feeds both) while both weight rows fit in registers.
__host__ __device__ constexpr int dtp_channels(int RP) { return RP <= 32 ? 2 : 1; }

// log(1 + exp(v)), the reference's own expression (inf for v beyond expf's
// range, like the reference), on the MUFU: exp2 and log2 (absolute error
// about 2.4e-7 over the softplus range; the reference's rounding of 1 + exp(v)
// alone is 6e-8).
__device__ __forceinline__ float softplus_ref(float v) { return __logf(1.0f + __expf(v)); }

// Shared-memory row of one rank index: DTP_TOKENS tokens, padded so that the
// transposing writes of the staging loop spread over 8 banks.
constexpr int DTP_XROW = DTP_TOKENS + 4;

// RP: dt_rank rounded up to a multiple of 4 (<= DTP_RMAX).  BWD: write
// dpre = gin * sigmoid(pre) instead of softplus(pre) (as its TF32 hi part in
// out and lo part in out_lo when out_lo is given), and when bpart is given
// the sum of dpre over the CTA's tokens per channel into row blockIdx.y of
// bpart (the dbias partials; summed over rows by the caller).  A CTA covers
// DTP_THREADS * dtp_channels(RP) channels x DTP_TOKENS tokens.
template <int RP, bool BWD>
__global__ void __launch_bounds__(DTP_THREADS)
    dt_softplus_kernel(const float* __restrict__ x, int64_t ldx, int R, const float* __restrict__ W,
                       const float* __restrict__ bias, const float* __restrict__ gin, int64_t ldg,
                       float* __restrict__ out, int64_t ldo, float* __restrict__ out_lo, float* __restrict__ bpart,
                       int64_t ntok, int Dn) {
  constexpr int CH = dtp_channels(RP);
  // xs[r][t]: x of token t0 + t at rank index r (transposed, so one 128-bit
  // load gives 4 tokens' values of one r for the packed FMAs below)
  __shared__ __align__(16) float xs[RP][DTP_XROW];
  const int64_t t0 = int64_t(blockIdx.y) * DTP_TOKENS;
  // staging: every thread's DTP_TOKENS * RP / DTP_THREADS loads are issued
  // before the first shared-memory store, so their latencies overlap
  constexpr int NSTG = DTP_TOKENS * RP / DTP_THREADS;
  static_assert(DTP_TOKENS * RP % DTP_THREADS == 0, "whole staging rounds");
  float xv[NSTG];
#pragma unroll
  for (int j = 0; j < NSTG; ++j) {
    const int i = threadIdx.x + j * DTP_THREADS;
    const int t = i / RP, r = i % RP;
    xv[j] = (t0 + t < ntok && r < R) ? x[(t0 + t) * ldx + r] : 0.f;
  }
#pragma unroll
  for (int j = 0; j < NSTG; ++j) {
    const int i = threadIdx.x + j * DTP_THREADS;
    xs[i % RP][i / RP] = xv[j];
  }
  __syncthreads();
  int dch[CH];
  bool vch[CH];
  float w[CH][RP], b[CH];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    dch[c] = blockIdx.x * DTP_THREADS * CH + c * DTP_THREADS + threadIdx.x;
    vch[c] = dch[c] < Dn;
#pragma unroll
    for (int r = 0; r < RP; ++r) w[c][r] = (vch[c] && r < R) ? W[int64_t(dch[c]) * R + r] : 0.f;
    b[c] = vch[c] ? bias[dch[c]] : 0.f;
  }
  const int nt = int(min(int64_t(DTP_TOKENS), ntok - t0));
  float bsum[CH];
#pragma unroll
  for (int c = 0; c < CH; ++c) bsum[c] = 0.f;
  // DTP_U = 4 tokens per iteration as two packed pairs (rows past nt are zero
  // in xs; their results are not stored); the VJP loads the incoming gradient
  // of the next 4 tokens while it works on the current ones
  float g[CH][DTP_U], gn[CH][DTP_U];
  auto load_g = [&](int tb, float (&dst)[CH][DTP_U]) {
#pragma unroll
    for (int c = 0; c < CH; ++c)
#pragma unroll
      for (int u = 0; u < DTP_U; ++u)
        dst[c][u] = (vch[c] && tb + u < nt) ? gin[(t0 + tb + u) * ldg + dch[c]] : 0.f;
  };
  if (BWD) load_g(0, g);
  for (int tb = 0; tb < nt; tb += DTP_U) {
    if (BWD) load_g(tb + DTP_U, gn);
    float2 a01[CH], a23[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) a01[c] = a23[c] = make_float2(b[c], b[c]);
#pragma unroll
    for (int r = 0; r < RP; ++r) {
      const float4 xv = *reinterpret_cast<const float4*>(&xs[r][tb]);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const float2 wr = make_float2(w[c][r], w[c][r]);
        a01[c] = fma2(make_float2(xv.x, xv.y), wr, a01[c]);
        a23[c] = fma2(make_float2(xv.z, xv.w), wr, a23[c]);
      }
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const float pre[DTP_U] = {a01[c].x, a01[c].y, a23[c].x, a23[c].y};
#pragma unroll
      for (int u = 0; u < DTP_U; ++u) {
        if (vch[c] && tb + u < nt) {
          const int64_t tt = t0 + tb + u;
          if (BWD) {
            const float sig = __fdividef(1.0f, 1.0f + __expf(-pre[u]));
            const float dp = g[c][u] * sig;
            if (out_lo != nullptr) {
              // the TF32 parts of dpre for its two GEMMs instead of dpre itself
              float hi, lo;
              split_tf32(dp, hi, lo);
              out[tt * ldo + dch[c]] = hi;
              out_lo[tt * ldo + dch[c]] = lo;
            } else {
              out[tt * ldo + dch[c]] = dp;
            }
            bsum[c] += dp;
          } else {
            out[tt * ldo + dch[c]] = softplus_ref(pre[u]);
          }
        }
      }
    }
    if (BWD) {
#pragma unroll
      for (int c = 0; c < CH; ++c)
#pragma unroll
        for (int u = 0; u < DTP_U; ++u) g[c][u] = gn[c][u];
    }
  }
  if (BWD && bpart != nullptr) {
#pragma unroll
    for (int c = 0; c < CH; ++c)
      if (vch[c]) bpart[int64_t(blockIdx.y) * Dn + dch[c]] = bsum[c];
  }
}

// Column sums of a row-major (rows x cols, row stride ld) array: out[c] =
// sum_r part[r * ld + c] (the dt_proj VJP's dbias partials, one row per
// 64-token CTA; the LayerNorm VJP's dw / db partials).  A
// CTA of 1024 threads owns 32 columns; thread (g, c) sums rows g, g + 32, g +
// 64, ... of column c with 8 loads in flight at a time, then the 32 group sums
// of a column are added in group order: a fixed order, so the result is
// deterministic.
constexpr int kSumRowsCols = 32, kSumRowsGroups = 32;
__global__ void __launch_bounds__(kSumRowsCols * kSumRowsGroups)
    sum_rows_kernel(const float* __restrict__ part, float* __restrict__ out, int rows, int cols, int64_t ld) {
  __shared__ float gs[kSumRowsGroups][kSumRowsCols];
  const int cl = threadIdx.x % kSumRowsCols, grp = threadIdx.x / kSumRowsCols;
  const int c = blockIdx.x * kSumRowsCols + cl;
  float acc = 0.f;
  if (c < cols) {
    int r = grp;
    for (; r + 7 * kSumRowsGroups < rows; r += 8 * kSumRowsGroups) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = part[int64_t(r + i * kSumRowsGroups) * ld + c];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc += v[i];
    }
    for (; r < rows; r += kSumRowsGroups) acc += part[int64_t(r) * ld + c];
  }
  gs[grp][cl] = acc;
  __syncthreads();
  if (grp == 0 && c < cols) {
    float t = gs[0][cl];
#pragma unroll
    for (int g = 1; g < kSumRowsGroups; ++g) t += gs[g][cl];
    out[c] = t;
  }
}

}  // namespace vmscan
