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
// Layout: a CTA owns DTP_THREADS channels x DTP_TOKENS tokens; the tokens'
// x rows (dt_rank floats, zero-padded to RP) are staged once in shared memory
// and read as broadcasts; each thread keeps its channel's weight row in
// registers, so the dt_rank-long dot product costs dt_rank FMAs and no loads.
// delta / dpre rows are written coalesced (consecutive channels per warp).
#pragma once

#include "vmscan_common.cuh"

namespace vmscan {

constexpr int DTP_THREADS = 256;
constexpr int DTP_TOKENS = 32;
constexpr int DTP_RMAX = 64;

// log(1 + exp(v)) as the reference writes it (inf for v beyond expf's range,
// like the reference); log1pf keeps full precision where exp(v) is small.
__device__ __forceinline__ float softplus_ref(float v) { return log1pf(__expf(v)); }

// RP: dt_rank rounded up to a multiple of 4 (<= DTP_RMAX).  BWD: write
// dpre = gin * sigmoid(pre) instead of softplus(pre).
template <int RP, bool BWD>
__global__ void __launch_bounds__(DTP_THREADS)
    dt_softplus_kernel(const float* __restrict__ x, int64_t ldx, int R, const float* __restrict__ W,
                       const float* __restrict__ bias, const float* __restrict__ gin, int64_t ldg,
                       float* __restrict__ out, int64_t ldo, int64_t ntok, int Dn) {
  __shared__ __align__(16) float xs[DTP_TOKENS][RP];
  const int64_t t0 = int64_t(blockIdx.y) * DTP_TOKENS;
  for (int i = threadIdx.x; i < DTP_TOKENS * RP; i += DTP_THREADS) {
    const int t = i / RP, r = i % RP;
    xs[t][r] = (t0 + t < ntok && r < R) ? x[(t0 + t) * ldx + r] : 0.f;
  }
  __syncthreads();
  const int d = blockIdx.x * DTP_THREADS + threadIdx.x;
  if (d >= Dn) return;
  float w[RP];
#pragma unroll
  for (int r = 0; r < RP; ++r) w[r] = r < R ? W[int64_t(d) * R + r] : 0.f;
  const float b = bias[d];
  const int nt = int(min(int64_t(DTP_TOKENS), ntok - t0));
  for (int t = 0; t < nt; ++t) {
    // two interleaved chains shorten the dependent FMA sequence
    float a0 = b, a1 = 0.f;
#pragma unroll
    for (int r = 0; r < RP; r += 4) {
      const float4 xv = *reinterpret_cast<const float4*>(&xs[t][r]);
      a0 = fmaf(xv.x, w[r], a0);
      a1 = fmaf(xv.y, w[r + 1], a1);
      a0 = fmaf(xv.z, w[r + 2], a0);
      a1 = fmaf(xv.w, w[r + 3], a1);
    }
    const float pre = a0 + a1;
    const int64_t tt = t0 + t;
    if (BWD) {
      const float sig = __fdividef(1.0f, 1.0f + __expf(-pre));
      out[tt * ldo + d] = gin[tt * ldg + d] * sig;
    } else {
      out[tt * ldo + d] = softplus_ref(pre);
    }
  }
}

}  // namespace vmscan
