// vmscan_bwd.cuh — fused selective-scan VJP for sm_100a.
//
// Gradient formulas (they match the reference reverse kernel,
// mlx_vision_mamba/mamba_metal_fused.py:66-145, and its host reductions
// :213-224; dy' is the cotangent before the gate, dy' = dy * silu(z)):
//   dh_t      = C_t * dy'_t + dA_{t+1} * dh_{t+1}
//   g_t[n]    = dh_t[n] * dA_t[n] * h_{t-1}[n]
//   du_t      = dy'_t * D + delta_t * sum_n dh_t[n] B_t[n]
//   ddelta_t  = sum_n A[n] g_t[n] + u_t * sum_n dh_t[n] B_t[n]
//   dA[d, n]  = sum_{b,t} delta_t g_t[n]
//   dB_t[n]   = sum_d dh_t[n] delta_t u_t
//   dC_t[n]   = sum_d dy'_t h_t[n]
//   dD[d]     = sum_{b,t} dy'_t u_t
//   dz_t      = dy_t * y_t * sigma(z_t) * (1 + z_t (1 - sigma(z_t)))
//
// Design.  Same CTA tiling as the forward (one batch row x DT channels, the
// whole sequence), but the boxes are visited last-to-first.  For each box the
// consumer quad reloads the checkpointed state that precedes it (bulk copy in
// the same TMA stage), recomputes the <= 16 forward steps keeping h in
// registers and exp(delta*A) in shared memory, so each exp is computed once,
// then runs the reverse adjoint over the box.  Sums over states use quad
// shuffles; sums over channels (dB, dC) use a warp reduce-scatter (7
// shuffles for 8 values) and a fixed-order cross-warp sum, then one partial
// per (CTA, step) goes to the workspace.  Two small kernels finish dB/dC (sum
// over channel tiles, scattered back to token order) and dA/dD (sum over the
// batch), always in the same order: the result is deterministic.
#pragma once

#include "vmscan_common.cuh"

namespace vmscan {

template <int NCW>
struct BwdCfg {
  static constexpr int DT = 8 * NCW;
  static constexpr int NCT = NCW * 32;
  static constexpr int NT = NCT + 32;
  static constexpr int NST = 3;
  static constexpr int TILE = TMAX * DT;
  static constexpr int BCT = TMAX * NS;
  static constexpr int CKT = DT * NS;
  // stage: u, delta, z, dy tiles, B, C tiles, checkpoint
  static constexpr int STAGE_F = 4 * TILE + 2 * BCT + CKT;
  static constexpr int HIST_F = TMAX * NCT * 4;  // exp(delta*A) per (step, thread, 4 states)
  static constexpr int OUT_F = 2 * 3 * TILE;     // du, ddelta, dz, double-buffered
  static constexpr int PART_F = NCW * TMAX * 32; // per-warp dB/dC partials
  static constexpr int OFF_HIST = NST * STAGE_F;
  static constexpr int OFF_OUT = OFF_HIST + HIST_F;
  static constexpr int OFF_PART = OFF_OUT + OUT_F;
  static constexpr int OFF_BAR = OFF_PART + PART_F;
  static constexpr size_t SMEM_BYTES = size_t(OFF_BAR) * 4 + 2 * NST * 8 + 16 + 1024;
};

// Rows of the per-(CTA, step) dB/dC partial: 16 dB values then 16 dC values.
constexpr int kPartRow = 2 * NS;

// Reduce-scatter of 8 values (vb = dB partials of states 4q..4q+3, vc = dC
// partials of the same states) over the 8 lanes that share q = lane & 3.
// Returns one fully reduced value; its slot is part_slot(lane).
__device__ __forceinline__ float warp_reduce8_scatter(const float vb[4], const float vc[4], int lane) {
  const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
  float w[4];
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const float keep = b4 ? vc[m] : vb[m];
    const float send = b4 ? vb[m] : vc[m];
    w[m] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  float x[2];
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    const float keep = b3 ? w[2 + m] : w[m];
    const float send = b3 ? w[m] : w[2 + m];
    x[m] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  const float keep = b2 ? x[1] : x[0];
  const float send = b2 ? x[0] : x[1];
  return keep + __shfl_xor_sync(0xffffffffu, send, 4);
}

__device__ __forceinline__ int part_slot(int lane) {
  const int b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
  return b4 * NS + 4 * (lane & 3) + 2 * b3 + b2;
}

template <int NCW, bool HAS_Z>
__global__ void __launch_bounds__(BwdCfg<NCW>::NT, 2)
    scan_bwd_kernel(const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_dt,
                    const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_dy,
                    const __grid_constant__ CUtensorMap tm_B, const __grid_constant__ CUtensorMap tm_C,
                    const __grid_constant__ CUtensorMap tm_du, const __grid_constant__ CUtensorMap tm_ddt,
                    const __grid_constant__ CUtensorMap tm_dz, const float* __restrict__ A,
                    const float* __restrict__ Dskip, const float* __restrict__ ckpt, float* __restrict__ wpart,
                    float* __restrict__ wA, float* __restrict__ wD, const ScanGeom g, int* __restrict__ status) {
  using Cfg = BwdCfg<NCW>;
  constexpr int DT = Cfg::DT, TILE = Cfg::TILE, BCT = Cfg::BCT, NST = Cfg::NST, NCT = Cfg::NCT;
  extern __shared__ unsigned char smem_raw[];
  float* sm = reinterpret_cast<float*>(align_up_1024(smem_raw));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Cfg::OFF_BAR);
  uint64_t* empty = full + NST;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + NST);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dtile = blockIdx.x, b = blockIdx.y;
  const int ndt = gridDim.x;
  const int d0 = dtile * DT;
  const int nvalid_ch = min(DT, g.d_inner - d0);

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == NCW) {
    // ---------------- producer warp ----------------
    if (lane == 0) {
      prefetch_tmap(&tm_u);
      prefetch_tmap(&tm_dt);
      if (HAS_Z) prefetch_tmap(&tm_z);
      prefetch_tmap(&tm_dy);
      prefetch_tmap(&tm_B);
      prefetch_tmap(&tm_C);
      const uint32_t tile_bytes = uint32_t(g.T) * uint32_t((HAS_Z ? 4 : 3) * DT + 2 * NS) * 4u;
      const uint32_t ck_bytes = uint32_t(nvalid_ch) * NS * 4u;
      for (int i = 0; i < g.nboxes; ++i) {
        const int st = i % NST;
        const uint32_t ph = uint32_t(i / NST) & 1u;
        if (!mbar_wait(&empty[st], ph ^ 1u, abort_flag, status)) break;
        const int ib = g.nboxes - 1 - i;  // forward processing index of this box
        const int k = g.reverse ? g.nboxes - 1 - ib : ib;
        int c[3], nv;
        box_coords(g, k, c, nv);
        float* base = sm + st * Cfg::STAGE_F;
        mbar_arrive_expect_tx(&full[st], tile_bytes + (ib > 0 ? ck_bytes : 0u));
        tma_load_5d(base, &tm_u, &full[st], d0, c[0], c[1], c[2], b);
        tma_load_5d(base + TILE, &tm_dt, &full[st], d0, c[0], c[1], c[2], b);
        if (HAS_Z) tma_load_5d(base + 2 * TILE, &tm_z, &full[st], d0, c[0], c[1], c[2], b);
        tma_load_5d(base + 3 * TILE, &tm_dy, &full[st], d0, c[0], c[1], c[2], b);
        tma_load_5d(base + 4 * TILE, &tm_B, &full[st], 0, c[0], c[1], c[2], b);
        tma_load_5d(base + 4 * TILE + BCT, &tm_C, &full[st], 0, c[0], c[1], c[2], b);
        if (ib > 0) {
          const float* src = ckpt + ((size_t(b) * g.nboxes + (ib - 1)) * g.d_inner + d0) * NS;
          bulk_load(base + 4 * TILE + 2 * BCT, src, ck_bytes, &full[st]);
        }
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int dl = warp * 8 + (lane >> 2);
  const int gq = lane & 3;
  const int d = d0 + dl;
  const bool dv = d < g.d_inner;
  float A2[4], Ar[4], P[4], dAacc[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    Ar[j] = dv ? A[size_t(d) * NS + 4 * gq + j] : 0.f;
    A2[j] = Ar[j] * kLog2e;
    P[j] = 0.f;
    dAacc[j] = 0.f;
  }
  const float Dd = dv ? Dskip[d] : 0.f;
  float dDacc = 0.f;
  float4* hist = reinterpret_cast<float4*>(sm + Cfg::OFF_HIST);
  float* part = sm + Cfg::OFF_PART;
  const int slot = part_slot(lane);
  bool alive = true;

  for (int i = 0; i < g.nboxes; ++i) {
    const int st = i % NST;
    const uint32_t ph = uint32_t(i / NST) & 1u;
    const int ib = g.nboxes - 1 - i;
    const int k = g.reverse ? g.nboxes - 1 - ib : ib;
    int c[3], nv;
    box_coords(g, k, c, nv);
    alive = alive && mbar_wait(&full[st], ph, abort_flag, status);
    float* o_du = sm + Cfg::OFF_OUT + (i & 1) * 3 * TILE;
    float* o_dt = o_du + TILE;
    float* o_dz = o_du + 2 * TILE;
    if (alive) {
      float* su = sm + st * Cfg::STAGE_F;
      const float* sdt = su + TILE;
      const float* sz = su + 2 * TILE;
      float* sdy = su + 3 * TILE;
      const float* sB = su + 4 * TILE;
      const float* sC = sB + BCT;
      const float* sck = sC + BCT;

      float hin[4] = {0.f, 0.f, 0.f, 0.f};
      if (ib > 0 && dv) {
        const float4 v = lds4(sck + dl * NS + 4 * gq);
        hin[0] = v.x; hin[1] = v.y; hin[2] = v.z; hin[3] = v.w;
      }

      // ---- recompute the box's forward steps ----
      float hh[TMAX][4];
      {
        float hc[4] = {hin[0], hin[1], hin[2], hin[3]};
#pragma unroll
        for (int s = 0; s < TMAX; ++s) {
          if (s < nv) {
            const int r = g.reverse ? nv - 1 - s : s;
            const float uu = su[r * DT + dl];
            const float dd = sdt[r * DT + dl];
            const float4 Bv = lds4(sB + r * NS + 4 * gq);
            const float du = dd * uu;
            const float e0 = ex2_approx(dd * A2[0]);
            const float e1 = ex2_approx(dd * A2[1]);
            const float e2 = ex2_approx(dd * A2[2]);
            const float e3 = ex2_approx(dd * A2[3]);
            hc[0] = fmaf(e0, hc[0], du * Bv.x);
            hc[1] = fmaf(e1, hc[1], du * Bv.y);
            hc[2] = fmaf(e2, hc[2], du * Bv.z);
            hc[3] = fmaf(e3, hc[3], du * Bv.w);
#pragma unroll
            for (int j = 0; j < 4; ++j) hh[s][j] = hc[j];
            hist[s * NCT + tid] = make_float4(e0, e1, e2, e3);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) hh[s][j] = 0.f;
          }
        }
      }

      // ---- gate: y_pre = C.h + u*D, dy' = dy*silu(z), dz ----
      if (HAS_Z) {
#pragma unroll
        for (int s0 = 0; s0 < TMAX; s0 += 4) {
          if (s0 < nv) {
            float yv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int s = s0 + q;
              yv[q] = 0.f;
              if (s < nv) {
                const int r = g.reverse ? nv - 1 - s : s;
                const float4 Cv = lds4(sC + r * NS + 4 * gq);
                float acc = hh[s][0] * Cv.x;
                acc = fmaf(hh[s][1], Cv.y, acc);
                acc = fmaf(hh[s][2], Cv.z, acc);
                acc = fmaf(hh[s][3], Cv.w, acc);
                yv[q] = acc;
              }
            }
            const float ys = quad_transpose_sum(yv, gq);
            const int s = s0 + gq;
            if (s < nv) {
              const int r = g.reverse ? nv - 1 - s : s;
              const float zz = sz[r * DT + dl];
              const float dyv = sdy[r * DT + dl];
              const float ypre = fmaf(su[r * DT + dl], Dd, ys);
              const float sig = __fdividef(1.0f, 1.0f + ex2_approx(-kLog2e * zz));
              const float slu = zz * sig;
              o_dz[r * DT + dl] = dyv * ypre * sig * fmaf(zz, 1.0f - sig, 1.0f);
              sdy[r * DT + dl] = dyv * slu;
            }
          }
        }
        __syncwarp();
      }

      // ---- reverse adjoint over the box ----
#pragma unroll
      for (int s = TMAX - 1; s >= 0; --s) {
        if (s < nv) {
          const int r = g.reverse ? nv - 1 - s : s;
          const float dyp = sdy[r * DT + dl];
          const float uu = su[r * DT + dl];
          const float dd = sdt[r * DT + dl];
          const float du = dd * uu;
          const float4 Bv = lds4(sB + r * NS + 4 * gq);
          const float4 Cv = lds4(sC + r * NS + 4 * gq);
          const float4 ev = hist[s * NCT + tid];
          const float Bj[4] = {Bv.x, Bv.y, Bv.z, Bv.w};
          const float Cj[4] = {Cv.x, Cv.y, Cv.z, Cv.w};
          const float ej[4] = {ev.x, ev.y, ev.z, ev.w};
          float sBsum = 0.f, sAg = 0.f;
          float vb[4], vc[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float hp = (s > 0) ? hh[s > 0 ? s - 1 : 0][j] : hin[j];
            const float dh = fmaf(Cj[j], dyp, P[j]);
            const float gg = dh * (ej[j] * hp);
            sBsum = fmaf(dh, Bj[j], sBsum);
            sAg = fmaf(Ar[j], gg, sAg);
            dAacc[j] = fmaf(dd, gg, dAacc[j]);
            vb[j] = dh * du;
            vc[j] = dyp * hh[s][j];
            P[j] = ej[j] * dh;
          }
          sBsum += __shfl_xor_sync(0xffffffffu, sBsum, 1);
          sAg += __shfl_xor_sync(0xffffffffu, sAg, 1);
          sBsum += __shfl_xor_sync(0xffffffffu, sBsum, 2);
          sAg += __shfl_xor_sync(0xffffffffu, sAg, 2);
          if (gq == 0) o_du[r * DT + dl] = fmaf(dyp, Dd, dd * sBsum);
          if (gq == 1) o_dt[r * DT + dl] = fmaf(uu, sBsum, sAg);
          if (gq == 2) dDacc = fmaf(dyp, uu, dDacc);
          const float red = warp_reduce8_scatter(vb, vc, lane);
          part[(warp * TMAX + r) * kPartRow + slot] = red;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    fence_proxy_async_smem();
    named_bar_sync(1, NCT);
    if (tid == 0) {
      if (alive) {
        tma_store_5d(&tm_du, o_du, d0, c[0], c[1], c[2], b);
        tma_store_5d(&tm_ddt, o_dt, d0, c[0], c[1], c[2], b);
        if (HAS_Z) tma_store_5d(&tm_dz, o_dz, d0, c[0], c[1], c[2], b);
      }
      bulk_commit();
      bulk_wait_read<1>();
    }
    if (alive) {
      float* dst = wpart + ((size_t(b) * g.nboxes + ib) * ndt + dtile) * (TMAX * kPartRow);
      for (int e = tid; e < TMAX * kPartRow; e += NCT) {
        const int rr = e / kPartRow;
        if (rr < nv) {
          float acc = 0.f;
#pragma unroll
          for (int w = 0; w < NCW; ++w) acc += part[w * TMAX * kPartRow + e];
          dst[e] = acc;
        }
      }
    }
    named_bar_sync(1, NCT);
  }

  if (dv) {
    *reinterpret_cast<float4*>(wA + (size_t(b) * g.d_inner + d) * NS + 4 * gq) =
        make_float4(dAacc[0], dAacc[1], dAacc[2], dAacc[3]);
    if (gq == 2) wD[size_t(b) * g.d_inner + d] = dDacc;
  }
  if (tid == 0) bulk_wait<0>();
}

// dB/dC: sum the per-(channel tile) partials in tile order and scatter each
// row back to its token.  grid (nboxes, batch), block TMAX*32.
__global__ void reduce_dbc_kernel(const float* __restrict__ wpart, float* __restrict__ dB, int64_t sBb,
                                  int64_t sBs, float* __restrict__ dC, int64_t sCb, int64_t sCs, const ScanGeom g,
                                  int ndt) {
  const int ib = blockIdx.x, b = blockIdx.y;
  const int k = g.reverse ? g.nboxes - 1 - ib : ib;
  int c[3], nv;
  box_coords(g, k, c, nv);
  const int e = threadIdx.x;
  const int r = e / kPartRow, slot = e % kPartRow;
  if (r >= nv) return;
  const float* p = wpart + ((size_t(b) * g.nboxes + ib) * ndt) * (TMAX * kPartRow) + e;
  float acc = 0.f;
  for (int t = 0; t < ndt; ++t) acc += p[size_t(t) * (TMAX * kPartRow)];
  const int64_t tok = box_row_token(g, c, r);
  if (slot < NS)
    dB[b * sBb + tok * sBs + slot] = acc;
  else
    dC[b * sCb + tok * sCs + (slot - NS)] = acc;
}

// dA (d_inner x 16) and dD (d_inner): sum the per-batch-row partials in order.
__global__ void reduce_dad_kernel(const float* __restrict__ wA, const float* __restrict__ wD,
                                  float* __restrict__ dA, float* __restrict__ dD, int batch, int d_inner) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const size_t nA = size_t(d_inner) * NS;
  if (idx < nA) {
    float acc = 0.f;
    for (int b = 0; b < batch; ++b) acc += wA[size_t(b) * nA + idx];
    dA[idx] = acc;
  }
  if (idx < d_inner) {
    float acc = 0.f;
    for (int b = 0; b < batch; ++b) acc += wD[size_t(b) * d_inner + idx];
    dD[idx] = acc;
  }
}

}  // namespace vmscan
