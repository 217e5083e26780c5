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
// Design.  One CTA (one warpgroup, 4 warps) owns one batch row and 64
// channels for the whole sequence and visits its boxes (<= 16 steps)
// last-to-first.  Warp 0 also acts as producer: per box it writes the row ->
// token table and the row count into the stage, and lane 0 issues the TMA
// loads of u, delta, z, dy, B, C and the bulk copy of the checkpointed state
// that precedes the box.  A consumer quad owns two adjacent channels; each
// lane holds 4 of the 16 states of both, so every shared-memory load, shuffle
// and epilogue serves two channels and the sums over channels start inside
// the lane.  The box's forward steps are recomputed once and exp(delta_t A),
// h_{t-1} of every step are parked in Tensor Memory (256 columns of the
// thread's TMEM lane), so the history costs neither registers nor
// shared-memory bandwidth; the gate (y_pre, dy', dz) is evaluated in that same
// pass.  The reverse pass streams the history back one step ahead of use from
// two alternating register buffers.  State math runs on packed fp32 pairs.
// du/ddelta come out of one quad reduce-scatter and go straight to global
// memory through the token table; dB/dC are reduce-scattered over the warp's
// 8 quads, summed over the 4 warps in a fixed order and written as one
// partial per (CTA, step); dA/dD partials are kept per thread.  Two small
// kernels finish dB/dC (sum over channel tiles, scattered to token order) and
// dA/dD (sum over the batch) in a fixed order: the result is deterministic.
#pragma once

#include "vmscan_common.cuh"

namespace vmscan {

struct BwdCfg {
  static constexpr int NCW = 4;            // one warpgroup: the 4 TMEM lane quarters
  static constexpr int DT = 16 * NCW;      // channels per CTA (2 per quad)
  static constexpr int NCT = NCW * 32;
  static constexpr int NT = NCT;
  static constexpr int NST = 2;
  static constexpr int TILE = TMAX * DT;
  static constexpr int BCT = TMAX * NS;
  static constexpr int CKT = DT * NS;
  static constexpr int TOKF = 32;             // 16 row tokens + row count
  static constexpr uint32_t TMEM_COLS = 128;  // 16 steps x 2 channels x 4 states of h_{t-1}
  // stage: u, delta, z, dy tiles, B, C tiles, checkpoint, token table
  static constexpr int OFF_DT = TILE, OFF_Z = 2 * TILE, OFF_DY = 3 * TILE, OFF_B = 4 * TILE,
                       OFF_C = 4 * TILE + BCT, OFF_CK = 4 * TILE + 2 * BCT, OFF_TOK = 4 * TILE + 2 * BCT + CKT;
  static constexpr int STAGE_F = 4 * TILE + 2 * BCT + CKT + TOKF;
  static constexpr int PART_F = 2 * TMAX * NCW * 32;  // double-buffered per-warp dB/dC partials
  static constexpr int OFF_PART = NST * STAGE_F;
  static constexpr int OFF_BAR = OFF_PART + PART_F;
  static constexpr size_t SMEM_BYTES = size_t(OFF_BAR) * 4 + 2 * NST * 8 + 32 + 1024;
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

// Quad reduce-scatter of v[0..3]: lane q of the quad receives the quad sum of v[q].
__device__ __forceinline__ float quad_scatter(const float v[4], int q) {
  const bool hi2 = (q & 2) != 0;
  float k0 = hi2 ? v[2] : v[0];
  float k1 = hi2 ? v[3] : v[1];
  const float s0 = hi2 ? v[0] : v[2];
  const float s1 = hi2 ? v[1] : v[3];
  k0 += __shfl_xor_sync(0xffffffffu, s0, 2);
  k1 += __shfl_xor_sync(0xffffffffu, s1, 2);
  const bool hi1 = (q & 1) != 0;
  const float keep = hi1 ? k1 : k0;
  const float send = hi1 ? k0 : k1;
  return keep + __shfl_xor_sync(0xffffffffu, send, 1);
}

// Per-thread state of the VJP that lives across boxes.
struct BwdLane {
  float2 Ar[2][2];     // A of the lane's 4 states, per channel, as pairs
  float2 P[2][2];      // dA_{t+1} * dh_{t+1} carried backwards
  float2 dAacc[2][2];  // running dA partials
  float dDacc;         // running dD partial (lanes gq < 2, channel gq)
};

// One box of the VJP.  FULL: the box has all TMAX rows (no per-step guards).
template <bool FULL, bool HAS_Z, bool REV>
__device__ __forceinline__ void bwd_box(BwdLane& L, float* stg, float* part, uint32_t taddr, int nv, int warp, int lane,
                                        int dl0, bool has_ck, bool v0, bool v1, const float (&Dd)[2], float* du_b,
                                        float* dt_b,
                                        float* dz_b, int64_t sdus, int64_t sdts, int64_t sdzs, bool ev) {
  using Cfg = BwdCfg;
  constexpr int DT = Cfg::DT;
  const int gq = lane & 3;
  const float* su = stg + dl0;
  const float* sdt = stg + Cfg::OFF_DT + dl0;
  const float* sz = stg + Cfg::OFF_Z + dl0;
  float* sdy = stg + Cfg::OFF_DY + dl0;
  const float* sB = stg + Cfg::OFF_B + 4 * gq;
  const float* sC = stg + Cfg::OFF_C + 4 * gq;
  const int* tok = reinterpret_cast<const int*>(stg + Cfg::OFF_TOK);
  const int ech = gq & 1;       // epilogue channel of this lane
  const int ekind = gq >> 1;    // gate pass: step parity; reverse pass: 0 du, 1 ddelta

  float2 h[2][2];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    // the checkpoint copy only covers valid channels; other rows are stale
    if (has_ck && (c ? v1 : v0)) {
      const float4 v = lds4(stg + Cfg::OFF_CK + (dl0 + c) * NS + 4 * gq);
      h[c][0] = make_float2(v.x, v.y);
      h[c][1] = make_float2(v.z, v.w);
    } else {
      h[c][0] = h[c][1] = make_float2(0.f, 0.f);
    }
  }
  const float2 log2e2 = bcast2(kLog2e), off2 = bcast2(kEx2ArgBias);

  // ---- forward pass: recompute, park history in TMEM, gate ----
#pragma unroll
  for (int s0 = 0; s0 < TMAX; s0 += 2) {
    if (FULL || s0 < nv) {
      float v[4];
#pragma unroll
      for (int p2 = 0; p2 < 2; ++p2) {
        const int s = s0 + p2;
        v[2 * p2] = v[2 * p2 + 1] = 0.f;
        if (FULL || s < nv) {
          const int r = REV ? nv - 1 - s : s;
          const float2 u2 = lds2(su + r * DT);
          const float2 t2 = lds2(sdt + r * DT);
          const float4 Bv = lds4(sB + r * NS);
          const float2 B2[2] = {make_float2(Bv.x, Bv.y), make_float2(Bv.z, Bv.w)};
          const float2 du2 = mul2(t2, u2);
          const float2 dl2 = mul2(t2, log2e2);
          const float duc[2] = {du2.x, du2.y}, dlc[2] = {dl2.x, dl2.y};
          const float hist[8] = {h[0][0].x, h[0][0].y, h[0][1].x, h[0][1].y,
                                 h[1][0].x, h[1][0].y, h[1][1].x, h[1][1].y};
          tmem_st8(taddr + 8 * s, hist);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const float2 dlb = bcast2(dlc[c]), dub = bcast2(duc[c]);
            const float2 a0 = fma2(dlb, L.Ar[c][0], off2);
            const float2 a1 = fma2(dlb, L.Ar[c][1], off2);
            const float2 e0 = make_float2(ex2_approx(a0.x), ex2_approx(a0.y));
            const float2 e1 = make_float2(ex2_approx(a1.x), ex2_approx(a1.y));
            h[c][0] = fma2(e0, h[c][0], mul2(dub, B2[0]));
            h[c][1] = fma2(e1, h[c][1], mul2(dub, B2[1]));
          }
          if (HAS_Z) {
            const float4 Cv = lds4(sC + r * NS);
            const float2 C01 = make_float2(Cv.x, Cv.y), C23 = make_float2(Cv.z, Cv.w);
            const float2 y0 = fma2(h[0][1], C23, mul2(h[0][0], C01));
            const float2 y1 = fma2(h[1][1], C23, mul2(h[1][0], C01));
            v[2 * p2] = y0.x + y0.y;
            v[2 * p2 + 1] = y1.x + y1.y;
          }
        }
      }
      if (HAS_Z) {
        // lane gq: step s0 + (gq >> 1), channel gq & 1
        const float ys = quad_scatter(v, gq);
        const int s = s0 + ekind;
        if (FULL || s < nv) {
          const int r = REV ? nv - 1 - s : s;
          const float zz = sz[r * DT + ech];
          const float dyv = sdy[r * DT + ech];
          const float ypre = fmaf(su[r * DT + ech], ech ? Dd[1] : Dd[0], ys);
          const float sig = __fdividef(1.0f, 1.0f + ex2_approx(-kLog2e * zz));
          if (ev) dz_b[ech + int64_t(tok[r]) * sdzs] = dyv * ypre * sig * fmaf(zz, 1.0f - sig, 1.0f);
          sdy[r * DT + ech] = dyv * (zz * sig);
        }
      }
    }
  }
  tmem_wait_st();
  __syncwarp();

  // ---- reverse adjoint over the box ----
  // dA / dD are summed per box first and folded into the running totals
  // once per box: L/16 + 16 additions per total instead of L in a row.
  float2 dAbox[2][2];
#pragma unroll
  for (int c = 0; c < 2; ++c) dAbox[c][0] = dAbox[c][1] = make_float2(0.f, 0.f);
  float dDbox = 0.f;
  float2 hs[2][2] = {{h[0][0], h[0][1]}, {h[1][0], h[1][1]}};
  uint32_t X[2][8];  // two alternating history buffers: h_{s-1} of slot s in X[s & 1]
  {
    const int s = FULL ? TMAX - 1 : nv - 1;
    if (FULL || (s & 1)) {
      tmem_ld8(taddr + 8 * s, X[1]);
      tmem_wait_ld8(X[1]);
    } else {
      tmem_ld8(taddr + 8 * s, X[0]);
      tmem_wait_ld8(X[0]);
    }
  }
#pragma unroll
  for (int s = TMAX - 1; s >= 0; --s) {
    if (FULL || s < nv) {
      uint32_t* cur = X[s & 1];
      if (s > 0) tmem_ld8(taddr + 8 * (s - 1), X[(s - 1) & 1]);
      const int r = REV ? nv - 1 - s : s;
      const float2 dy2 = lds2(sdy + r * DT);
      const float2 u2 = lds2(su + r * DT);
      const float2 t2 = lds2(sdt + r * DT);
      const float4 Bv = lds4(sB + r * NS);
      const float4 Cv = lds4(sC + r * NS);
      const float2 B2[2] = {make_float2(Bv.x, Bv.y), make_float2(Bv.z, Bv.w)};
      const float2 C2[2] = {make_float2(Cv.x, Cv.y), make_float2(Cv.z, Cv.w)};
      const float2 du2 = mul2(t2, u2);
      const float2 dl2 = mul2(t2, log2e2);
      const float dyc[2] = {dy2.x, dy2.y}, duc[2] = {du2.x, du2.y}, dtc[2] = {t2.x, t2.y},
                  uc[2] = {u2.x, u2.y}, dlc[2] = {dl2.x, dl2.y};
      float2 vb[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      float2 vc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      float red4[4];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        // exp(delta*A) recomputed exactly as in the forward pass (same operations)
        const float2 dlb = bcast2(dlc[c]);
        const float2 a0 = fma2(dlb, L.Ar[c][0], off2);
        const float2 a1 = fma2(dlb, L.Ar[c][1], off2);
        const float2 e[2] = {make_float2(ex2_approx(a0.x), ex2_approx(a0.y)),
                             make_float2(ex2_approx(a1.x), ex2_approx(a1.y))};
        const float2 hp[2] = {make_float2(__uint_as_float(cur[4 * c + 0]), __uint_as_float(cur[4 * c + 1])),
                              make_float2(__uint_as_float(cur[4 * c + 2]), __uint_as_float(cur[4 * c + 3]))};
        const float2 dyb = bcast2(dyc[c]), dub = bcast2(duc[c]), dtb = bcast2(dtc[c]);
        float2 sB2 = make_float2(0.f, 0.f), sAg2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const float2 dh = fma2(C2[p], dyb, L.P[c][p]);
          const float2 gg = mul2(dh, mul2(e[p], hp[p]));
          sB2 = fma2(dh, B2[p], sB2);
          sAg2 = fma2(L.Ar[c][p], gg, sAg2);
          dAbox[c][p] = fma2(dtb, gg, dAbox[c][p]);
          vb[p] = fma2(dh, dub, vb[p]);
          vc[p] = fma2(dyb, hs[c][p], vc[p]);
          L.P[c][p] = mul2(e[p], dh);
          hs[c][p] = hp[p];
        }
        const float sB = sB2.x + sB2.y;
        red4[c] = dtc[c] * sB;                        // -> du (minus the skip term)
        red4[2 + c] = fmaf(uc[c], sB, sAg2.x + sAg2.y);  // -> ddelta
      }
      // lane gq: gq < 2 -> du of channel gq, gq >= 2 -> ddelta of channel gq - 2
      const float w = quad_scatter(red4, gq);
      if (ev) {
        const int64_t tk = tok[r];
        if (ekind == 0)
          du_b[ech + tk * sdus] = fmaf(ech ? dyc[1] : dyc[0], ech ? Dd[1] : Dd[0], w);
        else
          dt_b[ech + tk * sdts] = w;
      }
      if (ekind == 0) dDbox = fmaf(ech ? dyc[1] : dyc[0], ech ? uc[1] : uc[0], dDbox);
      const float vbs[4] = {vb[0].x, vb[0].y, vb[1].x, vb[1].y};
      const float vcs[4] = {vc[0].x, vc[0].y, vc[1].x, vc[1].y};
      part[(r * Cfg::NCW + warp) * 32 + part_slot(lane)] = warp_reduce8_scatter(vbs, vcs, lane);
      if (s > 0) tmem_wait_ld8(X[(s - 1) & 1]);
    }
  }
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    L.dAacc[c][0] = add2(L.dAacc[c][0], dAbox[c][0]);
    L.dAacc[c][1] = add2(L.dAacc[c][1], dAbox[c][1]);
  }
  L.dDacc += dDbox;
}

template <bool HAS_Z, bool REV>
__global__ void __launch_bounds__(BwdCfg::NT, 3)
    scan_bwd_kernel(const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_dt,
                    const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_dy,
                    const __grid_constant__ CUtensorMap tm_B, const __grid_constant__ CUtensorMap tm_C,
                    float* __restrict__ du_out, int64_t sdub, int64_t sdus, float* __restrict__ ddt_out,
                    int64_t sdtb, int64_t sdts, float* __restrict__ dz_out, int64_t sdzb, int64_t sdzs,
                    const float* __restrict__ A, const float* __restrict__ Dskip, const float* __restrict__ ckpt,
                    float* __restrict__ wpart, float* __restrict__ wA, float* __restrict__ wD, const ScanGeom g,
                    int* __restrict__ status) {
  using Cfg = BwdCfg;
  constexpr int DT = Cfg::DT, NST = Cfg::NST, NCT = Cfg::NCT, NCW = Cfg::NCW;
  extern __shared__ unsigned char smem_raw[];
  float* sm = reinterpret_cast<float*>(align_up_1024(smem_raw));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Cfg::OFF_BAR);
  uint64_t* empty = full + NST;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + NST);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(empty + NST) + 4;

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
  if (warp == 0) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_fence_before_sync();
  }
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t taddr = tmem_base + (uint32_t(warp * 32) << 16);  // this warp's lane quarter

  // Warp 0 doubles as the producer: for box i it writes the row -> token table
  // (one row per lane) and the row count, then lane 0 issues the stage's TMA
  // loads and the checkpoint bulk copy.  A stage is reused once all warps
  // released it.
  auto issue = [&](int i) {  // called by one whole warp
    const int st = i % NST;
    const uint32_t ph = uint32_t(i / NST) & 1u;
    int ok = 1;
    if (lane == 0) ok = mbar_wait(&empty[st], ph ^ 1u, abort_flag, status) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) return;
    const int ib = g.nboxes - 1 - i;  // forward processing index of this box
    const int k = REV ? g.nboxes - 1 - ib : ib;
    int c[3], nv;
    box_coords(g, k, c, nv);
    float* base = sm + st * Cfg::STAGE_F;
    int* tok = reinterpret_cast<int*>(base + Cfg::OFF_TOK);
    if (lane < nv) tok[lane] = int(box_row_token(g, c, lane));
    if (lane == TMAX) tok[TMAX] = nv;
    __syncwarp();
    if (lane == 0) {
      const uint32_t tile_bytes = uint32_t(g.T) * uint32_t((HAS_Z ? 4 : 3) * DT + 2 * NS) * 4u;
      const uint32_t ck_bytes = uint32_t(nvalid_ch) * NS * 4u;
      mbar_arrive_expect_tx(&full[st], tile_bytes + (ib > 0 ? ck_bytes : 0u));
      tma_load_5d(base, &tm_u, &full[st], d0, c[0], c[1], c[2], b);
      tma_load_5d(base + Cfg::OFF_DT, &tm_dt, &full[st], d0, c[0], c[1], c[2], b);
      if (HAS_Z) tma_load_5d(base + Cfg::OFF_Z, &tm_z, &full[st], d0, c[0], c[1], c[2], b);
      tma_load_5d(base + Cfg::OFF_DY, &tm_dy, &full[st], d0, c[0], c[1], c[2], b);
      tma_load_5d(base + Cfg::OFF_B, &tm_B, &full[st], 0, c[0], c[1], c[2], b);
      tma_load_5d(base + Cfg::OFF_C, &tm_C, &full[st], 0, c[0], c[1], c[2], b);
      if (ib > 0) {
        const float* src = ckpt + ((size_t(b) * g.nboxes + (ib - 1)) * g.d_inner + d0) * NS;
        bulk_load(base + Cfg::OFF_CK, src, ck_bytes, &full[st]);
      }
    }
  };
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_u);
      prefetch_tmap(&tm_dt);
      if (HAS_Z) prefetch_tmap(&tm_z);
      prefetch_tmap(&tm_dy);
      prefetch_tmap(&tm_B);
      prefetch_tmap(&tm_C);
    }
    for (int i = 0; i < NST - 1 && i < g.nboxes; ++i) issue(i);
  }

  const int q = lane >> 2;
  const int gq = lane & 3;
  const int dl0 = warp * 16 + 2 * q;  // the quad's two channels: dl0, dl0 + 1
  const int dc = d0 + dl0;
  const bool v0 = dc < g.d_inner, v1 = dc + 1 < g.d_inner;
  BwdLane L;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const bool vc = c ? v1 : v0;
    const float4 a4 = vc ? *reinterpret_cast<const float4*>(A + size_t(dc + c) * NS + 4 * gq)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
    L.Ar[c][0] = make_float2(a4.x, a4.y);
    L.Ar[c][1] = make_float2(a4.z, a4.w);
    L.P[c][0] = L.P[c][1] = make_float2(0.f, 0.f);
    L.dAacc[c][0] = L.dAacc[c][1] = make_float2(0.f, 0.f);
  }
  L.dDacc = 0.f;
  const float Dd[2] = {v0 ? Dskip[dc] : 0.f, v1 ? Dskip[dc + 1] : 0.f};
  const bool ev = (gq & 1) ? v1 : v0;  // the epilogue channel of this lane exists
  float* du_b = du_out + b * sdub + dc;
  float* dt_b = ddt_out + b * sdtb + dc;
  float* dz_b = HAS_Z ? dz_out + b * sdzb + dc : nullptr;
  bool alive = true;

  for (int i = 0; i < g.nboxes; ++i) {
    const int st = i % NST;
    const uint32_t ph = uint32_t(i / NST) & 1u;
    const int ib = g.nboxes - 1 - i;
    // the stage of box i-1 was released by every warp before the barrier that
    // closed box i-1, so this wait does not stall; the producer role rotates
    // over the warps so the per-box barrier does not wait on one busy warp
    if (warp == (i % NCW) && alive && i + NST - 1 < g.nboxes) issue(i + NST - 1);
    alive = alive && mbar_wait(&full[st], ph, abort_flag, status);
    alive = __all_sync(0xffffffffu, alive);  // shuffles and tcgen05 below need the whole warp
    float* part = sm + Cfg::OFF_PART + (i & 1) * (TMAX * NCW * 32);
    float* stg = sm + st * Cfg::STAGE_F;
    const int nv = reinterpret_cast<const int*>(stg + Cfg::OFF_TOK)[TMAX];
    if (alive) {
      if (nv == TMAX)
        bwd_box<true, HAS_Z, REV>(L, stg, part, taddr, nv, warp, lane, dl0, ib > 0, v0, v1, Dd, du_b, dt_b, dz_b,
                                  sdus, sdts, sdzs, ev);
      else
        bwd_box<false, HAS_Z, REV>(L, stg, part, taddr, nv, warp, lane, dl0, ib > 0, v0, v1, Dd, du_b, dt_b, dz_b,
                                   sdus, sdts, sdzs, ev);
    }
    // dy' was written into the stage: order those generic-proxy writes before
    // the TMA load that will refill the stage
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    named_bar_sync(1, NCT);
    if (alive) {
      // fixed-order sum of the warps' partials -> one partial per (CTA, box row)
      float* dst = wpart + ((size_t(b) * g.nboxes + ib) * ndt + dtile) * (TMAX * kPartRow);
#pragma unroll
      for (int e = tid; e < TMAX * kPartRow; e += NCT) {
        const int rr = e / kPartRow;
        if (rr < nv) {
          const int sl = e % kPartRow;
          float acc = 0.f;
#pragma unroll
          for (int w = 0; w < NCW; ++w) acc += part[(rr * NCW + w) * 32 + sl];
          dst[e] = acc;
        }
      }
    }
  }

#pragma unroll
  for (int c = 0; c < 2; ++c) {
    if (c ? v1 : v0)
      *reinterpret_cast<float4*>(wA + (size_t(b) * g.d_inner + dc + c) * NS + 4 * gq) =
          make_float4(L.dAacc[c][0].x, L.dAacc[c][0].y, L.dAacc[c][1].x, L.dAacc[c][1].y);
  }
  if ((gq >> 1) == 0 && ev) wD[size_t(b) * g.d_inner + dc + (gq & 1)] = L.dDacc;
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tmem_fence_after_sync();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
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
