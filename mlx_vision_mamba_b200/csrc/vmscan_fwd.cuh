// vmscan_fwd.cuh — fused selective-scan forward for sm_100a.
//
// Semantics (mlx_vision_mamba/mamba_block.py:45-73, fused form
// mamba_metal_fused.py:21-63, gate mamba_block.py:190):
//   dA_t[n]  = exp(delta_t * A[d, n])
//   h_t[n]   = dA_t[n] * h_{t-1}[n] + delta_t * u_t * B_t[n]
//   y_t      = sum_n h_t[n] * C_t[n] + u_t * D[d]
//   out_t    = y_t * silu(z_t)            (when a gate is given)
//
// Design.  One CTA owns one batch row and DT = 16*NCW channels for the whole
// sequence.  A producer warp streams boxes of <= 16 scan steps of u, delta,
// z (DT channels each) and B, C (16 states) through an NST-stage TMA ring;
// the tensor maps carry the direction (token permutation), so the consumer
// code only knows "row r of the box".  The producer also writes the token of
// every row into the stage, which the consumers use to store y directly to
// global memory (no output staging, no CTA barriers).  Each consumer quad (4
// lanes) owns two adjacent channels; each lane holds 4 of the 16 states of
// both channels in registers, so B/C loads and the quad shuffles serve two
// channels.  The quad reduce-scatter of y leaves each lane one (step,
// channel) pair per two steps, so the skip/gate epilogue runs once per output.
// The state at the end of each box is stored as a checkpoint for the VJP.
#pragma once

#include "vmscan_common.cuh"

namespace vmscan {

template <int NCW>
struct FwdCfg {
  static constexpr int DT = 16 * NCW;          // channels per CTA (2 per quad)
  static constexpr int NCT = NCW * 32;         // consumer threads
  static constexpr int NT = NCT + 32;          // + producer warp
  static constexpr int NST = 3;                // TMA pipeline stages
  static constexpr int TILE = TMAX * DT;       // floats of one (step, channel) tile
  static constexpr int BCT = TMAX * NS;        // floats of one (step, state) tile
  static constexpr int TOKF = 32;              // row -> token table (int32), padded
  static constexpr int OFF_Z = 2 * TILE, OFF_B = 3 * TILE, OFF_C = 3 * TILE + BCT, OFF_TOK = 3 * TILE + 2 * BCT;
  static constexpr int STAGE_F = 3 * TILE + 2 * BCT + TOKF;
  static constexpr size_t SMEM_BYTES = size_t(NST * STAGE_F) * 4 + 2 * NST * 8 + 16 + 1024;
};

// One forward step for the two channels of a lane: updates h, returns the
// lane's partial of C.h for each channel.  Shared by the forward kernel and
// the VJP's recompute so both produce bit-identical states.
struct Step2 {
  float y0, y1;
};

template <bool WANT_Y>
__device__ __forceinline__ Step2 fwd_step2(float2 (&h)[2][2], const float2 (&Ar)[2][2], float u0, float u1,
                                           float dt0, float dt1, const float4& Bv, const float4& Cv) {
  const float du[2] = {dt0 * u0, dt1 * u1};
  const float dl[2] = {dt0 * kLog2e, dt1 * kLog2e};
  const float2 B2[2] = {make_float2(Bv.x, Bv.y), make_float2(Bv.z, Bv.w)};
  Step2 out{0.f, 0.f};
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const float2 du2 = bcast2(du[c]);
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float2 a = fma2(bcast2(dl[c]), Ar[c][p], bcast2(kEx2ArgBias));
      const float2 e = make_float2(ex2_approx(a.x), ex2_approx(a.y));
      h[c][p] = fma2(e, h[c][p], mul2(du2, B2[p]));
    }
  }
  if (WANT_Y) {
    const float2 C01 = make_float2(Cv.x, Cv.y), C23 = make_float2(Cv.z, Cv.w);
    const float2 y0 = fma2(h[0][1], C23, mul2(h[0][0], C01));
    const float2 y1 = fma2(h[1][1], C23, mul2(h[1][0], C01));
    out.y0 = y0.x + y0.y;
    out.y1 = y1.x + y1.y;
  }
  return out;
}

// Quad reduce-scatter of v = {ch0 step a, ch1 step a, ch0 step b, ch1 step b}:
// lane q of the quad receives the quad sum of v[q], i.e. step (q >> 1),
// channel (q & 1).
__device__ __forceinline__ float quad_scatter4(const float v[4], int q) {
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

template <int NCW, bool HAS_Z, bool SAVE_CK, bool STORE_Y, bool REV>
__global__ void __launch_bounds__(FwdCfg<NCW>::NT, 5)
    scan_fwd_kernel(const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_dt,
                    const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_B,
                    const __grid_constant__ CUtensorMap tm_C, float* __restrict__ y, int64_t syb, int sys,
                    const float* __restrict__ A, const float* __restrict__ Dskip, float* __restrict__ ckpt,
                    const ScanGeom g, int* __restrict__ status) {
  using Cfg = FwdCfg<NCW>;
  constexpr int DT = Cfg::DT, NST = Cfg::NST;
  constexpr bool LOAD_Z = HAS_Z && STORE_Y;
  extern __shared__ unsigned char smem_raw[];
  float* sm = smem_align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + NST * Cfg::STAGE_F);
  uint64_t* empty = full + NST;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + NST);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dtile = blockIdx.x, b = blockIdx.y;
  const int d0 = dtile * DT;

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
      if (LOAD_Z) prefetch_tmap(&tm_z);
      prefetch_tmap(&tm_B);
      if (STORE_Y) prefetch_tmap(&tm_C);
      const uint32_t bytes = uint32_t(g.T) * uint32_t((LOAD_Z ? 3 : 2) * DT + (STORE_Y ? 2 : 1) * NS) * 4u;
      for (int i = 0; i < g.nboxes; ++i) {
        const int st = i % NST;
        const uint32_t ph = uint32_t(i / NST) & 1u;
        if (!mbar_wait(&empty[st], ph ^ 1u, abort_flag, status)) break;
        const int k = REV ? g.nboxes - 1 - i : i;
        int c[3], nv;
        box_coords(g, k, c, nv);
        float* base = sm + st * Cfg::STAGE_F;
        if (STORE_Y) {
          int* tok = reinterpret_cast<int*>(base + Cfg::OFF_TOK);
          for (int r = 0; r < nv; ++r) tok[r] = int(box_row_token(g, c, r));
        }
        mbar_arrive_expect_tx(&full[st], bytes);
        tma_load_5d(base, &tm_u, &full[st], d0, c[0], c[1], c[2], b);
        tma_load_5d(base + Cfg::TILE, &tm_dt, &full[st], d0, c[0], c[1], c[2], b);
        if (LOAD_Z) tma_load_5d(base + Cfg::OFF_Z, &tm_z, &full[st], d0, c[0], c[1], c[2], b);
        tma_load_5d(base + Cfg::OFF_B, &tm_B, &full[st], 0, c[0], c[1], c[2], b);
        if (STORE_Y) tma_load_5d(base + Cfg::OFF_C, &tm_C, &full[st], 0, c[0], c[1], c[2], b);
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int q = lane >> 2;                   // quad within the warp
  const int gq = lane & 3;                   // state group: states 4*gq .. 4*gq+3
  const int dl0 = warp * 16 + 2 * q;         // first of the quad's two channels
  const int dc = d0 + dl0;
  const bool v0 = dc < g.d_inner, v1 = dc + 1 < g.d_inner;
  float2 Ar[2][2], h[2][2];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const bool vc = c ? v1 : v0;
    const float4 a4 = vc ? *reinterpret_cast<const float4*>(A + size_t(dc + c) * NS + 4 * gq)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
    Ar[c][0] = make_float2(a4.x, a4.y);
    Ar[c][1] = make_float2(a4.z, a4.w);
    h[c][0] = h[c][1] = make_float2(0.f, 0.f);
  }
  // epilogue role of this lane: channel (gq & 1), step parity (gq >> 1)
  const int ech = gq & 1;
  const bool evalid = ech ? v1 : v0;
  const float Dd = evalid ? Dskip[dc + ech] : 0.f;
  float* ybase = y + b * syb + dc + ech;
  bool alive = true;

  for (int i = 0; i < g.nboxes; ++i) {
    const int st = i % NST;
    const uint32_t ph = uint32_t(i / NST) & 1u;
    int nv;
    {
      const int k = REV ? g.nboxes - 1 - i : i;
      int c[3];
      box_coords(g, k, c, nv);
    }
    alive = alive && mbar_wait(&full[st], ph, abort_flag, status);
    alive = __all_sync(0xffffffffu, alive);  // shuffles below need the whole warp
    if (alive) {
      const float* su = sm + st * Cfg::STAGE_F + dl0;
      const float* sdt = su + Cfg::TILE;
      const float* sz = su + Cfg::OFF_Z;
      const float* sB = sm + st * Cfg::STAGE_F + Cfg::OFF_B + 4 * gq;
      const float* sC = sm + st * Cfg::STAGE_F + Cfg::OFF_C + 4 * gq;
      const int* tok = reinterpret_cast<const int*>(sm + st * Cfg::STAGE_F + Cfg::OFF_TOK);
      // two steps at a time: the quad scatter needs a pair
#pragma unroll
      for (int s0 = 0; s0 < TMAX; s0 += 2) {
        if (s0 < nv) {
          float v[4];
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            const int s = s0 + p;
            v[2 * p] = 0.f;
            v[2 * p + 1] = 0.f;
            if (s < nv) {
              const int r = REV ? nv - 1 - s : s;
              const float2 u2 = lds2(su + r * DT);
              const float2 t2 = lds2(sdt + r * DT);
              const float4 Bv = lds4(sB + r * NS);
              const float4 Cv = STORE_Y ? lds4(sC + r * NS) : make_float4(0.f, 0.f, 0.f, 0.f);
              const Step2 o = fwd_step2<STORE_Y>(h, Ar, u2.x, u2.y, t2.x, t2.y, Bv, Cv);
              v[2 * p] = o.y0;
              v[2 * p + 1] = o.y1;
            }
          }
          if (STORE_Y) {
            const float ys = quad_scatter4(v, gq);
            const int s = s0 + (gq >> 1);
            if (s < nv && evalid) {
              const int r = REV ? nv - 1 - s : s;
              float yy = fmaf(su[r * DT + ech], Dd, ys);
              if (HAS_Z) yy *= silu_f(sz[r * DT + ech]);
              ybase[int64_t(tok[r]) * sys] = yy;
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (SAVE_CK) {
      float* dst = ckpt + ((size_t(b) * g.nboxes + i) * g.d_inner + dc) * NS + 4 * gq;
      if (v0) *reinterpret_cast<float4*>(dst) = make_float4(h[0][0].x, h[0][0].y, h[0][1].x, h[0][1].y);
      if (v1) *reinterpret_cast<float4*>(dst + NS) = make_float4(h[1][0].x, h[1][0].y, h[1][1].x, h[1][1].y);
    }
  }
}

}  // namespace vmscan
