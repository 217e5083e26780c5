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
// Design.  One CTA (one warpgroup, 4 warps) owns one batch row and 128
// channels for the whole sequence and visits its boxes (<= 16 steps)
// last-to-first.  The producer role rotates over the warps: per box it writes
// the row -> token table and the row count into the stage, and its lane 0
// issues the TMA loads of u, delta, z, dy, B, C and the bulk copy of the
// checkpointed state that precedes the box.  A lane pair owns two adjacent
// channels; each lane of the pair holds 8 of the 16 states of both (lane bit
// 0 picks the half), so a warp covers 32 channels, every per-channel sum
// over states is one pair exchange, and the sums over channels for dB/dC
// start with two channels inside the lane.  The box's forward steps are
// recomputed once and h_{t-1} of every step (16 floats per lane) is parked in
// Tensor Memory (256 columns of the thread's TMEM lane), so the history costs
// neither registers nor shared-memory bandwidth; the gate (y_pre, dy', dz)
// is evaluated in that same pass for the lane's own channel.  The reverse
// pass streams the history back one step ahead of use from two alternating
// register buffers and recomputes exp(delta A) with the forward's exact
// operations.  State math runs on packed fp32 pairs.  du/ddelta of the own
// channel go straight to global memory through the token table; dB/dC are
// reduce-scattered over the 16 lanes holding the same state half (the state
// groups are stored in lane-dependent order so the first stage needs no
// selects), summed over the 4 warps in a fixed order and written as one
// partial per (CTA, step); dA/dD partials are kept per thread.  Two small
// kernels finish dB/dC (sum over channel tiles, scattered to token order) and
// dA/dD (sum over the batch) in a fixed order: the result is deterministic.
#pragma once

#include "vmscan_common.cuh"

namespace vmscan {

// T: element type of the sequence tensors (float, or __nv_bfloat16 for the
// bf16 I/O variant).  Stage offsets are in bytes.
template <typename T = float>
struct BwdCfg {
  static constexpr int NCW = 4;            // one warpgroup: the 4 TMEM lane quarters
  static constexpr int DT = 32 * NCW;      // channels per CTA (32 per warp, 2 per lane pair)
  static constexpr int NCT = NCW * 32;
  static constexpr int NT = NCT;
  static constexpr int NST = 2;
  static constexpr int TILE = TMAX * DT;
  static constexpr int BCT = TMAX * NS;
  static constexpr int CKT = DT * NS;
  static constexpr int TOKF = 32;             // 16 row tokens + row count
  static constexpr uint32_t TMEM_COLS = 256;  // 16 steps x 2 channels x 8 states of h_{t-1}
  static constexpr int ES = int(sizeof(T));
  static constexpr bool F32 = sizeof(T) == 4;
  // stage: u, delta, z, dy tiles (T), B, C tiles (T), checkpoint (fp32), token
  // table, and for 16-bit T an fp32 tile for dy' (fp32 T overwrites dy in place)
  static constexpr int OFF_DT_B = TILE * ES, OFF_Z_B = 2 * TILE * ES, OFF_DY_B = 3 * TILE * ES,
                       OFF_B_B = 4 * TILE * ES, OFF_C_B = 4 * TILE * ES + BCT * ES,
                       OFF_CK_B = (4 * TILE * ES + 2 * BCT * ES + 15) / 16 * 16,
                       OFF_TOK_B = OFF_CK_B + CKT * 4, OFF_DYP_B = F32 ? OFF_DY_B : OFF_TOK_B + TOKF * 4;
  static constexpr int STAGE_B = ((F32 ? OFF_TOK_B + TOKF * 4 : OFF_DYP_B + TILE * 4) + 127) / 128 * 128;
  static constexpr int PART_F = 2 * TMAX * NCW * 32;  // double-buffered per-warp dB/dC partials (fp32)
  static constexpr int OFF_PART_B = NST * STAGE_B;
  static constexpr int OFF_BAR_B = OFF_PART_B + PART_F * 4;
  // 16-bit T: each warp's fp32 copy of the box's B and C tiles, after the barriers
  static constexpr int OFF_BCF_B = OFF_BAR_B + 64;
  static constexpr int BCF_B = F32 ? 0 : NCW * 2 * BCT * 4;
  static constexpr size_t SMEM_BYTES = size_t(OFF_BCF_B) + BCF_B + 1024;
};

// Typed views of one VJP stage.
template <typename T>
struct BwdStage {
  const T* u;
  const T* dt;
  const T* z;
  const T* dy;
  float* dyp;  // dy' = dy silu(z) (fp32), written by the recompute pass
  const T* B;
  const T* C;
  const float* Bf;  // B and C as fp32: the stage tiles, or (16-bit T) the warp's widened copy
  const float* Cf;
  const float* ck;
  const int* tok;
  __device__ __forceinline__ explicit BwdStage(unsigned char* base) {
    using Cfg = BwdCfg<T>;
    u = reinterpret_cast<const T*>(base);
    dt = reinterpret_cast<const T*>(base + Cfg::OFF_DT_B);
    z = reinterpret_cast<const T*>(base + Cfg::OFF_Z_B);
    dy = reinterpret_cast<const T*>(base + Cfg::OFF_DY_B);
    dyp = reinterpret_cast<float*>(base + Cfg::OFF_DYP_B);
    B = reinterpret_cast<const T*>(base + Cfg::OFF_B_B);
    C = reinterpret_cast<const T*>(base + Cfg::OFF_C_B);
    ck = reinterpret_cast<const float*>(base + Cfg::OFF_CK_B);
    tok = reinterpret_cast<const int*>(base + Cfg::OFF_TOK_B);
    Bf = reinterpret_cast<const float*>(B);
    Cf = reinterpret_cast<const float*>(C);
  }
};

// Rows of the per-(CTA, step) dB/dC partial: 16 dB values then 16 dC values.
constexpr int kPartRow = 2 * NS;

// Reduce-scatter of the lane's dB partials vb (8 states, slot order, pairs)
// and dC partials vc over the 16 lanes that hold the same state half.
// Returns one fully reduced value: dB (b1 == 0) or dC (b1 == 1) of state
// 8 hb + 4 b4 + 2 b3 + b2, i.e. PairLane::part_slot().
__device__ __forceinline__ float dbc_reduce_scatter(const float2 vb[4], const float2 vc[4], const PairLane& pl) {
  // lanes l and l^16 hold opposite state groups in slot group 1: send it, keep slot group 0
  const float2 xb0 = add2(vb[0], shfl_xor2(vb[2], 16));
  const float2 xb1 = add2(vb[1], shfl_xor2(vb[3], 16));
  const float2 xc0 = add2(vc[0], shfl_xor2(vc[2], 16));
  const float2 xc1 = add2(vc[1], shfl_xor2(vc[3], 16));
  // state bit 1
  const bool p3 = pl.b3 != 0;
  const float2 yb = add2(sel2(p3, xb1, xb0), shfl_xor2(sel2(p3, xb0, xb1), 8));
  const float2 yc = add2(sel2(p3, xc1, xc0), shfl_xor2(sel2(p3, xc0, xc1), 8));
  // state bit 0 (dB and dC exchanged as one pair)
  const bool p2 = pl.b2 != 0;
  const float2 keep = p2 ? make_float2(yb.y, yc.y) : make_float2(yb.x, yc.x);
  const float2 send = p2 ? make_float2(yb.x, yc.x) : make_float2(yb.y, yc.y);
  const float2 z = add2(keep, shfl_xor2(send, 4));
  // dB or dC
  const bool p1 = pl.b1 != 0;
  return (p1 ? z.y : z.x) + __shfl_xor_sync(0xffffffffu, p1 ? z.x : z.y, 2);
}

// Per-thread state of the VJP that lives across boxes.
//
// dA and dD sum batch x L terms per element, which in a plain running sum
// would cost accuracy at elements whose exact value cancels to near zero.
// dD is summed with Kahan compensation every step (dDcomp).  dA is summed in
// short partials (about eight reverse steps) that are folded into the running total
// by Fast2Sum; the rounding error of each fold starts the next partial
// (dAerr carries it across boxes), so only the products' own roundings
// remain.
struct BwdLane {
  float2 Ar[2][4];     // A of the lane's 8 states (slot order), per channel
  float2 P[2][4];      // dA_{t+1} * dh_{t+1} carried backwards
  float2 dAacc[2][4];  // running dA partials
  float2 dAerr[2][4];  // rounding error of the last fold into dAacc
  float dDacc;         // running dD partial of the own channel
  float dDcomp;        // its Kahan compensation
};

// Folds the short dA partial into the running total (Fast2Sum); the partial
// is left holding the fold's rounding error.
__device__ __forceinline__ void fold_dA(BwdLane& L, float2 (&part)[2][4]) {
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 s = add2(L.dAacc[c][j], part[c][j]);
      const float2 t = add2(s, make_float2(-L.dAacc[c][j].x, -L.dAacc[c][j].y));
      part[c][j] = add2(part[c][j], make_float2(-t.x, -t.y));
      L.dAacc[c][j] = s;
    }
}

// What a reverse step hands to its epilogue.  The epilogue (cross-lane sums,
// stores) of step s runs after the state math of step s - 1, so its shuffle
// chains overlap independent work instead of stalling the in-order warp.
struct RevCarry {
  float2 vb[4], vc[4];  // dB / dC partials of the lane's 8 states (2 channels summed)
  float sBc[2], sAc[2];  // per channel: sum_n dh B, sum_n A g over the lane's states
  float dyo, uo, to;     // own channel: dy', u, delta
  int r;                 // stage row
};

// State math of one reverse step (row r) with the history h_{s-1} in hp.
template <typename T, bool HAS_Z>
__device__ __forceinline__ void bwd_rev_math(BwdLane& L, float2 (&hs)[2][4], float2 (&dAbox)[2][4],
                                             const uint32_t (&hp)[16], const BwdStage<T>& S, int r, int c0l,
                                             const PairLane& pl, RevCarry& k) {
  constexpr int DT = BwdCfg<T>::DT;
  // dy' of the gated scan is the recompute pass's fp32 tile; without a gate
  // dy' = dy (for fp32 T the two are the same tile)
  const float2 dy2 = (HAS_Z || BwdCfg<T>::F32) ? lds2(S.dyp + r * DT + c0l) : ld_pair(S.dy + r * DT + c0l);
  const float2 u2 = ld_pair(S.u + r * DT + c0l);
  const float2 t2 = ld_pair(S.dt + r * DT + c0l);
  float2 B2[4], C2[4];
  load8(S.Bf + r * NS, pl, B2);
  load8(S.Cf + r * NS, pl, C2);
  const float2 du2 = mul2(t2, u2);
  const float2 dl2 = mul2(t2, bcast2(kLog2e));
  const float dyc[2] = {dy2.x, dy2.y}, duc[2] = {du2.x, du2.y}, dtc[2] = {t2.x, t2.y}, dlc[2] = {dl2.x, dl2.y};
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    float2 e[4];
    decay8(dlc[c], L.Ar[c], e);
    const float2 dyb = bcast2(dyc[c]), dub = bcast2(duc[c]), dtb = bcast2(dtc[c]);
    // two accumulators per sum keep the dependent chains short
    float2 sB2[2], sA2[2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 h1 = make_float2(__uint_as_float(hp[8 * c + 2 * j]), __uint_as_float(hp[8 * c + 2 * j + 1]));
      const float2 dh = fma2(C2[j], dyb, L.P[c][j]);
      const float2 pn = mul2(e[j], dh);
      const float2 gg = mul2(pn, h1);
      sB2[j & 1] = j < 2 ? mul2(dh, B2[j]) : fma2(dh, B2[j], sB2[j & 1]);
      sA2[j & 1] = j < 2 ? mul2(L.Ar[c][j], gg) : fma2(L.Ar[c][j], gg, sA2[j & 1]);
      dAbox[c][j] = fma2(dtb, gg, dAbox[c][j]);
      k.vb[j] = c ? fma2(dh, dub, k.vb[j]) : mul2(dh, dub);
      k.vc[j] = c ? fma2(dyb, hs[c][j], k.vc[j]) : mul2(dyb, hs[c][j]);
      L.P[c][j] = pn;
      hs[c][j] = h1;
    }
    const float2 sB = add2(sB2[0], sB2[1]), sA = add2(sA2[0], sA2[1]);
    k.sBc[c] = sB.x + sB.y;
    k.sAc[c] = sA.x + sA.y;
  }
  k.dyo = pl.hb ? dy2.y : dy2.x;
  k.uo = pl.hb ? u2.y : u2.x;
  k.to = pl.hb ? t2.y : t2.x;
  k.r = r;
  // dD += dy' u, Kahan-compensated
  const float yk = fmaf(k.dyo, k.uo, -L.dDcomp);
  const float tk = L.dDacc + yk;
  L.dDcomp = (tk - L.dDacc) - yk;
  L.dDacc = tk;
}

// Epilogue of a reverse step: du / ddelta of the own channel, dB / dC row partial.
template <typename T>
__device__ __forceinline__ void bwd_rev_epilogue(const RevCarry& k, const BwdStage<T>& S, float* __restrict__ part,
                                                 int warp, const PairLane& pl, float Down, T* du_b, T* dt_b, int sdus,
                                                 int sdts, bool ev) {
  const int tk = S.tok[k.r];
  const float sB = pair_scatter(k.sBc[0], k.sBc[1], pl.hb);
  const float sA = pair_scatter(k.sAc[0], k.sAc[1], pl.hb);
  stg_if_t(du_b + int64_t(tk) * sdus, fmaf(k.dyo, Down, k.to * sB), ev);
  stg_if_t(dt_b + int64_t(tk) * sdts, fmaf(k.uo, sB, sA), ev);
  part[(k.r * BwdCfg<T>::NCW + warp) * 32 + pl.part_slot()] = dbc_reduce_scatter(k.vb, k.vc, pl);
}

// What a recompute step hands to its gate epilogue.
struct FwdCarry {
  float yp[2];  // C . h over the lane's 8 states, per channel
  float uo;     // own channel u
  int r;
};

// One box of the VJP (nv rows).  The loops are kept rolled (pairs of steps):
// a fully unrolled box overflows the instruction cache and runs slower.
template <typename T, bool HAS_Z, bool REV, bool SPLIT>
__device__ __forceinline__ void bwd_box(BwdLane& L, const BwdStage<T>& S, float* __restrict__ part, uint32_t taddr,
                                        int nv, int warp, int lane, int c0l, const PairLane& pl, bool has_ck,
                                        bool v0, bool v1, float Down, T* du_b, T* dt_b, T* dz_b, float* dzlo_b,
                                        int sdus, int sdts, int sdzs, bool ev) {
  constexpr int DT = BwdCfg<T>::DT;
  const int* tok = S.tok;
  const int own = c0l + pl.hb;

  float2 h[2][4];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    // the checkpoint copy only covers valid channels; other rows are stale
    if (has_ck && (c ? v1 : v0)) {
      load8(S.ck + (c0l + c) * NS, pl, h[c]);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) h[c][j] = make_float2(0.f, 0.f);
    }
  }

  // ---- forward pass: recompute, park history in TMEM, gate ----
  auto fwd_math = [&](int s, FwdCarry& k) {
    const int r = REV ? nv - 1 - s : s;
    const float2 u2 = ld_pair(S.u + r * DT + c0l);
    const float2 t2 = ld_pair(S.dt + r * DT + c0l);
    float2 B2[4];
    load8(S.Bf + r * NS, pl, B2);
    const float2 du2 = mul2(t2, u2);
    const float2 dl2 = mul2(t2, bcast2(kLog2e));
    const float duc[2] = {du2.x, du2.y}, dlc[2] = {dl2.x, dl2.y};
    float hist[16];
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        hist[8 * c + 2 * j] = h[c][j].x;
        hist[8 * c + 2 * j + 1] = h[c][j].y;
      }
    tmem_st16(taddr + 16 * s, hist);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float2 e[4];
      decay8(dlc[c], L.Ar[c], e);
      const float2 dub = bcast2(duc[c]);
#pragma unroll
      for (int j = 0; j < 4; ++j) h[c][j] = fma2(e[j], h[c][j], mul2(dub, B2[j]));
    }
    if (HAS_Z) {
      float2 C2[4];
      load8(S.Cf + r * NS, pl, C2);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const float2 acc = add2(fma2(C2[1], h[c][1], mul2(C2[0], h[c][0])), fma2(C2[3], h[c][3], mul2(C2[2], h[c][2])));
        k.yp[c] = acc.x + acc.y;
      }
      k.uo = pl.hb ? u2.y : u2.x;
      k.r = r;
    }
  };
  // gate of the own channel: y_pre, dy' (into the stage's fp32 dy' tile,
  // which for fp32 I/O is the dy tile itself), dz
  auto fwd_epilogue = [&](const FwdCarry& k) {
    const float ys = pair_scatter(k.yp[0], k.yp[1], pl.hb);
    const float zz = ld_one(S.z + k.r * DT + own);
    const float dyv = ld_one(S.dy + k.r * DT + own);
    const float ypre = fmaf(k.uo, Down, ys);
    const float sig = __fdividef(1.0f, 1.0f + ex2_approx(-kLog2e * zz));
    const float dzv = dyv * ypre * sig * fmaf(zz, 1.0f - sig, 1.0f);
    const int64_t off = int64_t(tok[k.r]) * sdzs;
    if constexpr (SPLIT) {
      // dz as TF32 parts (hi into dz, lo into dz_lo) for the in_proj gradient GEMMs
      float hi, lo;
      split_tf32(dzv, hi, lo);
      stg_if_t(dz_b + off, hi, ev);
      stg_if(dzlo_b + off, lo, ev);
    } else {
      stg_if_t(dz_b + off, dzv, ev);
    }
    S.dyp[k.r * DT + own] = dyv * (zz * sig);
  };
  {
    FwdCarry fa, fb;
    fwd_math(0, fa);
#pragma unroll 2
    for (int s = 1; s < nv; ++s) {
      fwd_math(s, fb);
      if (HAS_Z) fwd_epilogue(fa);
      fa = fb;
    }
    if (HAS_Z) fwd_epilogue(fa);
  }
  tmem_wait_st();
  __syncwarp();

  // ---- reverse adjoint over the box ----
  // dA partials of about eight steps at a time (every fourth step pair),
  // folded into the running totals (fold_dA); the first starts at the error
  // left by the previous box's last fold
  float2 dAbox[2][4];
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j) dAbox[c][j] = L.dAerr[c][j];
  float2 hs[2][4];
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j) hs[c][j] = h[c][j];
  // Two history buffers: the current step's h_{s-1} and the next one in
  // flight.  Each step's epilogue runs after the next step's math.  The pair
  // loop body has no branch; its look-ahead load is clamped to column 0
  // (re-reading a valid column) on the last pair.
  uint32_t XA[16], XB[16];
  RevCarry ka, kb;
  auto row = [&](int s) { return REV ? nv - 1 - s : s; };
  int s = nv - 1;
  tmem_ld16(taddr + 16 * s, XA);
  tmem_wait_ld16(XA);
  if (s > 0) tmem_ld16(taddr + 16 * (s - 1), XB);
  bwd_rev_math<T, HAS_Z>(L, hs, dAbox, XA, S, row(s), c0l, pl, ka);
  if (s > 0) tmem_wait_ld16(XB);
  int pairs = 0;
#pragma unroll 1
  for (--s; s >= 1; s -= 2, ++pairs) {
    tmem_ld16(taddr + 16 * (s - 1), XA);
    bwd_rev_math<T, HAS_Z>(L, hs, dAbox, XB, S, row(s), c0l, pl, kb);
    bwd_rev_epilogue(ka, S, part, warp, pl, Down, du_b, dt_b, sdus, sdts, ev);
    tmem_wait_ld16(XA);
    tmem_ld16(taddr + 16 * max(s - 2, 0), XB);
    bwd_rev_math<T, HAS_Z>(L, hs, dAbox, XA, S, row(s - 1), c0l, pl, ka);
    bwd_rev_epilogue(kb, S, part, warp, pl, Down, du_b, dt_b, sdus, sdts, ev);
    if ((pairs & 3) == 3) fold_dA(L, dAbox);
    tmem_wait_ld16(XB);
  }
  if (s == 0) {
    bwd_rev_math<T, HAS_Z>(L, hs, dAbox, XB, S, row(0), c0l, pl, kb);
    bwd_rev_epilogue(ka, S, part, warp, pl, Down, du_b, dt_b, sdus, sdts, ev);
    bwd_rev_epilogue(kb, S, part, warp, pl, Down, du_b, dt_b, sdus, sdts, ev);
  } else {
    bwd_rev_epilogue(ka, S, part, warp, pl, Down, du_b, dt_b, sdus, sdts, ev);
  }
  fold_dA(L, dAbox);
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j) L.dAerr[c][j] = dAbox[c][j];
}

// Chunked VJP over L.  Chunk c holds forward boxes [c * bpc, min((c + 1) *
// bpc, nboxes)); its CTA runs them last-to-first starting from the adjoint
// carry p_in[c] (dA_{t+1} dh_{t+1} at the chunk end; zero for the last
// chunk).  The carry depends linearly on the later chunks: a chunk maps an
// incoming carry P to exp(A * sum_t delta_t) P + p_local, where p_local is
// the carry it produces from a zero start (scan_bwd_carry_kernel), chained by
// carry_bwd_kernel.  dA / dD partials are kept per (batch, chunk).
struct BwdChunkArgs {
  int bpc;
  int nchunks;
  const float* p_in;  // (batch, nchunks, d_inner, 16); row nchunks-1 unused
};

// SPLIT: write dz as TF32 parts (hi into dz, lo into dz_lo) for the in_proj
// gradient GEMMs; a separate instantiation, so the plain output path carries no
// per-step test for it.
template <typename T, bool HAS_Z, bool REV, bool SPLIT = false>
__global__ void __launch_bounds__(BwdCfg<T>::NT, 2)
    scan_bwd_kernel(const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_dt,
                    const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_dy,
                    const __grid_constant__ CUtensorMap tm_B, const __grid_constant__ CUtensorMap tm_C,
                    T* __restrict__ du_out, int64_t sdub, int sdus, T* __restrict__ ddt_out,
                    int64_t sdtb, int sdts, T* __restrict__ dz_out, int64_t sdzb, int sdzs, float* __restrict__ dz_lo,
                    const float* __restrict__ A, const float* __restrict__ Dskip, const float* __restrict__ ckpt,
                    float* __restrict__ wpart, float* __restrict__ wA, float* __restrict__ wD,
                    const BwdChunkArgs chunk, const ScanGeom g, int* __restrict__ status) {
  using Cfg = BwdCfg<T>;
  constexpr int DT = Cfg::DT, NST = Cfg::NST, NCT = Cfg::NCT, NCW = Cfg::NCW;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smb = reinterpret_cast<unsigned char*>(smem_align1024(smem_raw));
  uint64_t* full = reinterpret_cast<uint64_t*>(smb + Cfg::OFF_BAR_B);
  uint64_t* empty = full + NST;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + NST);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(empty + NST) + 4;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dtile = blockIdx.x, b = blockIdx.y, cidx = blockIdx.z;
  const int ndt = gridDim.x;
  const int d0 = dtile * DT;
  const int nvalid_ch = min(DT, g.d_inner - d0);
  // this CTA's chunk: forward box indices [i0, i1), visited last-to-first
  const int i0 = cidx * chunk.bpc, i1 = min(i0 + chunk.bpc, g.nboxes), nbx = i1 - i0;

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

  // The producer (warp 0 for the first stages, then warp i % NCW issuing box
  // i + NST - 1) writes the row -> token table (one row per lane) and the row
  // count, then its lane 0 issues the stage's TMA loads and the checkpoint
  // bulk copy.  A stage is reused once all warps released it.
  auto issue = [&](int i) {  // called by one whole warp
    const int st = i % NST;
    const uint32_t ph = uint32_t(i / NST) & 1u;
    int ok = 1;
    if (lane == 0) ok = mbar_wait(&empty[st], ph ^ 1u, abort_flag, status) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) return;
    const int ib = i1 - 1 - i;  // forward processing index of this box
    const int k = REV ? g.nboxes - 1 - ib : ib;
    int c[3], nv;
    box_coords(g, k, c, nv);
    unsigned char* base = smb + st * Cfg::STAGE_B;
    int* tok = reinterpret_cast<int*>(base + Cfg::OFF_TOK_B);
    if (lane < nv) tok[lane] = int(box_row_token(g, c, lane));
    if (lane == TMAX) tok[TMAX] = nv;
    __syncwarp();
    if (lane == 0) {
      const uint32_t tile_bytes = uint32_t(g.T) * uint32_t((HAS_Z ? 4 : 3) * DT + 2 * NS) * uint32_t(Cfg::ES);
      const uint32_t ck_bytes = uint32_t(nvalid_ch) * NS * 4u;
      mbar_arrive_expect_tx(&full[st], tile_bytes + (ib > 0 ? ck_bytes : 0u));
      tma_load_5d(base, &tm_u, &full[st], d0, c[0], c[1], c[2], b);
      tma_load_5d(base + Cfg::OFF_DT_B, &tm_dt, &full[st], d0, c[0], c[1], c[2], b);
      if (HAS_Z) tma_load_5d(base + Cfg::OFF_Z_B, &tm_z, &full[st], d0, c[0], c[1], c[2], b);
      tma_load_5d(base + Cfg::OFF_DY_B, &tm_dy, &full[st], d0, c[0], c[1], c[2], b);
      tma_load_5d(base + Cfg::OFF_B_B, &tm_B, &full[st], 0, c[0], c[1], c[2], b);
      tma_load_5d(base + Cfg::OFF_C_B, &tm_C, &full[st], 0, c[0], c[1], c[2], b);
      if (ib > 0) {
        const float* src = ckpt + ((size_t(b) * g.nboxes + (ib - 1)) * g.d_inner + d0) * NS;
        bulk_load(base + Cfg::OFF_CK_B, src, ck_bytes, &full[st]);
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
    for (int i = 0; i < NST - 1 && i < nbx; ++i) issue(i);
  }

  const PairLane pl(lane);
  const int c0l = warp * 32 + (lane & ~1);  // the pair's two channels: c0l, c0l + 1 (tile-local)
  const int dc = d0 + c0l;
  const bool v0 = dc < g.d_inner, v1 = dc + 1 < g.d_inner;
  const bool ev = pl.hb ? v1 : v0;  // the own channel d0 + c0l + hb exists
  BwdLane L;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const bool vc = c ? v1 : v0;
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
      const float4 a4 = vc ? *reinterpret_cast<const float4*>(A + size_t(dc + c) * NS + pl.group_state(gi))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      L.Ar[c][2 * gi] = make_float2(a4.x, a4.y);
      L.Ar[c][2 * gi + 1] = make_float2(a4.z, a4.w);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) L.P[c][j] = L.dAacc[c][j] = L.dAerr[c][j] = make_float2(0.f, 0.f);
    // a chunk other than the last starts from the adjoint carry of the chunks after it
    if (cidx + 1 < chunk.nchunks && vc) {
      const float* src = chunk.p_in + ((size_t(b) * chunk.nchunks + cidx) * g.d_inner + dc + c) * NS;
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        const float4 v = *reinterpret_cast<const float4*>(src + pl.group_state(gi));
        L.P[c][2 * gi] = make_float2(v.x, v.y);
        L.P[c][2 * gi + 1] = make_float2(v.z, v.w);
      }
    }
  }
  L.dDacc = 0.f;
  L.dDcomp = 0.f;
  const int own = dc + pl.hb;
  const float Down = ev ? Dskip[own] : 0.f;
  T* du_b = du_out + b * sdub + own;
  T* dt_b = ddt_out + b * sdtb + own;
  T* dz_b = HAS_Z ? dz_out + b * sdzb + own : nullptr;
  static_assert(!SPLIT || (HAS_Z && Cfg::F32), "TF32 parts of an fp32 dz");
  float* dzlo_b = SPLIT ? dz_lo + b * sdzb + own : nullptr;
  bool alive = true;

  for (int i = 0; i < nbx; ++i) {
    const int st = i % NST;
    const uint32_t ph = uint32_t(i / NST) & 1u;
    const int ib = i1 - 1 - i;
    // the stage of box i-1 was released by every warp before the barrier that
    // closed box i-1, so this wait does not stall; the producer role rotates
    // over the warps so the per-box barrier does not wait on one busy warp
    if (warp == (i % NCW) && alive && i + NST - 1 < nbx) issue(i + NST - 1);
    alive = alive && mbar_wait(&full[st], ph, abort_flag, status);
    alive = __all_sync(0xffffffffu, alive);  // shuffles and tcgen05 below need the whole warp
    float* part = reinterpret_cast<float*>(smb + Cfg::OFF_PART_B) + (i & 1) * (TMAX * NCW * 32);
    BwdStage<T> S(smb + st * Cfg::STAGE_B);
    if constexpr (!Cfg::F32) {
      if (alive) {
        float* bcf = reinterpret_cast<float*>(smb + Cfg::OFF_BCF_B) + warp * 2 * Cfg::BCT;
        widen_bc_tile(S.B, bcf, lane);
        widen_bc_tile(S.C, bcf + Cfg::BCT, lane);
        __syncwarp();
        S.Bf = bcf;
        S.Cf = bcf + Cfg::BCT;
      }
    }
    const int nv = S.tok[TMAX];
    if (alive)
      bwd_box<T, HAS_Z, REV, SPLIT>(L, S, part, taddr, nv, warp, lane, c0l, pl, ib > 0, v0, v1, Down, du_b, dt_b, dz_b,
                          dzlo_b, sdus, sdts, sdzs, ev);
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
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j) L.dAacc[c][j] = add2(L.dAacc[c][j], L.dAerr[c][j]);
  L.dDacc -= L.dDcomp;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    if (c ? v1 : v0) {
#pragma unroll
      for (int gi = 0; gi < 2; ++gi)
        *reinterpret_cast<float4*>(wA + ((size_t(b) * chunk.nchunks + cidx) * g.d_inner + dc + c) * NS +
                                   pl.group_state(gi)) =
            make_float4(L.dAacc[c][2 * gi].x, L.dAacc[c][2 * gi].y, L.dAacc[c][2 * gi + 1].x,
                        L.dAacc[c][2 * gi + 1].y);
    }
  }
  if (ev) wD[(size_t(b) * chunk.nchunks + cidx) * g.d_inner + own] = L.dDacc;
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tmem_fence_after_sync();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

template <typename T = float>
struct BwdCarryCfg {
  static constexpr int NCW = 4;
  static constexpr int DT = 32 * NCW;  // the VJP's channel tile (same tensor maps)
  static constexpr int NCT = NCW * 32;
  static constexpr int NT = NCT + 32;  // + producer warp
  static constexpr int NST = 2;
  static constexpr int TILE = TMAX * DT;
  static constexpr int BCT = TMAX * NS;
  static constexpr int ES = int(sizeof(T));
  static constexpr int OFF_Z_B = TILE * ES, OFF_DY_B = 2 * TILE * ES, OFF_C_B = 3 * TILE * ES,
                       OFF_NV_B = 3 * TILE * ES + BCT * ES;
  static constexpr int STAGE_B = (OFF_NV_B + 128 + 127) / 128 * 128;
  static constexpr size_t SMEM_BYTES = size_t(NST) * STAGE_B + 2 * NST * 8 + 16 + 1024;
};
static_assert(BwdCarryCfg<>::DT == BwdCfg<>::DT, "the carry pass reads the VJP's tensor maps");

// Adjoint carry of chunks 1 .. nchunks-1 (grid z = chunk - 1) from a zero
// carry at the chunk end: runs dh = C dy' + P, P = exp(delta A) dh backwards
// over the chunk with the VJP's exact operations (gate included) and writes
// P at the chunk start (p_local) and the chunk's sum of delta (carry_s).  The
// state history is not needed for the carry, so this pass only streams
// delta, z, dy and C.
template <typename T, bool HAS_Z, bool REV>
__global__ void __launch_bounds__(BwdCarryCfg<T>::NT, 4)
    scan_bwd_carry_kernel(const __grid_constant__ CUtensorMap tm_dt, const __grid_constant__ CUtensorMap tm_z,
                          const __grid_constant__ CUtensorMap tm_dy, const __grid_constant__ CUtensorMap tm_C,
                          const float* __restrict__ A, float* __restrict__ p_local, float* __restrict__ carry_s,
                          int bpc, int nchunks, const ScanGeom g, int* __restrict__ status) {
  using Cfg = BwdCarryCfg<T>;
  constexpr int DT = Cfg::DT, NST = Cfg::NST, NCW = Cfg::NCW;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smb = reinterpret_cast<unsigned char*>(smem_align1024(smem_raw));
  uint64_t* full = reinterpret_cast<uint64_t*>(smb + NST * Cfg::STAGE_B);
  uint64_t* empty = full + NST;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + NST);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dtile = blockIdx.x, b = blockIdx.y, cidx = blockIdx.z + 1;
  const int d0 = dtile * DT;
  const int i0 = cidx * bpc, i1 = min(i0 + bpc, g.nboxes), nbx = i1 - i0;

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
    // producer: boxes last-to-first, stage = delta, z, dy, C and the row count
    if (lane == 0) {
      prefetch_tmap(&tm_dt);
      if (HAS_Z) prefetch_tmap(&tm_z);
      prefetch_tmap(&tm_dy);
      prefetch_tmap(&tm_C);
      const uint32_t bytes = uint32_t(g.T) * uint32_t((HAS_Z ? 3 : 2) * DT + NS) * uint32_t(Cfg::ES);
      for (int i = 0; i < nbx; ++i) {
        const int st = i % NST;
        const uint32_t ph = uint32_t(i / NST) & 1u;
        if (!mbar_wait<true>(&empty[st], ph ^ 1u, abort_flag, status)) break;
        const int ib = i1 - 1 - i;
        const int k = REV ? g.nboxes - 1 - ib : ib;
        int c[3], nv;
        box_coords(g, k, c, nv);
        unsigned char* base = smb + st * Cfg::STAGE_B;
        reinterpret_cast<int*>(base + Cfg::OFF_NV_B)[0] = nv;
        mbar_arrive_expect_tx(&full[st], bytes);
        tma_load_5d(base, &tm_dt, &full[st], d0, c[0], c[1], c[2], b);
        if (HAS_Z) tma_load_5d(base + Cfg::OFF_Z_B, &tm_z, &full[st], d0, c[0], c[1], c[2], b);
        tma_load_5d(base + Cfg::OFF_DY_B, &tm_dy, &full[st], d0, c[0], c[1], c[2], b);
        tma_load_5d(base + Cfg::OFF_C_B, &tm_C, &full[st], 0, c[0], c[1], c[2], b);
      }
    }
    return;
  }

  const PairLane pl(lane);
  const int c0l = warp * 32 + (lane & ~1);
  const int dc = d0 + c0l;
  const bool v0 = dc < g.d_inner, v1 = dc + 1 < g.d_inner;
  float2 Ar[2][4], P[2][4];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const bool vc = c ? v1 : v0;
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
      const float4 a4 = vc ? *reinterpret_cast<const float4*>(A + size_t(dc + c) * NS + pl.group_state(gi))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      Ar[c][2 * gi] = make_float2(a4.x, a4.y);
      Ar[c][2 * gi + 1] = make_float2(a4.z, a4.w);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) P[c][j] = make_float2(0.f, 0.f);
  }
  float2 dsum = make_float2(0.f, 0.f);
  bool alive = true;
  for (int i = 0; i < nbx; ++i) {
    const int st = i % NST;
    const uint32_t ph = uint32_t(i / NST) & 1u;
    alive = alive && mbar_wait(&full[st], ph, abort_flag, status);
    if (alive) {
      const unsigned char* sb = smb + st * Cfg::STAGE_B;
      const T* __restrict__ sdt = reinterpret_cast<const T*>(sb);
      const T* __restrict__ sz = reinterpret_cast<const T*>(sb + Cfg::OFF_Z_B);
      const T* __restrict__ sdy = reinterpret_cast<const T*>(sb + Cfg::OFF_DY_B);
      const T* __restrict__ sC = reinterpret_cast<const T*>(sb + Cfg::OFF_C_B);
      const int nv = reinterpret_cast<const int*>(sb + Cfg::OFF_NV_B)[0];
#pragma unroll 2
      for (int s = nv - 1; s >= 0; --s) {
        const int r = REV ? nv - 1 - s : s;
        const float2 t2 = ld_pair(sdt + r * DT + c0l);
        float2 dy2 = ld_pair(sdy + r * DT + c0l);
        if (HAS_Z) {
          const float2 z2 = ld_pair(sz + r * DT + c0l);
          const float s0 = __fdividef(1.0f, 1.0f + ex2_approx(-kLog2e * z2.x));
          const float s1 = __fdividef(1.0f, 1.0f + ex2_approx(-kLog2e * z2.y));
          dy2 = make_float2(dy2.x * (z2.x * s0), dy2.y * (z2.y * s1));
        }
        float2 C2[4];
        load8t(sC + r * NS, pl, C2);
        const float2 dl2 = mul2(t2, bcast2(kLog2e));
        dsum = add2(dsum, t2);
        const float dyc[2] = {dy2.x, dy2.y}, dlc[2] = {dl2.x, dl2.y};
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float2 e[4];
          decay8(dlc[c], Ar[c], e);
          const float2 dyb = bcast2(dyc[c]);
#pragma unroll
          for (int j = 0; j < 4; ++j) P[c][j] = mul2(e[j], fma2(C2[j], dyb, P[c][j]));
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  if (!alive) return;
  float* dst = p_local + ((size_t(b) * nchunks + cidx) * g.d_inner + dc) * NS;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    if (c ? v1 : v0) {
#pragma unroll
      for (int gi = 0; gi < 2; ++gi)
        *reinterpret_cast<float4*>(dst + c * NS + pl.group_state(gi)) =
            make_float4(P[c][2 * gi].x, P[c][2 * gi].y, P[c][2 * gi + 1].x, P[c][2 * gi + 1].y);
    }
  }
  if (pl.hb ? v1 : v0) carry_s[(size_t(b) * nchunks + cidx) * g.d_inner + dc + pl.hb] = pl.hb ? dsum.y : dsum.x;
}

// Chains the chunk maps P -> exp(A carry_s[c]) P + p_local[c] from the last
// chunk backwards (zero carry after it) and writes the carry entering every
// chunk c < nchunks-1 at its end into p_in.  One thread per (batch, channel,
// state).
__global__ void carry_bwd_kernel(const float* __restrict__ A, const float* __restrict__ p_local,
                                 const float* __restrict__ carry_s, float* __restrict__ p_in, int batch, int nchunks,
                                 int d_inner) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= int64_t(batch) * d_inner * NS) return;
  const int n = int(idx % NS);
  const int d = int((idx / NS) % d_inner);
  const int b = int(idx / (int64_t(NS) * d_inner));
  const float a = A[int64_t(d) * NS + n];
  float pp = 0.f;
  for (int c = nchunks - 1; c >= 1; --c) {
    const size_t row = size_t(b) * nchunks + c;
    pp = fmaf(expf(a * carry_s[row * d_inner + d]), pp, p_local[(row * d_inner + d) * NS + n]);
    p_in[((row - 1) * d_inner + d) * NS + n] = pp;
  }
}

// dB/dC: sum the per-(channel tile) partials in tile order and scatter each
// row back to its token.  grid (nboxes, batch), block TMAX*32.
template <typename T>
__global__ void reduce_dbc_kernel(const float* __restrict__ wpart, T* __restrict__ dB, int64_t sBb, int64_t sBs,
                                  T* __restrict__ dC, int64_t sCb, int64_t sCs, const ScanGeom g, int ndt) {
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

// dA (d_inner x 16) and dD (d_inner): sum the per-(batch row, chunk)
// partials in order, compensated (each addition's exact rounding error from
// TwoSum is accumulated and added once at the end).
__global__ void reduce_dad_kernel(const float* __restrict__ wA, const float* __restrict__ wD,
                                  float* __restrict__ dA, float* __restrict__ dD, int batch, int d_inner) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const size_t nA = size_t(d_inner) * NS;
  if (idx < nA) {
    float acc = 0.f, comp = 0.f;
    for (int b = 0; b < batch; ++b) {
      float x = wA[size_t(b) * nA + idx];
      two_sum1(acc, x);
      comp += x;
    }
    dA[idx] = acc + comp;
  }
  if (idx < d_inner) {
    float acc = 0.f, comp = 0.f;
    for (int b = 0; b < batch; ++b) {
      float x = wD[size_t(b) * d_inner + idx];
      two_sum1(acc, x);
      comp += x;
    }
    dD[idx] = acc + comp;
  }
}

}  // namespace vmscan
