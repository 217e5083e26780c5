// vmscan_fwd.cuh — fused selective-scan forward for sm_100a.
//
// Semantics (mlx_vision_mamba/mamba_block.py:45-73, fused form
// mamba_metal_fused.py:21-63, gate mamba_block.py:190):
//   dA_t[n]  = exp(delta_t * A[d, n])
//   h_t[n]   = dA_t[n] * h_{t-1}[n] + delta_t * u_t * B_t[n]
//   y_t      = sum_n h_t[n] * C_t[n] + u_t * D[d]
//   out_t    = y_t * silu(z_t)            (when a gate is given)
//
// Design.  One CTA owns one batch row and DT = 32*NCW channels for the whole
// sequence.  A producer warp streams boxes of <= 16 scan steps of u, delta,
// z (DT channels each) and B, C (16 states) through an NST-stage TMA ring;
// the tensor maps carry the direction (token permutation), so the consumer
// code only knows "row r of the box".  The producer also writes the token of
// every row into the stage, which the consumers use to store y directly to
// global memory (no output staging, no CTA barriers).  A lane pair owns two
// adjacent channels and each lane holds 8 of the 16 states of both (lane bit
// 0 picks the half), so every B/C load serves two channels and the sum of
// C.h over states is one pair exchange that leaves each lane the output of
// its own channel.  Each step's epilogue (that exchange, the skip term, the
// gate and the store) runs after the next step's state math so its latency
// overlaps independent work.  The state at the end of each box is stored as
// a checkpoint for the VJP.
#pragma once

#include "vmscan_common.cuh"

namespace vmscan {


// T: element type of the sequence tensors (float, or __nv_bfloat16 for the
// bf16 I/O variant); the stage tiles hold T, offsets are in bytes.
template <int NCW, typename T = float>
struct FwdCfg {
  static constexpr int DT = 32 * NCW;          // channels per CTA (32 per warp, 2 per lane pair)
  static constexpr int NCT = NCW * 32;         // consumer threads
  static constexpr int NT = NCT + 32;          // + producer warp
  static constexpr int NST = 2;                // TMA pipeline stages
  static constexpr int TILE = TMAX * DT;       // elements of one (step, channel) tile
  static constexpr int BCT = TMAX * NS;        // elements of one (step, state) tile
  static constexpr int TOKF = 32;              // row -> token table (int32), padded
  static constexpr int ES = int(sizeof(T));
  static constexpr int OFF_DT_B = TILE * ES, OFF_Z_B = 2 * TILE * ES, OFF_B_B = 3 * TILE * ES,
                       OFF_C_B = 3 * TILE * ES + BCT * ES, OFF_TOK_B = 3 * TILE * ES + 2 * BCT * ES;
  static constexpr int STAGE_B = (OFF_TOK_B + TOKF * 4 + 127) / 128 * 128;
  // 16-bit T: each consumer warp's fp32 copy of the box's B and C tiles, after
  // the barriers
  static constexpr int OFF_BCF_B = NST * STAGE_B + 128;
  static constexpr int BCF_B = ES == 4 ? 0 : NCW * 2 * BCT * 4;
  static constexpr size_t SMEM_BYTES = size_t(OFF_BCF_B) + BCF_B + 1024;
};

// Chunked scan over L.  Chunk c holds boxes [c * bpc, min((c + 1) * bpc,
// nboxes)) and runs in its own CTA (grid z).  A CARRY launch runs chunks
// 0 .. nchunks-2 from a zero state and records, per channel, the state at the
// chunk end (carry_h, 16 floats) and the chunk's sum of delta (carry_s): the
// chunk maps a start state h0 to prod_t exp(delta_t A) h0 + carry_h =
// exp(A * carry_s) h0 + carry_h.  carry_fwd_kernel chains those maps into
// h_start, and the main launch starts chunk c from h_start[c].
struct ChunkArgs {
  int bpc;                  // boxes per chunk
  int nchunks;
  const float* h_start;     // (batch, nchunks, d_inner, 16); row c = 0 unused
  float* carry_h;           // (batch, nchunks, d_inner, 16)
  float* carry_s;           // (batch, nchunks, d_inner)
};

// SPLIT: write y as TF32 parts (hi into y, lo into y_lo) for the out_proj
// GEMM; a separate instantiation, so the plain output path carries no per-step
// test for it.
template <int NCW, typename T, bool HAS_Z, bool SAVE_CK, bool STORE_Y, bool REV, bool CARRY = false, bool SPLIT = false>
__global__ void __launch_bounds__(FwdCfg<NCW, T>::NT, 4)
    scan_fwd_kernel(const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_dt,
                    const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_B,
                    const __grid_constant__ CUtensorMap tm_C, T* __restrict__ y, int64_t syb, int sys,
                    float* __restrict__ y_lo, const float* __restrict__ A, const float* __restrict__ Dskip,
                    float* __restrict__ ckpt,
                    const ChunkArgs chunk, const ScanGeom g, int* __restrict__ status) {
  using Cfg = FwdCfg<NCW, T>;
  constexpr int DT = Cfg::DT, NST = Cfg::NST;
  static_assert(!CARRY || (!HAS_Z && !SAVE_CK && !STORE_Y), "a carry pass stores nothing but the carries");
  static_assert(!SPLIT || (STORE_Y && sizeof(T) == 4), "TF32 parts of an fp32 output");
  constexpr bool LOAD_Z = HAS_Z && STORE_Y;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smb = reinterpret_cast<unsigned char*>(smem_align1024(smem_raw));
  uint64_t* full = reinterpret_cast<uint64_t*>(smb + NST * Cfg::STAGE_B);
  uint64_t* empty = full + NST;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + NST);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dtile = blockIdx.x, b = blockIdx.y, cidx = blockIdx.z;
  const int d0 = dtile * DT;
  const int i0 = cidx * chunk.bpc, i1 = min(i0 + chunk.bpc, g.nboxes);  // this CTA's boxes

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
    // Per box: lane 0 waits for the stage to drain (sleeping between polls),
    // lanes < nv write the row -> token table, lane TMAX the row count, then
    // lane 0 issues the TMA loads.
    if (lane == 0) {
      prefetch_tmap(&tm_u);
      prefetch_tmap(&tm_dt);
      if (LOAD_Z) prefetch_tmap(&tm_z);
      prefetch_tmap(&tm_B);
      if (STORE_Y) prefetch_tmap(&tm_C);
    }
    const uint32_t bytes = uint32_t(g.T) * uint32_t((LOAD_Z ? 3 : 2) * DT + (STORE_Y ? 2 : 1) * NS) * Cfg::ES;
    for (int i = i0; i < i1; ++i) {
      const int st = (i - i0) % NST;
      const uint32_t ph = uint32_t((i - i0) / NST) & 1u;
      int ok = 1;
      if (lane == 0) ok = mbar_wait<true>(&empty[st], ph ^ 1u, abort_flag, status) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      const int k = REV ? g.nboxes - 1 - i : i;
      int c[3], nv;
      box_coords(g, k, c, nv);
      unsigned char* base = smb + st * Cfg::STAGE_B;
      int* tok = reinterpret_cast<int*>(base + Cfg::OFF_TOK_B);
      if (STORE_Y && lane < nv) tok[lane] = int(box_row_token(g, c, lane));
      if (lane == TMAX) tok[TMAX] = nv;
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[st], bytes);
        tma_load_5d(base, &tm_u, &full[st], d0, c[0], c[1], c[2], b);
        tma_load_5d(base + Cfg::OFF_DT_B, &tm_dt, &full[st], d0, c[0], c[1], c[2], b);
        if (LOAD_Z) tma_load_5d(base + Cfg::OFF_Z_B, &tm_z, &full[st], d0, c[0], c[1], c[2], b);
        tma_load_5d(base + Cfg::OFF_B_B, &tm_B, &full[st], 0, c[0], c[1], c[2], b);
        if (STORE_Y) tma_load_5d(base + Cfg::OFF_C_B, &tm_C, &full[st], 0, c[0], c[1], c[2], b);
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const PairLane pl(lane);
  const int c0l = warp * 32 + (lane & ~1);  // the pair's two channels: c0l, c0l + 1 (tile-local)
  const int dc = d0 + c0l;
  const bool v0 = dc < g.d_inner, v1 = dc + 1 < g.d_inner;
  const bool ev = pl.hb ? v1 : v0;  // the own channel d0 + c0l + hb exists
  float2 Ar[2][4], h[2][4];
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
    for (int j = 0; j < 4; ++j) h[c][j] = make_float2(0.f, 0.f);
    // a later chunk of a chunked scan starts from the chained carry
    if (!CARRY && cidx > 0 && vc) {
      const float* src = chunk.h_start + ((size_t(b) * chunk.nchunks + cidx) * g.d_inner + dc + c) * NS;
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        const float4 v = *reinterpret_cast<const float4*>(src + pl.group_state(gi));
        h[c][2 * gi] = make_float2(v.x, v.y);
        h[c][2 * gi + 1] = make_float2(v.z, v.w);
      }
    }
  }
  float2 dsum = make_float2(0.f, 0.f);  // CARRY: sum of delta over the chunk, both channels
  const int own = c0l + pl.hb;
  const float Down = ev ? Dskip[d0 + own] : 0.f;
  T* ybase = STORE_Y ? y + b * syb + d0 + own : nullptr;
  float* ylo_base = SPLIT ? y_lo + b * syb + d0 + own : nullptr;
  bool alive = true;

  struct Carry {
    float yp[2];  // C . h over the lane's 8 states, per channel
    float uo;     // own channel u (already in registers: no second shared load)
    int r;
  };

  for (int i = i0; i < i1; ++i) {
    const int st = (i - i0) % NST;
    const uint32_t ph = uint32_t((i - i0) / NST) & 1u;
    alive = alive && mbar_wait(&full[st], ph, abort_flag, status);
    alive = __all_sync(0xffffffffu, alive);  // shuffles below need the whole warp
    if (alive) {
      const unsigned char* sb = smb + st * Cfg::STAGE_B;
      const T* __restrict__ su = reinterpret_cast<const T*>(sb);
      const T* __restrict__ sdt = reinterpret_cast<const T*>(sb + Cfg::OFF_DT_B);
      const T* __restrict__ sz = reinterpret_cast<const T*>(sb + Cfg::OFF_Z_B);
      const T* __restrict__ sB = reinterpret_cast<const T*>(sb + Cfg::OFF_B_B);
      const T* __restrict__ sC = reinterpret_cast<const T*>(sb + Cfg::OFF_C_B);
      // B and C as fp32: the stage itself, or (16-bit T) this warp's widened copy
      const float* __restrict__ sBf;
      const float* __restrict__ sCf;
      if constexpr (Cfg::ES == 4) {
        sBf = reinterpret_cast<const float*>(sB);
        sCf = reinterpret_cast<const float*>(sC);
      } else {
        float* bcf = reinterpret_cast<float*>(smb + Cfg::OFF_BCF_B) + warp * 2 * Cfg::BCT;
        widen_bc_tile(sB, bcf, lane);
        if (STORE_Y) widen_bc_tile(sC, bcf + Cfg::BCT, lane);
        __syncwarp();
        sBf = bcf;
        sCf = bcf + Cfg::BCT;
      }
      const int* tok = reinterpret_cast<const int*>(sb + Cfg::OFF_TOK_B);
      const int nv = tok[TMAX];
      auto math = [&](int s, Carry& k) {
        const int r = REV ? nv - 1 - s : s;
        const float2 u2 = ld_pair(su + r * DT + c0l);
        const float2 t2 = ld_pair(sdt + r * DT + c0l);
        float2 B2[4];
        load8(sBf + r * NS, pl, B2);
        const float2 du2 = mul2(t2, u2);
        const float2 dl2 = mul2(t2, bcast2(kLog2e));
        if (CARRY) dsum = add2(dsum, t2);
        const float duc[2] = {du2.x, du2.y}, dlc[2] = {dl2.x, dl2.y};
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float2 e[4];
          decay8(dlc[c], Ar[c], e);
          const float2 dub = bcast2(duc[c]);
#pragma unroll
          for (int j = 0; j < 4; ++j) h[c][j] = fma2(e[j], h[c][j], mul2(dub, B2[j]));
        }
        if (STORE_Y) {
          float2 C2[4];
          load8(sCf + r * NS, pl, C2);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const float2 acc =
                add2(fma2(C2[1], h[c][1], mul2(C2[0], h[c][0])), fma2(C2[3], h[c][3], mul2(C2[2], h[c][2])));
            k.yp[c] = acc.x + acc.y;
          }
          k.uo = pl.hb ? u2.y : u2.x;
          k.r = r;
        }
      };
      auto epilogue = [&](const Carry& k) {
        const float ys = pair_scatter(k.yp[0], k.yp[1], pl.hb);
        float yy = fmaf(k.uo, Down, ys);
        if (HAS_Z) yy *= silu_f(ld_one(sz + k.r * DT + own));
        const int64_t off = int64_t(tok[k.r]) * sys;
        if constexpr (SPLIT) {
          float hi, lo;
          split_tf32(yy, hi, lo);
          stg_if_t(ybase + off, hi, ev);
          stg_if(ylo_base + off, lo, ev);
        } else {
          stg_if_t(ybase + off, yy, ev);
        }
      };
      Carry ka, kb;
      math(0, ka);
#pragma unroll 2
      for (int s = 1; s < nv; ++s) {
        math(s, kb);
        if (STORE_Y) epilogue(ka);
        ka = kb;
      }
      if (STORE_Y) epilogue(ka);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (SAVE_CK) {
      float* dst = ckpt + ((size_t(b) * g.nboxes + i) * g.d_inner + dc) * NS;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        if (c ? v1 : v0) {
#pragma unroll
          for (int gi = 0; gi < 2; ++gi)
            *reinterpret_cast<float4*>(dst + c * NS + pl.group_state(gi)) =
                make_float4(h[c][2 * gi].x, h[c][2 * gi].y, h[c][2 * gi + 1].x, h[c][2 * gi + 1].y);
        }
      }
    }
  }
  if (CARRY && alive) {
    float* dst = chunk.carry_h + ((size_t(b) * chunk.nchunks + cidx) * g.d_inner + dc) * NS;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      if (c ? v1 : v0) {
#pragma unroll
        for (int gi = 0; gi < 2; ++gi)
          *reinterpret_cast<float4*>(dst + c * NS + pl.group_state(gi)) =
              make_float4(h[c][2 * gi].x, h[c][2 * gi].y, h[c][2 * gi + 1].x, h[c][2 * gi + 1].y);
      }
    }
    if (ev) chunk.carry_s[(size_t(b) * chunk.nchunks + cidx) * g.d_inner + d0 + own] = pl.hb ? dsum.y : dsum.x;
  }
}

// Chains the chunk maps h -> exp(A carry_s[c]) h + carry_h[c] over c = 0 ..
// nchunks-2 from a zero state and writes the state entering every chunk c >= 1
// into h_start.  One thread per (batch, channel, state); exp by the accurate
// expf (the per-step decays of the scan use MUFU ex2; both approximate
// prod_t exp(delta_t A) = exp(A sum_t delta_t)).
__global__ void carry_fwd_kernel(const float* __restrict__ A, const float* __restrict__ carry_h,
                                 const float* __restrict__ carry_s, float* __restrict__ h_start, int batch,
                                 int nchunks, int d_inner) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= int64_t(batch) * d_inner * NS) return;
  const int n = int(idx % NS);
  const int d = int((idx / NS) % d_inner);
  const int b = int(idx / (int64_t(NS) * d_inner));
  const float a = A[int64_t(d) * NS + n];
  float hh = 0.f;
  for (int c = 0; c + 1 < nchunks; ++c) {
    const size_t row = size_t(b) * nchunks + c;
    hh = fmaf(expf(a * carry_s[row * d_inner + d]), hh, carry_h[(row * d_inner + d) * NS + n]);
    h_start[((row + 1) * d_inner + d) * NS + n] = hh;
  }
}

}  // namespace vmscan
