// vmscan_common.cuh — PTX helpers (mbarrier, TMA, MUFU ex2, named barriers),
// the scan-box geometry shared by every kernel, and the sticky device status.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vmscan {

constexpr int NS = 16;     // d_state; the reference hard-codes 16 (mamba_metal_fused.py:28)
constexpr int TMAX = 16;   // scan steps per box (one TMA box, one checkpoint interval)
constexpr float kLog2e = 1.4426950408889634f;

// Bounded waits: each try_wait may suspend at most kSuspendNs; after kWaitLimit
// tries (about one second) the wait gives up, sets the device status and the
// CTA's abort flag, and the kernel drains and returns.
constexpr uint32_t kSuspendNs = 1000;
constexpr uint32_t kWaitLimit = 1u << 20;
constexpr uint32_t kBackoffNs = 200;

constexpr int kStatusTimeout = 9;  // == VMSCAN_ERR_TIMEOUT

// ---------------------------------------------------------------------------
// Scan geometry.  The scan order of a direction is described by up to three
// "scan dims" (fastest first) with a size and a token stride each.  A box is
// `T = P * bj` consecutive scan steps: the full extent of dims < j (product P)
// times `bj` steps of dim j.  Boxes are numbered in scan order; the last box
// along dim j may be ragged, in which case only its first `nvalid` rows exist.
// ---------------------------------------------------------------------------
struct ScanGeom {
  int32_t nsd;            // number of scan dims (1..3)
  int32_t size[3];        // scan dim sizes, fastest first (unused dims: 1)
  int64_t tstride[3];     // token stride of each scan dim
  int32_t j;              // the dim the box is partial along
  int32_t bj;             // box extent along dim j
  int32_t nj;             // ceil(size[j] / bj)
  int32_t P;              // product of size[i] for i < j
  int32_t T;              // rows per box = P * bj (<= TMAX)
  int32_t nboxes;         // boxes per sequence
  int32_t reverse;        // scan runs last -> first
  int32_t batch;
  int32_t d_inner;
  int32_t seqlen;
};

// Box k -> TMA coordinates of scan dims 0..2 and the number of valid rows.
__host__ __device__ __forceinline__ void box_coords(const ScanGeom& g, int k, int c[3], int& nvalid) {
  int rest = k;
  const int cj = (rest % g.nj) * g.bj;
  rest /= g.nj;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (i < g.j) {
      c[i] = 0;
    } else if (i == g.j) {
      c[i] = cj;
    } else if (i < g.nsd) {
      c[i] = rest % g.size[i];
      rest /= g.size[i];
    } else {
      c[i] = 0;
    }
  }
  const int sj = g.j == 0 ? g.size[0] : (g.j == 1 ? g.size[1] : g.size[2]);
  const int left = sj - cj;
  nvalid = g.P * (left < g.bj ? left : g.bj);
}

// Token index of row r of a box with coordinates c.
__host__ __device__ __forceinline__ int64_t box_row_token(const ScanGeom& g, const int c[3], int r) {
  int64_t tok = 0;
  int rem = r;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (i >= g.nsd) break;
    int x;
    if (i < g.j) {
      x = rem % g.size[i];
      rem /= g.size[i];
    } else if (i == g.j) {
      x = c[i] + rem;
    } else {
      x = c[i];
    }
    tok += (int64_t)x * g.tstride[i];
  }
  return tok;
}

// Scan position p (0 = first step taken) -> token index.
__host__ __device__ __forceinline__ int64_t scan_pos_token(const ScanGeom& g, int p) {
  if (g.reverse) p = g.seqlen - 1 - p;
  int64_t tok = 0;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (i >= g.nsd) break;
    const int x = p % g.size[i];
    p /= g.size[i];
    tok += (int64_t)x * g.tstride[i];
  }
  return tok;
}

#if defined(__CUDACC__)

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Exponentials use MUFU ex2.approx.ftz.f32 directly.  Measured on B200 its
// mean relative error is -0.05 .. -0.22 * 2^-23 for arguments in (-0.2, 0)
// (exp(delta*A) close to 1, where the recurrence has a long memory and a
// bias would accumulate), -0.04 .. -0.2 on (-1, -0.2) and -0.42 on (-4, -1).
// A multiplicative correction cannot act below half an ulp of the result, so
// it would over-correct exactly where the memory is long.  Instead the
// argument is shifted by 2^-25 (folded into the FFMA that forms it): measured
// mean relative error is then within +-0.13 * 2^-23 over (-0.2, 0) and -0.16
// on (-1, -0.2).
constexpr float kEx2ArgBias = 2.98023223876953125e-08f;  // 2^-25

__device__ __forceinline__ float2 lds2(const float* p) { return *reinterpret_cast<const float2*>(p); }

// ---- packed fp32 pairs (sm_100 FFMA2 / FMUL2 / FADD2) ----
__device__ __forceinline__ float2 bcast2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }

// ---- Tensor Memory (TMEM) as per-thread scratch ----
// A CTA allocates ncols columns; warp w of a 4-warp group owns TMEM lanes
// 32*(w%4) .. 32*(w%4)+31, thread i of the warp lane 32*(w%4)+i.  The
// 32x32b shape moves one 32-bit column per register for each thread's lane.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tmem_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}


// Store 16 consecutive columns of this thread's lane.  The 16-column TMEM
// helpers carry no memory clobber: Tensor Memory is not reachable by ordinary
// loads and stores, the tcgen05 statements stay ordered among themselves (all
// volatile), and loaded registers are tied to the wait, so shared/global
// accesses may be scheduled across them.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float v[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])));
}

// Issue a load of 16 consecutive columns; valid after tmem_wait_ld16 on the same array.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t r[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }


__device__ __forceinline__ void tmem_wait_ld16(uint32_t r[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]));
}


// silu(z) = z / (1 + 2^(-z*log2 e))
__device__ __forceinline__ float silu_f(float z) {
  return __fdividef(z, 1.0f + ex2_approx(-kLog2e * z));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// CL: acquire at cluster scope (a barrier that the other CTA of a cluster
// arrives on).
template <bool CL = false>
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  if constexpr (CL)
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity.  Returns false (after setting the
// CTA abort flag and the device status) when the wait ran out or another
// thread of the CTA already aborted.
// BACKOFF: sleep kBackoffNs between polls (a producer waiting for a stage to
// drain would otherwise spend issue slots its consumers need).
template <bool BACKOFF = false, bool CL = false>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                          uint32_t limit = kWaitLimit) {
  for (uint32_t it = 0; it < limit; ++it) {
    if (mbar_try_wait<CL>(bar, parity)) return true;
    if (*abort_flag) return false;
    if (BACKOFF) __nanosleep(kBackoffNs);
  }
  *abort_flag = 1;
  atomicExch(status, kStatusTimeout);
  return false;
}

// 5-D tiled TMA load into shared memory, completing on an mbarrier.
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned addresses, size % 16 == 0).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Make generic-proxy shared-memory writes visible to the TMA (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }


// First 1024-byte aligned float of the dynamic shared-memory window.  The
// offset is added to the shared array itself (not through an integer cast),
// so the compiler keeps the shared address space: accesses through the
// result are LDS/STS with 32-bit addresses instead of generic loads.
__device__ __forceinline__ float* smem_align1024(unsigned char* raw) {
  const uint32_t a = smem_u32(raw);
  return reinterpret_cast<float*>(raw + ((1024u - (a & 1023u)) & 1023u));
}

// ---- lane-pair layout shared by the forward and VJP kernels ----

// Lane roles.  Lane l of a warp: pair l >> 1 owns channels 2(l >> 1) and
// 2(l >> 1) + 1 of the warp; the lane's own channel (epilogue) is l.  The
// lane holds states 8 hb .. 8 hb + 7 (hb = l & 1) of both channels, in slot
// order: slot group g (4 states) holds state group g ^ b4 (b4 = bit 4 of l).
struct PairLane {
  int hb, b4, b3, b2, b1;
  __device__ __forceinline__ explicit PairLane(int lane)
      : hb(lane & 1), b4((lane >> 4) & 1), b3((lane >> 3) & 1), b2((lane >> 2) & 1), b1((lane >> 1) & 1) {}
  // first state of slot group g
  __device__ __forceinline__ int group_state(int g) const { return 8 * hb + 4 * (g ^ b4); }
  // slot of this lane's value in the 32-float dB/dC row after dbc_reduce_scatter
  __device__ __forceinline__ int part_slot() const { return 16 * b1 + 8 * hb + 4 * b4 + 2 * b3 + b2; }
};

__device__ __forceinline__ float2 sel2(bool p, float2 a, float2 b) { return p ? a : b; }

// TwoSum (Knuth): acc <- fl(acc + x) and x <- the exact rounding error of
// that addition, for any magnitudes (6 additions, no branch).
__device__ __forceinline__ void two_sum1(float& acc, float& x) {
  const float s = acc + x;
  const float bb = s - acc;
  const float err = (acc - (s - bb)) + (x - bb);
  acc = s;
  x = err;
}

// TF32 hi / lo parts of an fp32 value for the tensor-core GEMM: hi = x
// rounded to 11 significant bits (to nearest, ties away from zero: add half a
// TF32 unit to the magnitude bits, clear the 13 low bits), lo = (x - hi)
// rounded the same way (x - hi is exact).  Integer ALU only, so producers can
// emit the parts beside their fp32 output without loading the exp unit.
__device__ __forceinline__ float tf32_round(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = tf32_round(x);
  lo = tf32_round(x - hi);
}
__device__ __forceinline__ void split_tf32_4(const float4& x, float4& hi, float4& lo) {
  split_tf32(x.x, hi.x, lo.x);
  split_tf32(x.y, hi.y, lo.y);
  split_tf32(x.z, hi.z, lo.z);
  split_tf32(x.w, hi.w, lo.w);
}

__device__ __forceinline__ float2 shfl_xor2(float2 v, int m) {
  return make_float2(__shfl_xor_sync(0xffffffffu, v.x, m), __shfl_xor_sync(0xffffffffu, v.y, m));
}

// Sum over the lane pair: lane hb receives the pair sum of v[hb].
__device__ __forceinline__ float pair_scatter(float v0, float v1, int hb) {
  const float keep = hb ? v1 : v0;
  const float send = hb ? v0 : v1;
  return keep + __shfl_xor_sync(0xffffffffu, send, 1);
}

// exp(delta A) of the lane's 8 states of one channel (MUFU ex2.approx with
// the bias-correcting argument offset); the VJP's forward recompute and its
// reverse pass call this with identical arguments.
__device__ __forceinline__ void decay8(float dl, const float2 Ar[4], float2 e[4]) {
  const float2 dlb = bcast2(dl), off2 = bcast2(kEx2ArgBias);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 a = fma2(dlb, Ar[j], off2);
    e[j] = make_float2(ex2_approx(a.x), ex2_approx(a.y));
  }
}

__device__ __forceinline__ void load8(const float* p, const PairLane& pl, float2 v[4]) {
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const float4 q = lds4(p + pl.group_state(g));
    v[2 * g] = make_float2(q.x, q.y);
    v[2 * g + 1] = make_float2(q.z, q.w);
  }
}

// Global store under a predicate (no branch, no reconvergence region).
__device__ __forceinline__ void stg_if(float* p, float v, bool pred) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q st.global.f32 [%0], %1;\n\t}" ::"l"(p), "f"(v),
      "r"(int(pred)));
}

// ---- element-type access for the scan's input / output tensors ----
// The scans keep their state, accumulations, checkpoints and dA / dD in
// fp32; the sequence tensors (u, delta, z, B, C, dy and y, du, ddelta, dz,
// dB, dC) are fp32 or bf16 (the optional bf16 I/O variant).  Shared-memory
// tiles hold the tensor's own element type; these helpers widen on load and
// round (to nearest even) on store.
template <typename T>
__device__ __forceinline__ float2 ld_pair(const T* p);
template <>
__device__ __forceinline__ float2 ld_pair<float>(const float* p) {
  return lds2(p);
}
template <>
__device__ __forceinline__ float2 ld_pair<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}

template <typename T>
__device__ __forceinline__ float ld_one(const T* p) {
  return float(*p);
}
template <>
__device__ __forceinline__ float ld_one<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

// 8 states of slot order from a row of 16 (B or C of one step).
template <typename T>
__device__ __forceinline__ void load8t(const T* p, const PairLane& pl, float2 v[4]);
template <>
__device__ __forceinline__ void load8t<float>(const float* p, const PairLane& pl, float2 v[4]) {
  load8(p, pl, v);
}
template <>
__device__ __forceinline__ void load8t<__nv_bfloat16>(const __nv_bfloat16* p, const PairLane& pl, float2 v[4]) {
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const uint2 q = *reinterpret_cast<const uint2*>(p + pl.group_state(g));  // 4 bf16
    v[2 * g] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.x));
    v[2 * g + 1] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.y));
  }
}

// Widens a box's B or C tile (TMAX x 16 values of T) into fp32 once per
// box, one warp: lane l converts values 8 l .. 8 l + 7.  For the bf16 I/O
// variant the scans then read the fp32 copy every step (plain 128-bit loads)
// instead of unpacking bf16 pairs at every use.
__device__ __forceinline__ void widen_bc_tile(const __nv_bfloat16* src, float* dst, int lane) {
  const uint4 q = *reinterpret_cast<const uint4*>(src + 8 * lane);
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
  float f[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
    f[2 * k] = v.x;
    f[2 * k + 1] = v.y;
  }
  *reinterpret_cast<float4*>(dst + 8 * lane) = make_float4(f[0], f[1], f[2], f[3]);
  *reinterpret_cast<float4*>(dst + 8 * lane + 4) = make_float4(f[4], f[5], f[6], f[7]);
}

template <typename T>
__device__ __forceinline__ void stg_if_t(T* p, float v, bool pred);
template <>
__device__ __forceinline__ void stg_if_t<float>(float* p, float v, bool pred) {
  stg_if(p, v, pred);
}
template <>
__device__ __forceinline__ void stg_if_t<__nv_bfloat16>(__nv_bfloat16* p, float v, bool pred) {
  const unsigned short bits = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q st.global.b16 [%0], %1;\n\t}" ::"l"(p), "h"(bits),
      "r"(int(pred)));
}

#endif  // __CUDACC__

}  // namespace vmscan
