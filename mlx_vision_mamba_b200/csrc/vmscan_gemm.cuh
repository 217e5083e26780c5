// vmscan_gemm.cuh — fp32-accurate projection GEMMs on the sm_100a tensor
// cores (tcgen05, kind::tf32) for the Mamba block's in_proj / out_proj
// (mlx_vision_mamba/mamba_block.py:165,191 and the direction sum :562-566).
//
// Precision.  TF32 keeps 11 significant bits.  Each fp32 operand x is split
// into hi = tf32(x) and lo = tf32(x - hi) (split_tf32: round to nearest,
// ties away; x - hi is exact), so x =
// hi + lo to about 2^-22 |x|, and
//     C = A_hi B_hi + (A_hi B_lo + A_lo B_hi)
// drops only A_lo B_lo (~2^-22 of a product).  The large products and the
// two correction products accumulate in separate TMEM accumulators, summed
// once in fp32 by the epilogue, so the rounding of the running sum acts on
// the large products alone, as it does in an fp32 FFMA loop.  The split is a
// separate elementwise pass (tf32_split_kernel), or written by the kernel
// that produces the operand, and the GEMM reads the two parts.
//
// Design.  A persistent CTA per SM walks the 128 x BN output tiles (and K
// splits), 320 threads: warp 0 lane 0 issues the TMA loads of the hi / lo
// tiles of A and B into an NST-stage ring of mbarriers; warp 1 owns the TMEM
// allocation and its lane 0 issues the tcgen05.mma instructions (3 per K=8
// step) and the tcgen05.commit that releases each stage; warps 2..9 (two per
// TMEM lane quarter, half the columns each) read the accumulators back with
// tcgen05.ld, add them and store the tile.  Operand tiles use a 128-byte swizzle; an operand is
// either K-major (rows of K contiguous, one TMA box of 32 x rows, 16-byte
// chunks swizzled) or MN-major (rows of M or N contiguous: 32-element column
// blocks of 32 K rows each, 4 KB apart, 32-byte chunks swizzled).  Every wait is bounded: on time-out the kernel
// records VMSCAN_ERR_TIMEOUT in the device status and drains.
//
// Weight gradients (MN-major A, 128-column tiles, M a multiple of 256) run
// as CTA pairs instead: clusters of 2 CTAs compute 256 x 128 items with
// cta_group::2 MMAs issued by the leader, each CTA holding its 128 rows of A
// and half of B, so the ring has 4 stages of 48 KB instead of 3 of 64 KB.
// The pairs' TMA loads carry no multicast (the same code runs on every GPU
// of a multi-GPU job).
#pragma once

#include "vmscan_common.cuh"

namespace vmscan {

constexpr int GM_BM = 128;
constexpr int GM_BK = 32;  // fp32 elements per k-block: one 128-byte swizzle row
constexpr int GM_THREADS = 320;
constexpr int GM_EPI_WARP0 = 2;  // warps 2..9: two epilogue warps per TMEM lane quarter
constexpr int GM_EPI_WARPS = 8;

// Large-product TMEM buffers for narrower tiles (128-column tiles use two,
// which with the two correction buffers fill TMEM), and k-blocks per
// promotion chain.  Measured on B200 inside CUDA graphs at the VisionMamba-2D
// shapes: chains of 2 k-blocks run the 128-column GEMMs 9-14 % faster than
// chains of 1 (half the MMA / epilogue hand-overs), chains of 3 another 2-7 %
// (training step 21.66 -> 21.07 ms; 4 gain nothing more).  RMS error of the
// output RMS on N(0,1) operands at K = 384 / 3072 / 12544: chains of 2
// 2.0 / 2.3 / 2.7e-7, of 3 2.7 / 2.9 / 3.1e-7, of 4 3.4 / 3.5 / 3.6e-7,
// against PyTorch's fp32 GEMM 3.5 / 9.9 / 20e-7; 4 narrow buffers instead of
// 2 change little.
#ifndef VMSCAN_GEMM_NB_NARROW
#define VMSCAN_GEMM_NB_NARROW 4
#endif
#ifndef VMSCAN_GEMM_PK
#define VMSCAN_GEMM_PK 3
#endif

// Ring stages and shared-memory layout of one CTA.  PAIR: the CTA is one of
// a cluster pair that computes a 256 x BN tile with cta_group::2 MMAs; each
// CTA holds its own 128 rows of A but only its half (BN / 2 rows) of B, so a
// stage is 48 KB instead of 64 KB and the ring gets 4 stages instead of 3.
template <int BN, bool PAIR = false>
struct GemmCfg {
  static_assert(BN == 32 || BN == 64 || BN == 128, "BN: 32, 64 or 128");
  static_assert(!PAIR || BN == 128, "CTA pairs use 128-column tiles");
  static constexpr int BM = PAIR ? 2 * GM_BM : GM_BM;  // output rows of a work item
  static constexpr int BROWS = PAIR ? BN / 2 : BN;      // rows of B one CTA loads
  static constexpr int A_TILE_B = GM_BM * GM_BK * 4;  // 16 KB
  static constexpr int B_TILE_B = BROWS * GM_BK * 4;
  static constexpr int OFF_ALO = A_TILE_B, OFF_BHI = 2 * A_TILE_B, OFF_BLO = 2 * A_TILE_B + B_TILE_B;
  static constexpr int STAGE_B = 2 * A_TILE_B + 2 * B_TILE_B;
  static constexpr int NST = (196 * 1024) / STAGE_B < 6 ? (196 * 1024) / STAGE_B : 6;
  static_assert(NST >= 2, "at least two stages");
  // accumulators: NB large-product buffers (columns 0 .. NB BN), two
  // correction buffers after them
  static constexpr int NB = BN == 128 ? 2 : VMSCAN_GEMM_NB_NARROW;
  static constexpr int PK = VMSCAN_GEMM_PK;  // k-blocks whose large products share one buffer
  static_assert((NB + 2) * BN <= 512, "accumulators fit in TMEM");
  static constexpr uint32_t TMEM_COLS =
      (NB + 2) * BN <= 128 ? 128u : ((NB + 2) * BN <= 256 ? 256u : 512u);
  static constexpr int OFF_BAR = NST * STAGE_B;
  static_assert((2 * NST + 2 * NB + 2) * 8 + 8 <= 256, "barriers, abort flag and TMEM slot fit in 256 bytes");
  // per epilogue warp a 32-row x EPI_SC-column fp32 staging tile: the warp
  // writes its rows (one per lane) there and stores whole row pieces to global
  static constexpr int EPI_SC = BN / 2 < 32 ? BN / 2 : 32;
  static constexpr int OFF_EPI = OFF_BAR + 256;
  static constexpr int EPI_B = GM_EPI_WARPS * 32 * EPI_SC * 4;
  static constexpr size_t SMEM_BYTES = size_t(OFF_EPI) + EPI_B + 1024;
  static_assert(SMEM_BYTES <= 232448, "fits the 227 KB opt-in shared memory");
};

// ---- tcgen05 helpers ----

// Shared-memory matrix descriptor (sm_100 format, version 1).  lbo / sbo in
// bytes; layout 2 = 128-byte swizzle of 16-byte chunks (K-major tiles), 1 =
// 128-byte swizzle of 32-byte chunks (the layout 32-bit MN-major tiles need).
__device__ __forceinline__ uint64_t umma_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = uint64_t((saddr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;  // descriptor version
  d |= uint64_t(layout) << 61;
  return d;
}

// Instruction descriptor: D fp32, A and B tf32, M = m (128, or 256 for a CTA
// pair), N = n.
__host__ __device__ constexpr uint32_t umma_idesc_tf32(int n, bool a_mn, bool b_mn, int m = GM_BM) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
         (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation issued so far by this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---- CTA-pair (cta_group::2) helpers ----

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the variable at p in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}

// Every thread of both CTAs of the cluster.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Tiled load into this CTA's shared memory whose bytes are counted on the
// barrier at shared::cluster address `bar` (the pair leader's).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

// One 256 x N x 8 MMA of the pair, issued by the leader: A rows 0..127 and B
// columns 0..N/2-1 from the leader's shared memory, A rows 128..255 and B
// columns N/2..N-1 from the peer's (same offsets), D rows split the same way
// over the two CTAs' TMEM.
__device__ __forceinline__ void umma_tf32_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at this offset in both CTAs of the pair once the
// pair's MMAs issued so far have completed: one commit per CTA's barrier
// (shared::cluster addresses of rank 0 and rank 1).
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   cluster_addr(bar, 0))
               : "memory");
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   cluster_addr(bar, 1))
               : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t r[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// hi / lo split of n fp32 values (split_tf32, the same rounding the
// producer kernels use when they emit the parts themselves).  The host
// guarantees n % 4 == 0 and 16-byte aligned pointers.
__global__ void tf32_split_kernel(const float4* __restrict__ x, float4* __restrict__ hi, float4* __restrict__ lo,
                                  int64_t n4) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
    float4 h, l;
    split_tf32_4(x[i], h, l);
    hi[i] = h;
    lo[i] = l;
  }
}

// Several tensors' hi / lo splits in one launch (the weights of a block):
// the table travels in the kernel parameters, so the launch can be captured
// in a CUDA graph.  blockIdx.y picks the tensor.
constexpr int kSplitMaxTensors = 16;
struct SplitTable {
  const float4* x[kSplitMaxTensors];
  float4* hi[kSplitMaxTensors];
  float4* lo[kSplitMaxTensors];
  int64_t n4[kSplitMaxTensors];
};

__global__ void tf32_split_multi_kernel(const __grid_constant__ SplitTable t) {
  const int k = blockIdx.y;
  const float4* __restrict__ x = t.x[k];
  float4* __restrict__ hi = t.hi[k];
  float4* __restrict__ lo = t.lo[k];
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < t.n4[k]; i += int64_t(gridDim.x) * blockDim.x) {
    float4 h, l;
    split_tf32_4(x[i], h, l);
    hi[i] = h;
    lo[i] = l;
  }
}

// Loads the hi and lo tiles of one operand for k-block kb.  K-major: one box
// {32 k, rows} at (k0, r0).  MN-major: nbox <= rows/32 boxes {32 mn, 32 k} at
// (r0 + 32 j, k0), 4 KB apart; boxes that would lie wholly past the operand's
// last row are not issued (their smem rows only feed outputs that are not
// stored).  Boxes that straddle the edge are zero-filled by the TMA.
// PAIR: the bytes are counted on the pair leader's barrier (bar_c, its
// shared::cluster address) instead of bar.
template <bool PAIR>
__device__ __forceinline__ void gemm_tma(void* dst, const CUtensorMap* map, uint64_t* bar, uint32_t bar_c, int c0,
                                         int c1) {
  if constexpr (PAIR)
    tma_load_2d_pair(dst, map, bar_c, c0, c1);
  else
    tma_load_2d(dst, map, bar, c0, c1);
}

template <int ROWS, bool MN, bool PAIR = false>
__device__ __forceinline__ void gemm_load_operand(unsigned char* hi_dst, unsigned char* lo_dst, const CUtensorMap* mhi,
                                                  const CUtensorMap* mlo, uint64_t* bar, uint32_t bar_c, int r0,
                                                  int k0, int nbox) {
  if (!MN) {
    gemm_tma<PAIR>(hi_dst, mhi, bar, bar_c, k0, r0);
    gemm_tma<PAIR>(lo_dst, mlo, bar, bar_c, k0, r0);
  } else {
#pragma unroll
    for (int j = 0; j < ROWS / 32; ++j) {
      if (j < nbox) {
        gemm_tma<PAIR>(hi_dst + j * 4096, mhi, bar, bar_c, r0 + 32 * j, k0);
        gemm_tma<PAIR>(lo_dst + j * 4096, mlo, bar, bar_c, r0 + 32 * j, k0);
      }
    }
  }
}

// Boxes of an MN-major operand tile starting at row r0 of `rows` that hold at
// least one row (all ROWS/32 for a K-major operand, which loads one box).
template <int ROWS, bool MN>
__device__ __forceinline__ int gemm_nbox(int r0, int rows) {
  return MN ? max(0, min(ROWS / 32, (rows - r0 + 31) / 32)) : ROWS / 32;
}

// Descriptor of the kk-th K=8 step of an operand tile.  K-major: rows of
// 128 bytes (32 k), 8-row atoms 1 KB apart (SBO), the step advances 32 bytes
// along the row.  MN-major: 32-element column blocks of GM_BK rows 4 KB apart
// (LBO), 4-row atoms of the 32-byte-chunk swizzle 512 bytes apart (SBO), the
// step advances 8 rows.
template <bool MN>
__device__ __forceinline__ uint64_t gemm_desc(uint32_t tile, int kk) {
  return MN ? umma_sdesc(tile + uint32_t(kk) * 1024u, uint32_t(GM_BK) * 128u, 512u, 1u)
            : umma_sdesc(tile + uint32_t(kk) * 32u, 16u, 1024u, 2u);
}

struct GemmArgs {
  int M, N, K;
  int splits;        // K splits (work items = output tiles x splits)
  int kb_per_split;  // k-blocks per split
  int accumulate;    // C += A B (one split only) instead of C = A B
  float* C;          // output (splits == 1) or the split partials (M x N each, row stride N)
  int64_t ldc;
  int64_t split_stride;  // elements between split partials
};

// Waits for this thread's outstanding tcgen05.ld and ties the 32 loaded
// registers to the wait, so no use of them is scheduled before it.
__device__ __forceinline__ void tmem_wait_ld32(uint32_t r[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

// Loads NC (16, 32 or 64) consecutive TMEM columns of this thread's lane into
// r and waits for them.
template <int NC>
__device__ __forceinline__ void tmem_load_cols(uint32_t taddr, uint32_t (&r)[NC]) {
  static_assert(NC == 16 || NC == 32 || NC == 64, "16, 32 or 64 columns");
  if constexpr (NC == 16) {
    tmem_ld16(taddr, r);
    tmem_wait_ld16(r);
  } else if constexpr (NC == 32) {
    tmem_ld32(taddr, r);
    tmem_wait_ld32(r);
  } else {
    tmem_ld32(taddr, r);
    tmem_ld32(taddr + 32u, r + 32);
    tmem_wait_ld32(r);
    tmem_wait_ld32(r + 32);
  }
}

// Work items of a launch: (output tile, K split) pairs, n fastest, so that
// the CTAs working at the same time share A row blocks (and B) in L2.
struct GemmItem {
  int m0, n0, split, kb0, nkb;
};

__device__ __forceinline__ GemmItem gemm_item(const GemmArgs& a, int w, int bm, int bn, int tiles_n) {
  GemmItem it;
  const int splits = a.splits;
  it.split = w % splits;
  const int t = w / splits;
  it.n0 = (t % tiles_n) * bn;
  it.m0 = (t / tiles_n) * bm;
  const int nkb_total = (a.K + GM_BK - 1) / GM_BK;
  it.kb0 = it.split * a.kb_per_split;
  it.nkb = max(0, min(a.kb_per_split, nkb_total - it.kb0));
  return it;
}

// Persistent GEMM: each CTA walks the work items blockIdx.x, + gridDim.x, ...
// and every role keeps running counts over them: k-blocks g drive the stage
// ring (g % NST), promotion chains cg (PK k-blocks of one item) the
// large-product buffers (cg % NB).
//
// Accumulation.  The tensor core's fp32 accumulation rounds toward zero
// (measured on B200: with exactly representable TF32 inputs the error of a
// chain of n MMAs has a mean of about -1.3e-8 n of the output's RMS, growing
// with n).  So the large products of each chain of PK k-blocks go into a
// fresh TMEM accumulator (NB buffers in turn) and the epilogue warps add
// every chain's result into fp32 registers (round to nearest) while the next
// chains run; the correction products (2^-11 of the size) accumulate in one
// TMEM accumulator per work item (two, alternating between items, so that an
// item's store overlaps the next item's MMAs).
//
// Roles (GM_THREADS = 320): warp 0 lane 0 TMA producer, warp 1 TMEM owner and
// (lane 0) MMA issuer, warps 2..9 epilogue: warp w reads TMEM lane quarter
// w % 4 and column half (w - 2) / 4 of the tile.
//
// PAIR (launched as clusters of 2 CTAs): the pair walks 256 x BN work items,
// item w for cluster blockIdx.x / 2.  Each CTA's producer loads its 128 A rows
// and its BN / 2 rows of B into its own ring, counting the bytes on the
// leader's (rank 0) full barrier; only the leader's MMA thread issues, with
// cta_group::2 MMAs whose commits arrive on the barrier of both CTAs (stage
// free, chain ready); both CTAs' epilogues read their own TMEM rows and
// report a drained buffer on the leader's barriers (16 warps).
template <int BN, bool A_MN, bool B_MN, bool PAIR = false>
__global__ void __launch_bounds__(GM_THREADS, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                       const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
                       const GemmArgs args, int* __restrict__ status) {
  using Cfg = GemmCfg<BN, PAIR>;
  constexpr int BM = Cfg::BM, BROWS = Cfg::BROWS;
  constexpr int EPI_ARRIVALS = GM_EPI_WARPS * (PAIR ? 2 : 1);
  constexpr int NST = Cfg::NST;
  constexpr int HC = BN / 2;  // columns per epilogue warp
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smb = reinterpret_cast<unsigned char*>(smem_align1024(smem_raw));
  uint64_t* full = reinterpret_cast<uint64_t*>(smb + Cfg::OFF_BAR);
  uint64_t* empty = full + NST;
  constexpr int NB = Cfg::NB, PK = Cfg::PK;
  uint64_t* accf = empty + NST;  // [NB]: a chain's large products ready in buffer b
  uint64_t* acce = accf + NB;    // [NB]: large-product buffer b drained by the 8 epilogue warps
  uint64_t* sme = acce + NB;     // [2]: correction buffer c drained by the 8 epilogue warps
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sme + 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sme + 2) + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_n = (args.N + BN - 1) / BN;
  const int tiles_m = (args.M + BM - 1) / BM;
  const int items = tiles_m * tiles_n * args.splits;
  // this CTA's first work item and stride (a pair shares its items), its rank in the pair
  const int w0 = PAIR ? int(blockIdx.x >> 1) : int(blockIdx.x);
  const int wstep = PAIR ? int(gridDim.x >> 1) : int(gridDim.x);
  const uint32_t rank = PAIR ? cluster_rank() : 0u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], EPI_ARRIVALS);
    }
    for (int c = 0; c < 2; ++c) mbar_init(&sme[c], EPI_ARRIVALS);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    if constexpr (PAIR)
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    else
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_fence_before_sync();
  }
  __syncthreads();
  // a pair: both CTAs' barriers are initialised before any commit or load reaches them
  if constexpr (PAIR) cluster_sync_all();
  tmem_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  // TMEM columns: large-product buffers at 0 and BN, correction buffers at 2 BN and 3 BN

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    prefetch_tmap(&ta_hi);
    prefetch_tmap(&ta_lo);
    prefetch_tmap(&tb_hi);
    prefetch_tmap(&tb_lo);
    int g = 0;
    bool ok = true;
    for (int w = w0; w < items && ok; w += wstep) {
      const GemmItem it = gemm_item(args, w, BM, BN, tiles_n);
      // this CTA's A rows and B rows
      const int am0 = it.m0 + GM_BM * int(rank), bn0 = it.n0 + BROWS * int(rank);
      const int nba = gemm_nbox<GM_BM, A_MN>(am0, args.M), nbb = gemm_nbox<BROWS, B_MN>(bn0, args.N);
      // bytes landing per stage on the (leader's) full barrier: hi + lo of
      // every box the pair issues (32 x 32 fp32 = 4 KB)
      int boxes = nba + nbb;
      if constexpr (PAIR)
        boxes = gemm_nbox<GM_BM, A_MN>(it.m0, args.M) + gemm_nbox<GM_BM, A_MN>(it.m0 + GM_BM, args.M) +
                gemm_nbox<BROWS, B_MN>(it.n0, args.N) + gemm_nbox<BROWS, B_MN>(it.n0 + BROWS, args.N);
      const uint32_t tx = 2u * 4096u * uint32_t(boxes);
      for (int i = 0; i < it.nkb; ++i, ++g) {
        const int s = g % NST;
        if (g >= NST && !mbar_wait<true>(&empty[s], uint32_t((g / NST) - 1) & 1u, abort_flag, status)) {
          ok = false;
          break;
        }
        unsigned char* st = smb + s * Cfg::STAGE_B;
        if (rank == 0) mbar_arrive_expect_tx(&full[s], tx);
        const uint32_t full_c = PAIR ? cluster_addr(&full[s], 0) : 0u;
        const int k0 = (it.kb0 + i) * GM_BK;
        gemm_load_operand<GM_BM, A_MN, PAIR>(st, st + Cfg::OFF_ALO, &ta_hi, &ta_lo, &full[s], full_c, am0, k0, nba);
        gemm_load_operand<BROWS, B_MN, PAIR>(st + Cfg::OFF_BHI, st + Cfg::OFF_BLO, &tb_hi, &tb_lo, &full[s], full_c,
                                             bn0, k0, nbb);
      }
    }
    // Drain: the last load of every stage has landed before the CTA may exit
    // (on the normal path the MMA warp consumed them all already).  A pair's
    // loads all count on the leader's barriers, so the leader drains for both
    // (the final cluster barrier keeps the peer until then).
    if (rank == 0)
      for (int i = max(0, g - NST); i < g; ++i)
        (void)mbar_wait<true>(&full[i % NST], uint32_t(i / NST) & 1u, abort_flag, status);
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ---- MMA issuer (a pair's leader) ----
    constexpr uint32_t idesc = umma_idesc_tf32(BN, A_MN, B_MN, BM);
    // Operand descriptors of stage 0, K step 0: a stage or K step moves only the
    // 14-bit start-address field (shared addresses < 256 KB, so the addition
    // never carries out of it), which saves rebuilding 4 descriptors per K step
    // in the one thread that issues every MMA (measured 2-4 % faster GEMMs).
    const uint32_t st0 = smem_u32(smb);
    const uint64_t D_ahi = gemm_desc<A_MN>(st0, 0), D_alo = gemm_desc<A_MN>(st0 + Cfg::OFF_ALO, 0);
    const uint64_t D_bhi = gemm_desc<B_MN>(st0 + Cfg::OFF_BHI, 0), D_blo = gemm_desc<B_MN>(st0 + Cfg::OFF_BLO, 0);
    constexpr uint32_t KS_A = (A_MN ? 1024u : 32u) >> 4, KS_B = (B_MN ? 1024u : 32u) >> 4;
    int g = 0, cg = 0, j = 0;  // k-blocks, promotion chains, items so far
    bool ok = true;
    for (int w = w0; w < items && ok; w += wstep, ++j) {
      const GemmItem it = gemm_item(args, w, BM, BN, tiles_n);
      const int c = j & 1;
      // correction buffer c last held item j - 2: wait until the epilogue read it
      if (j >= 2 && !mbar_wait<false, PAIR>(&sme[c], uint32_t((j >> 1) - 1) & 1u, abort_flag, status)) break;
      const uint32_t d_small = tmem_base + uint32_t((NB + c) * BN);
      for (int i = 0; i < it.nkb; ++i, ++g) {
        const int s = g % NST, b = cg % NB, ci = i % PK;
        // a chain's first k-block: buffer b last held chain cg - NB; wait until the epilogue read it
        if (ci == 0 && cg >= NB &&
            !mbar_wait<false, PAIR>(&acce[b], uint32_t((cg / NB) - 1) & 1u, abort_flag, status)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&full[s], uint32_t(g / NST) & 1u, abort_flag, status)) {
          ok = false;
          break;
        }
        tmem_fence_after_sync();
        const uint64_t so = uint64_t(uint32_t(s) * uint32_t(Cfg::STAGE_B >> 4));
        const uint32_t d_big = tmem_base + uint32_t(b * BN);
#pragma unroll
        for (int kk = 0; kk < GM_BK / 8; ++kk) {
          const uint64_t ahi = D_ahi + so + kk * KS_A, alo = D_alo + so + kk * KS_A;
          const uint64_t bhi = D_bhi + so + kk * KS_B, blo = D_blo + so + kk * KS_B;
          if constexpr (PAIR) {
            umma_tf32_pair(d_big, ahi, bhi, idesc, (ci > 0 || kk > 0) ? 1u : 0u);
            umma_tf32_pair(d_small, ahi, blo, idesc, (i > 0 || kk > 0) ? 1u : 0u);
            umma_tf32_pair(d_small, alo, bhi, idesc, 1u);
          } else {
            umma_tf32(d_big, ahi, bhi, idesc, (ci > 0 || kk > 0) ? 1u : 0u);
            umma_tf32(d_small, ahi, blo, idesc, (i > 0 || kk > 0) ? 1u : 0u);
            umma_tf32(d_small, alo, bhi, idesc, 1u);
          }
        }
        // the stage is free once these MMAs have read it
        if constexpr (PAIR)
          umma_commit_pair(&empty[s]);
        else
          umma_commit(&empty[s]);
        if (ci == PK - 1 || i == it.nkb - 1) {
          // buffer b holds this chain's large products
          if constexpr (PAIR)
            umma_commit_pair(&accf[b]);
          else
            umma_commit(&accf[b]);
          ++cg;
        }
      }
    }
  } else if (warp >= GM_EPI_WARP0) {
    // ---- epilogue: per k-block TMEM -> fp32 registers, per item the tile -> global ----
    const int q = warp & 3;                          // TMEM lane quarter
    const int h = (warp - GM_EPI_WARP0) >> 2;        // column half
    const uint32_t lane_addr = tmem_base + (uint32_t(32 * q) << 16) + uint32_t(h * HC);
    const bool vec = (args.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(args.C) & 15u) == 0) &&
                     (args.split_stride % 4 == 0);
    int cg = 0, j = 0;  // promotion chains, items so far
    bool ok = true;
    for (int w = w0; w < items && ok; w += wstep, ++j) {
      const GemmItem it = gemm_item(args, w, BM, BN, tiles_n);
      float acc[HC];
#pragma unroll
      for (int x = 0; x < HC; ++x) acc[x] = 0.f;
      const int nch = (it.nkb + PK - 1) / PK;
      for (int ch = 0; ch < nch; ++ch, ++cg) {
        const int b = cg % NB;
        ok = __all_sync(0xffffffffu, mbar_wait(&accf[b], uint32_t(cg / NB) & 1u, abort_flag, status));
        if (!ok) break;
        tmem_fence_after_sync();
        uint32_t r[HC];
        tmem_load_cols<HC>(lane_addr + uint32_t(b * BN), r);
#pragma unroll
        for (int x = 0; x < HC; ++x) acc[x] += __uint_as_float(r[x]);
        tmem_fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR)
            mbar_arrive_cluster(cluster_addr(&acce[b], 0));  // the leader's
          else
            mbar_arrive(&acce[b]);
        }
      }
      if (!ok || it.nkb == 0) break;
      // the item's last chain commit also covered all of its correction-product MMAs
      const int c = j & 1;
      uint32_t r[HC];
      tmem_load_cols<HC>(lane_addr + uint32_t((NB + c) * BN), r);
      tmem_fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(cluster_addr(&sme[c], 0));
        else
          mbar_arrive(&sme[c]);
      }
      const int mrow0 = it.m0 + GM_BM * int(rank) + 32 * q;  // this warp's first output row
      const int row = mrow0 + lane;
      float* tile = args.C + int64_t(it.split) * args.split_stride;
      const int col0 = it.n0 + h * HC;
      if (vec && col0 + HC <= args.N) {
        // Through the warp's staging tile, SC columns per pass: lane l writes
        // row l, then each store instruction covers 32 / TPR whole row pieces
        // of SC * 4 bytes (rows strided by ldc) instead of 32 rows x 16 bytes.
        // 16-byte chunk k of row r sits at chunk k ^ ((r / RPL) % TPR), so both
        // the row-wise writes and the piece-wise reads hit distinct banks in
        // every 8-lane phase.
        constexpr int SC = Cfg::EPI_SC, TPR = SC / 4, RPL = 8 / TPR;
        float* st = reinterpret_cast<float*>(smb + Cfg::OFF_EPI) + (warp - GM_EPI_WARP0) * 32 * SC;
#pragma unroll
        for (int p = 0; p < HC; p += SC) {
#pragma unroll
          for (int k = 0; k < TPR; ++k) {
            const int x = p + 4 * k;
            float4 v;
            v.x = acc[x] + __uint_as_float(r[x]);
            v.y = acc[x + 1] + __uint_as_float(r[x + 1]);
            v.z = acc[x + 2] + __uint_as_float(r[x + 2]);
            v.w = acc[x + 3] + __uint_as_float(r[x + 3]);
            reinterpret_cast<float4*>(st + lane * SC)[k ^ ((lane / RPL) & (TPR - 1))] = v;
          }
          __syncwarp();
          const int k = lane % TPR;
          // C += A B: the pass's old values are all loaded before its first
          // store (a load placed after a store through the same pointer
          // would wait for it: one global round trip per row piece)
          float4 old[TPR];
          if (args.accumulate) {
#pragma unroll
            for (int i = 0; i < TPR; ++i) {
              const int grow = mrow0 + i * (32 / TPR) + lane / TPR;
              old[i] = grow < args.M ? *reinterpret_cast<const float4*>(tile + int64_t(grow) * args.ldc + col0 + p +
                                                                         4 * k)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
#pragma unroll
          for (int i = 0; i < TPR; ++i) {
            const int rr = i * (32 / TPR) + lane / TPR;
            float4 v = reinterpret_cast<const float4*>(st + rr * SC)[k ^ ((rr / RPL) & (TPR - 1))];
            const int grow = mrow0 + rr;
            if (grow < args.M) {
              float4* dst = reinterpret_cast<float4*>(tile + int64_t(grow) * args.ldc + col0 + p + 4 * k);
              if (args.accumulate) {
                v.x += old[i].x;
                v.y += old[i].y;
                v.z += old[i].z;
                v.w += old[i].w;
              }
              *dst = v;
            }
          }
          __syncwarp();
        }
      } else {
        if (row >= args.M) continue;
        float* out = tile + int64_t(row) * args.ldc;
#pragma unroll
        for (int x = 0; x < HC; ++x)
          if (col0 + x < args.N) {
            const float v = acc[x] + __uint_as_float(r[x]);
            out[col0 + x] = args.accumulate ? out[col0 + x] + v : v;
          }
      }
    }
  }
  tmem_fence_before_sync();
  __syncthreads();
  // a pair: the leader's MMAs read the peer's shared memory and write its
  // TMEM, and the peer's loads and arrivals reach the leader's barriers; both
  // stay until the other is done
  if constexpr (PAIR) cluster_sync_all();
  if (warp == 1) {
    tmem_fence_after_sync();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// Sums the K-split partials in split order: C = sum_s P_s (P_s: M x N, row
// stride N, split_stride apart), or C += that sum.
__global__ void gemm_splitk_reduce_kernel(const float* __restrict__ part, float* __restrict__ C, int64_t ldc, int M,
                                          int N, int splits, int64_t split_stride, int accumulate) {
  const int64_t total = int64_t(M) * N;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    float acc = part[i];
    for (int s = 1; s < splits; ++s) acc += part[int64_t(s) * split_stride + i];
    const int64_t m = i / N, n = i % N;
    C[m * ldc + n] = accumulate ? C[m * ldc + n] + acc : acc;
  }
}

}  // namespace vmscan
