// vmscan.cu — C ABI of libvmscan.so (declared in include/vmscan.h).
//
// Host side of the selective-scan hot path: argument validation, the scan
// geometry of a direction, TMA tensor-map encoding (the direction lives in
// the maps' dims and strides) and kernel launches.  No allocation, no stream
// synchronisation (except vmscan_device_status), no global state besides the
// driver entry point and the sticky device status word.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "../../include/vmscan.h"
#include "vmscan_bwd.cuh"
#include "vmscan_common.cuh"
#include "vmscan_conv.cuh"
#include "vmscan_dt.cuh"
#include "vmscan_fwd.cuh"
#include "vmscan_gemm.cuh"
#include "vmscan_norm.cuh"

using namespace vmscan;

// Sticky device status: kernels set it when a bounded wait gives up.
__device__ int g_vmscan_status = 0;

// Scratch of vmscan_bwd_noalloc (see include/vmscan.h).  Host code only ever
// uses its per-device address from cudaGetSymbolAddress, never the symbol.
static __device__ __align__(256) unsigned char g_vmscan_noalloc_scratch[VMSCAN_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kFwdNCW = 4;


// Driver entry points, resolved once through the runtime (no link-time libcuda).
struct DriverFns {
  PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  PFN_cuCtxGetCurrent_v4000 ctx_get = nullptr;
  PFN_cuCtxSetCurrent_v4000 ctx_set = nullptr;
  PFN_cuPointerGetAttribute_v4000 ptr_attr = nullptr;
};

template <typename F>
void resolve(const char* name, int version, F& out) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion(name, &p, version, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    out = reinterpret_cast<F>(p);
}

const DriverFns& driver() {
  static DriverFns fns;
  static std::once_flag once;
  std::call_once(once, [] {
    resolve("cuTensorMapEncodeTiled", 12000, fns.encode);
    resolve("cuCtxGetCurrent", 4000, fns.ctx_get);
    resolve("cuCtxSetCurrent", 4000, fns.ctx_set);
    resolve("cuPointerGetAttribute", 4000, fns.ptr_attr);
  });
  return fns;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() { return driver().encode; }

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

// The C ABI can be called from a thread on which no CUDA context is current
// yet (e.g. PyTorch's autograd worker thread).  Driver calls such as the
// tensor-map encoder need one, so bind the context that owns the caller's
// device buffer when the thread has none.  A context that is already current
// is left untouched.
int ensure_context(const void* devptr) {
  const DriverFns& d = driver();
  if (d.ctx_get == nullptr || d.ctx_set == nullptr || d.ptr_attr == nullptr)
    return fail(VMSCAN_ERR_DRIVER, "CUDA driver entry points unavailable");
  CUcontext cur = nullptr;
  if (d.ctx_get(&cur) == CUDA_SUCCESS && cur != nullptr) return VMSCAN_OK;
  CUcontext owner = nullptr;
  const CUresult r = d.ptr_attr(&owner, CU_POINTER_ATTRIBUTE_CONTEXT, reinterpret_cast<CUdeviceptr>(devptr));
  if (r != CUDA_SUCCESS || owner == nullptr)
    return fail(VMSCAN_ERR_DRIVER, "no current CUDA context and buffer %p has no owning context (CUresult %d)",
                devptr, int(r));
  if (d.ctx_set(owner) != CUDA_SUCCESS) return fail(VMSCAN_ERR_DRIVER, "cuCtxSetCurrent failed");
  return VMSCAN_OK;
}

int* status_ptr() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_vmscan_status) != cudaSuccess) return nullptr;
  return static_cast<int*>(p);
}

struct ScanDim {
  int64_t size;
  int64_t tstride;
};

// Builds the scan geometry of `dir` for a sequence of `seqlen` tokens.
int make_geom(int64_t batch, int64_t seqlen, int64_t d_inner, const vmscan_direction* dir, ScanGeom& g) {
  if (batch <= 0 || seqlen <= 0 || d_inner <= 0) return VMSCAN_ERR_SHAPE;
  if (batch > 65535 || seqlen > (int64_t(1) << 30) || d_inner > (int64_t(1) << 24)) return VMSCAN_ERR_SHAPE;
  ScanDim dims[4];
  int nd = 0;
  if (dir == nullptr || dir->ndim == 0) {
    dims[nd++] = {seqlen, 1};
  } else {
    const int n = dir->ndim;
    if (n < 1 || n > 4) return VMSCAN_ERR_DIRECTION;
    int64_t prod = 1;
    bool seen[4] = {false, false, false, false};
    for (int i = 0; i < n; ++i) {
      if (dir->grid[i] < 1) return VMSCAN_ERR_DIRECTION;
      prod *= dir->grid[i];
      const int a = dir->axes[i];
      if (a < 0 || a >= n || seen[a]) return VMSCAN_ERR_DIRECTION;
      seen[a] = true;
    }
    if (prod != seqlen) return VMSCAN_ERR_DIRECTION;
    int64_t ts[4];
    int64_t acc = 1;
    for (int i = n - 1; i >= 0; --i) {
      ts[i] = acc;
      acc *= dir->grid[i];
    }
    // fastest scan dim first; drop unit dims; merge dims contiguous in token order
    for (int q = n - 1; q >= 0; --q) {
      const int a = dir->axes[q];
      const ScanDim sd = {dir->grid[a], ts[a]};
      if (sd.size == 1) continue;
      if (nd > 0 && sd.tstride == dims[nd - 1].tstride * dims[nd - 1].size) {
        dims[nd - 1].size *= sd.size;
      } else {
        dims[nd++] = sd;
      }
    }
    if (nd == 0) dims[nd++] = {1, 1};
  }
  if (nd > 3) return VMSCAN_ERR_DIRECTION;
  g.nsd = nd;
  for (int i = 0; i < 3; ++i) {
    g.size[i] = i < nd ? int32_t(dims[i].size) : 1;
    g.tstride[i] = i < nd ? dims[i].tstride : 0;
  }
  int64_t P = 1;
  int j = nd - 1;
  for (int i = 0; i < nd; ++i) {
    if (i < nd - 1 && P * g.size[i] <= TMAX) {
      P *= g.size[i];
      continue;
    }
    j = i;
    break;
  }
  const int64_t bj = std::min<int64_t>(g.size[j], TMAX / P);
  g.j = j;
  g.bj = int32_t(bj);
  g.nj = int32_t((g.size[j] + bj - 1) / bj);
  g.P = int32_t(P);
  g.T = int32_t(P * bj);
  int64_t nb = g.nj;
  for (int i = j + 1; i < nd; ++i) nb *= g.size[i];
  if (nb > (int64_t(1) << 30)) return VMSCAN_ERR_SHAPE;
  g.nboxes = int32_t(nb);
  g.reverse = (dir != nullptr && dir->reverse) ? 1 : 0;
  g.batch = int32_t(batch);
  g.d_inner = int32_t(d_inner);
  g.seqlen = int32_t(seqlen);
  return VMSCAN_OK;
}

void box_extent(const ScanGeom& g, cuuint32_t box[3]) {
  for (int i = 0; i < 3; ++i) box[i] = (i < g.j) ? cuuint32_t(g.size[i]) : (i == g.j ? cuuint32_t(g.bj) : 1u);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Output tensors are written with plain stores at (token * seq stride); the
// kernels take that stride as a 32-bit int so the address is one wide
// multiply-add.
int seq_stride32(const char* what, vmscan_strides s, int64_t seqlen, int& out) {
  if (seqlen > 1 && (s.seq <= 0 || s.seq > INT32_MAX))
    return fail(VMSCAN_ERR_SHAPE, "%s seq stride %lld must be in 1..2^31-1", what, (long long)s.seq);
  out = int(seqlen > 1 ? s.seq : 0);
  return VMSCAN_OK;
}

// Tensor map of a (batch, seq, inner) view of esize-byte elements (4: fp32,
// 2: bf16) seen in scan order: dims {inner, scan0, scan1, scan2, batch}, box
// {box_inner, box...}.  Strides must be whole 16-byte multiples.
int encode_map(CUtensorMap* m, const char* what, const void* ptr, int64_t inner, int box_inner,
               vmscan_strides st, const ScanGeom& g, int esize) {
  if (ptr == nullptr) return fail(VMSCAN_ERR_NULL, "%s is NULL", what);
  if (!aligned16(ptr)) return fail(VMSCAN_ERR_ALIGN, "%s base %p is not 16-byte aligned", what, ptr);
  const int64_t q = 16 / esize;
  if ((g.seqlen > 1 && (st.seq <= 0 || st.seq % q != 0)) || (g.batch > 1 && (st.batch <= 0 || st.batch % q != 0)))
    return fail(VMSCAN_ERR_ALIGN, "%s strides {batch %lld, seq %lld} must be positive multiples of %lld", what,
                (long long)st.batch, (long long)st.seq, (long long)q);
  auto fn = encode_fn();
  if (fn == nullptr) return fail(VMSCAN_ERR_DRIVER, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[5];
  cuuint64_t strides[4];
  dims[0] = cuuint64_t(inner);
  for (int i = 0; i < 3; ++i) {
    dims[1 + i] = cuuint64_t(g.size[i]);
    int64_t s = (i < g.nsd && g.size[i] > 1) ? g.tstride[i] * st.seq * esize : 16;
    strides[i] = cuuint64_t(s);
  }
  dims[4] = cuuint64_t(g.batch);
  strides[3] = cuuint64_t(g.batch > 1 ? st.batch * esize : 16);
  for (int i = 0; i < 4; ++i)
    if (strides[i] == 0 || strides[i] % 16 != 0 || strides[i] >= (cuuint64_t(1) << 40))
      return fail(VMSCAN_ERR_ALIGN, "%s byte stride %llu of dim %d is invalid", what, (unsigned long long)strides[i],
                  i + 1);
  cuuint32_t box3[3];
  box_extent(g, box3);
  cuuint32_t box[5] = {cuuint32_t(box_inner), box3[0], box3[1], box3[2], 1u};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUtensorMapDataType dtype = esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = fn(m, dtype, 5, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(VMSCAN_ERR_DRIVER,
                "cuTensorMapEncodeTiled(%s) -> CUresult %d; dims {%llu,%llu,%llu,%llu,%llu} strides "
                "{%llu,%llu,%llu,%llu} box {%u,%u,%u,%u,%u}",
                what, int(r), (unsigned long long)dims[0], (unsigned long long)dims[1], (unsigned long long)dims[2],
                (unsigned long long)dims[3], (unsigned long long)dims[4], (unsigned long long)strides[0],
                (unsigned long long)strides[1], (unsigned long long)strides[2], (unsigned long long)strides[3],
                box[0], box[1], box[2], box[3], box[4]);
  return VMSCAN_OK;
}

#define VM_TRY(expr)                 \
  do {                               \
    const int _rc = (expr);          \
    if (_rc != VMSCAN_OK) return _rc; \
  } while (0)

int check_launch() {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return VMSCAN_OK;
  return fail(VMSCAN_ERR_LAUNCH, "kernel launch failed: %s", cudaGetErrorString(e));
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct BwdWorkspace {
  int nc, bpc;  // chunks over L and boxes per chunk
  size_t part, wA, wD, p_local, carry_s, p_in, ck, fws, total;
};

int sm_count();
int scan_chunks(int64_t ctas, int64_t slots, int nboxes, int min_boxes);
size_t fwd_chunk_bytes(const ScanGeom& g);

// VJP workspace: dB/dC partials per (batch, box, channel tile); dA/dD
// partials per (batch, chunk); the adjoint carries of a chunked VJP; and,
// when the VJP rebuilds the checkpoints, their buffer and the forward's
// chunk carries.
BwdWorkspace bwd_layout(const ScanGeom& g, int ndt, bool with_ck) {
  BwdWorkspace w;
  w.nc = scan_chunks(int64_t(g.batch) * ndt, int64_t(sm_count()) * 2, g.nboxes, 2);
  w.bpc = (g.nboxes + w.nc - 1) / w.nc;
  const size_t rows = size_t(g.batch) * w.nc * g.d_inner;
  w.part = 0;
  const size_t part_bytes = size_t(g.batch) * g.nboxes * ndt * TMAX * kPartRow * 4;
  w.wA = align256(w.part + part_bytes);
  w.wD = align256(w.wA + rows * NS * 4);
  w.p_local = align256(w.wD + rows * 4);
  const size_t carry = w.nc > 1 ? rows * NS * 4 : 0;
  w.carry_s = align256(w.p_local + carry);
  w.p_in = align256(w.carry_s + (w.nc > 1 ? rows * 4 : 0));
  w.ck = align256(w.p_in + carry);
  const size_t ck_bytes = with_ck ? size_t(g.batch) * g.nboxes * g.d_inner * NS * 4 : 0;
  w.fws = align256(w.ck + ck_bytes);
  w.total = align256(w.fws + (with_ck ? fwd_chunk_bytes(g) : 0));
  return w;
}

// SMs of the current device (cached per device).
int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int n = 0;
    cache[dev] = (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0) ? n : 148;
  }
  return cache[dev];
}

// Number of chunks over L for a scan whose unchunked grid has `ctas` CTAs
// when `slots` CTAs fit on the GPU at once: 1 while the grid fills at least
// half the slots (chunking costs an extra pass), otherwise enough chunks to
// fill them, each chunk at least `min_boxes` boxes, at most 32 chunks.
int scan_chunks(int64_t ctas, int64_t slots, int nboxes, int min_boxes) {
  if (ctas * 2 >= slots) return 1;
  int nc = int(std::min<int64_t>(slots / ctas, 32));
  nc = std::min(nc, nboxes / min_boxes);
  if (nc < 2) return 1;
  const int bpc = (nboxes + nc - 1) / nc;
  return (nboxes + bpc - 1) / bpc;
}

struct ChunkPlan {
  int nc, bpc;
  size_t bytes;  // workspace for the carries (0 when nc == 1)
};

ChunkPlan fwd_chunk_plan(const ScanGeom& g) {
  using Cfg = FwdCfg<kFwdNCW>;
  const int64_t tiles = (g.d_inner + Cfg::DT - 1) / Cfg::DT;
  // the forward's carry pass and extra launches cost more than they save on
  // chunks shorter than 8 boxes (measured at L = 196)
  const int nc = scan_chunks(int64_t(g.batch) * tiles, int64_t(sm_count()) * 4, g.nboxes, 8);
  const size_t per = size_t(g.batch) * nc * g.d_inner;
  return {nc, (g.nboxes + nc - 1) / nc, nc > 1 ? 2 * align256(per * NS * 4) + align256(per * 4) : 0};
}

size_t fwd_chunk_bytes(const ScanGeom& g) { return fwd_chunk_plan(g).bytes; }

template <typename T, bool HAS_Z, bool SAVE_CK, bool STORE_Y, bool REV, bool CARRY>
int launch_fwd_t(const CUtensorMap& mu, const CUtensorMap& mdt, const CUtensorMap& mz, const CUtensorMap& mB,
                 const CUtensorMap& mC, T* y, vmscan_strides sy, float* y_lo, const float* A, const float* D,
                 float* ckpt, const ChunkArgs& ch, int nz, const ScanGeom& g, cudaStream_t stream) {
  using Cfg = FwdCfg<kFwdNCW, T>;
  auto kern = scan_fwd_kernel<kFwdNCW, T, HAS_Z, SAVE_CK, STORE_Y, REV, CARRY>;
  // y as TF32 parts: its own instantiation (fp32 outputs of a main pass only)
  if constexpr (std::is_same<T, float>::value && STORE_Y && !CARRY) {
    if (y_lo != nullptr) kern = scan_fwd_kernel<kFwdNCW, T, HAS_Z, SAVE_CK, STORE_Y, REV, CARRY, true>;
  }
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Cfg::SMEM_BYTES)) != cudaSuccess)
    return fail(VMSCAN_ERR_LAUNCH, "cudaFuncSetAttribute(scan_fwd_kernel) failed");
  int* st = status_ptr();
  if (st == nullptr) return fail(VMSCAN_ERR_LAUNCH, "status symbol unavailable");
  int sys = 0;
  if (STORE_Y) VM_TRY(seq_stride32("y", sy, g.seqlen, sys));
  const dim3 grid(unsigned((g.d_inner + Cfg::DT - 1) / Cfg::DT), unsigned(g.batch), unsigned(nz));
  kern<<<grid, Cfg::NT, Cfg::SMEM_BYTES, stream>>>(mu, mdt, mz, mB, mC, y, sy.batch, sys, y_lo, A, D, ckpt, ch, g,
                                                   st);
  return check_launch();
}

// Forward scan, chunked over L when the grid would leave most of the GPU idle
// and `ws` (fwd_chunk_plan(g).bytes) is given: a carry pass over chunks
// 0 .. nc-2, the carry chain, then the main pass over all chunks.
template <typename T, bool HAS_Z, bool SAVE_CK, bool STORE_Y, bool REV>
int run_fwd_t(const CUtensorMap& mu, const CUtensorMap& mdt, const CUtensorMap& mz, const CUtensorMap& mB,
              const CUtensorMap& mC, T* y, vmscan_strides sy, float* y_lo, const float* A, const float* D,
              float* ckpt, void* ws, size_t ws_bytes, const ScanGeom& g, cudaStream_t stream) {
  const ChunkPlan plan = fwd_chunk_plan(g);
  if (plan.nc == 1 || ws == nullptr || ws_bytes < plan.bytes) {
    const ChunkArgs one{g.nboxes, 1, nullptr, nullptr, nullptr};
    return launch_fwd_t<T, HAS_Z, SAVE_CK, STORE_Y, REV, false>(mu, mdt, mz, mB, mC, y, sy, y_lo, A, D, ckpt, one,
                                                                1, g, stream);
  }
  const size_t per = size_t(g.batch) * plan.nc * g.d_inner;
  char* w = static_cast<char*>(ws);
  float* carry_h = reinterpret_cast<float*>(w);
  float* h_start = reinterpret_cast<float*>(w + align256(per * NS * 4));
  float* carry_s = reinterpret_cast<float*>(w + 2 * align256(per * NS * 4));
  const ChunkArgs ch{plan.bpc, plan.nc, h_start, carry_h, carry_s};
  VM_TRY((launch_fwd_t<T, false, false, false, REV, true>(mu, mdt, mz, mB, mC, nullptr, vmscan_strides{0, 0},
                                                         nullptr, A, D, nullptr, ch, plan.nc - 1, g, stream)));
  const int64_t n = int64_t(g.batch) * g.d_inner * NS;
  carry_fwd_kernel<<<unsigned((n + 255) / 256), 256, 0, stream>>>(A, carry_h, carry_s, h_start, g.batch, plan.nc,
                                                                  g.d_inner);
  VM_TRY(check_launch());
  return launch_fwd_t<T, HAS_Z, SAVE_CK, STORE_Y, REV, false>(mu, mdt, mz, mB, mC, y, sy, y_lo, A, D, ckpt, ch,
                                                              plan.nc, g, stream);
}

template <typename T, bool HAS_Z, bool SAVE_CK, bool STORE_Y>
int launch_fwd(const CUtensorMap& mu, const CUtensorMap& mdt, const CUtensorMap& mz, const CUtensorMap& mB,
               const CUtensorMap& mC, T* y, vmscan_strides sy, float* y_lo, const float* A, const float* D,
               float* ckpt, void* ws, size_t ws_bytes, const ScanGeom& g, cudaStream_t stream) {
  if (g.reverse)
    return run_fwd_t<T, HAS_Z, SAVE_CK, STORE_Y, true>(mu, mdt, mz, mB, mC, y, sy, y_lo, A, D, ckpt, ws, ws_bytes,
                                                       g, stream);
  return run_fwd_t<T, HAS_Z, SAVE_CK, STORE_Y, false>(mu, mdt, mz, mB, mC, y, sy, y_lo, A, D, ckpt, ws, ws_bytes,
                                                      g, stream);
}

template <typename T>
struct BwdOut {
  T* du;
  vmscan_strides sdu;
  T* ddt;
  vmscan_strides sddt;
  T* dz;
  vmscan_strides sdz;
  float* dz_lo;  // fp32 only: dz as TF32 parts (hi into dz) when not NULL
};

template <typename T, bool HAS_Z, bool REV>
int launch_bwd_t(const CUtensorMap& mu, const CUtensorMap& mdt, const CUtensorMap& mz, const CUtensorMap& mdy,
                 const CUtensorMap& mB, const CUtensorMap& mC, const BwdOut<T>& o, const float* A, const float* D,
                 const float* ckpt, float* wpart, float* wA, float* wD, const BwdWorkspace& wl, char* ws,
                 const ScanGeom& g, cudaStream_t stream) {
  using Cfg = BwdCfg<T>;
  int* st = status_ptr();
  if (st == nullptr) return fail(VMSCAN_ERR_LAUNCH, "status symbol unavailable");
  const unsigned ndt = unsigned((g.d_inner + Cfg::DT - 1) / Cfg::DT);
  float* p_in = nullptr;
  if (wl.nc > 1) {
    // adjoint carries of the chunks, then their chain
    using CC = BwdCarryCfg<T>;
    auto ck = scan_bwd_carry_kernel<T, HAS_Z, REV>;
    if (cudaFuncSetAttribute(ck, cudaFuncAttributeMaxDynamicSharedMemorySize, int(CC::SMEM_BYTES)) != cudaSuccess)
      return fail(VMSCAN_ERR_LAUNCH, "cudaFuncSetAttribute(scan_bwd_carry_kernel) failed");
    float* p_local = reinterpret_cast<float*>(ws + wl.p_local);
    float* carry_s = reinterpret_cast<float*>(ws + wl.carry_s);
    p_in = reinterpret_cast<float*>(ws + wl.p_in);
    ck<<<dim3(ndt, unsigned(g.batch), unsigned(wl.nc - 1)), CC::NT, CC::SMEM_BYTES, stream>>>(
        mdt, mz, mdy, mC, A, p_local, carry_s, wl.bpc, wl.nc, g, st);
    VM_TRY(check_launch());
    const int64_t n = int64_t(g.batch) * g.d_inner * NS;
    carry_bwd_kernel<<<unsigned((n + 255) / 256), 256, 0, stream>>>(A, p_local, carry_s, p_in, g.batch, wl.nc,
                                                                    g.d_inner);
    VM_TRY(check_launch());
  }
  auto kern = scan_bwd_kernel<T, HAS_Z, REV>;
  // dz as TF32 parts: its own instantiation (gated fp32 VJP only)
  if constexpr (std::is_same<T, float>::value && HAS_Z) {
    if (o.dz_lo != nullptr) kern = scan_bwd_kernel<T, HAS_Z, REV, true>;
  }
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Cfg::SMEM_BYTES)) != cudaSuccess)
    return fail(VMSCAN_ERR_LAUNCH, "cudaFuncSetAttribute(scan_bwd_kernel) failed");
  int sdus = 0, sdts = 0, sdzs = 0;
  VM_TRY(seq_stride32("du", o.sdu, g.seqlen, sdus));
  VM_TRY(seq_stride32("ddelta", o.sddt, g.seqlen, sdts));
  if (HAS_Z) VM_TRY(seq_stride32("dz", o.sdz, g.seqlen, sdzs));
  const BwdChunkArgs chunk{wl.bpc, wl.nc, p_in};
  const dim3 grid(ndt, unsigned(g.batch), unsigned(wl.nc));
  kern<<<grid, Cfg::NT, Cfg::SMEM_BYTES, stream>>>(mu, mdt, mz, mdy, mB, mC, o.du, o.sdu.batch, sdus, o.ddt,
                                                   o.sddt.batch, sdts, o.dz, o.sdz.batch, sdzs, o.dz_lo, A, D, ckpt,
                                                   wpart, wA, wD, chunk, g, st);
  return check_launch();
}

template <typename T, bool HAS_Z>
int launch_bwd(const CUtensorMap& mu, const CUtensorMap& mdt, const CUtensorMap& mz, const CUtensorMap& mdy,
               const CUtensorMap& mB, const CUtensorMap& mC, const BwdOut<T>& o, const float* A, const float* D,
               const float* ckpt, float* wpart, float* wA, float* wD, const BwdWorkspace& wl, char* ws,
               const ScanGeom& g, cudaStream_t stream) {
  if (g.reverse)
    return launch_bwd_t<T, HAS_Z, true>(mu, mdt, mz, mdy, mB, mC, o, A, D, ckpt, wpart, wA, wD, wl, ws, g, stream);
  return launch_bwd_t<T, HAS_Z, false>(mu, mdt, mz, mdy, mB, mC, o, A, D, ckpt, wpart, wA, wD, wl, ws, g, stream);
}

int check_common(int64_t d_state, const float* A, const float* D) {
  if (d_state != NS) return VMSCAN_ERR_DSTATE;
  if (A == nullptr || D == nullptr) return VMSCAN_ERR_NULL;
  return VMSCAN_OK;
}

// Forward entry (fp32 or bf16 sequence tensors; A, D and the checkpoints are fp32).
template <typename T>
int fwd_impl(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state, const T* u, vmscan_strides su,
             const T* delta, vmscan_strides sdelta, const float* A, const T* B, vmscan_strides sB, const T* C,
             vmscan_strides sC, const float* D, const T* z, vmscan_strides sz, T* y, vmscan_strides sy,
             float* y_lo, float* ckpt, const vmscan_direction* dir, void* workspace, size_t workspace_bytes,
             vmscan_stream_t stream) {
  constexpr int ES = int(sizeof(T));
  VM_TRY(check_common(d_state, A, D));
  if (u == nullptr || delta == nullptr || B == nullptr || C == nullptr || y == nullptr) return VMSCAN_ERR_NULL;
  if (ckpt != nullptr && !aligned16(ckpt)) return fail(VMSCAN_ERR_ALIGN, "ckpt is not 16-byte aligned");
  if (y_lo != nullptr && ES != 4) return fail(VMSCAN_ERR_SHAPE, "y_lo (TF32 parts) needs fp32 outputs");
  ScanGeom g;
  VM_TRY(make_geom(batch, seqlen, d_inner, dir, g));
  VM_TRY(ensure_context(u));
  using Cfg = FwdCfg<kFwdNCW, T>;
  CUtensorMap mu, mdt, mz, mB, mC;
  VM_TRY(encode_map(&mu, "u", u, d_inner, Cfg::DT, su, g, ES));
  VM_TRY(encode_map(&mdt, "delta", delta, d_inner, Cfg::DT, sdelta, g, ES));
  if (z != nullptr) {
    VM_TRY(encode_map(&mz, "z", z, d_inner, Cfg::DT, sz, g, ES));
  } else {
    mz = mu;
  }
  VM_TRY(encode_map(&mB, "B", B, NS, NS, sB, g, ES));
  VM_TRY(encode_map(&mC, "C", C, NS, NS, sC, g, ES));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool hz = z != nullptr, ck = ckpt != nullptr;
  void* ws = workspace;
  const size_t wb = workspace_bytes;
  if (ws != nullptr && !aligned16(ws)) return fail(VMSCAN_ERR_ALIGN, "workspace is not 16-byte aligned");
  if (hz && ck) return launch_fwd<T, true, true, true>(mu, mdt, mz, mB, mC, y, sy, y_lo, A, D, ckpt, ws, wb, g, s);
  if (hz) return launch_fwd<T, true, false, true>(mu, mdt, mz, mB, mC, y, sy, y_lo, A, D, ckpt, ws, wb, g, s);
  if (ck) return launch_fwd<T, false, true, true>(mu, mdt, mz, mB, mC, y, sy, y_lo, A, D, ckpt, ws, wb, g, s);
  return launch_fwd<T, false, false, true>(mu, mdt, mz, mB, mC, y, sy, y_lo, A, D, ckpt, ws, wb, g, s);
}

// VJP entry (fp32 or bf16 sequence tensors and their gradients; A, D, dA,
// dD and the checkpoints are fp32).
template <typename T>
int bwd_impl(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state, const T* u, vmscan_strides su,
             const T* delta, vmscan_strides sdelta, const float* A, const T* B, vmscan_strides sB, const T* C,
             vmscan_strides sC, const float* D, const T* z, vmscan_strides sz, const float* ckpt, const T* dy,
             vmscan_strides sdy, T* du, vmscan_strides sdu, T* ddelta, vmscan_strides sddelta, float* dA, T* dB,
             vmscan_strides sdB, T* dC, vmscan_strides sdC, float* dD, T* dz, vmscan_strides sdz, float* dz_lo,
             const vmscan_direction* dir, void* workspace, size_t workspace_bytes, vmscan_stream_t stream) {
  constexpr int ES = int(sizeof(T));
  VM_TRY(check_common(d_state, A, D));
  if (u == nullptr || delta == nullptr || B == nullptr || C == nullptr || dy == nullptr || du == nullptr ||
      ddelta == nullptr || dA == nullptr || dB == nullptr || dC == nullptr || dD == nullptr)
    return VMSCAN_ERR_NULL;
  if (z != nullptr && dz == nullptr) return VMSCAN_ERR_NULL;
  if (dz_lo != nullptr && ES != 4) return fail(VMSCAN_ERR_SHAPE, "dz_lo (TF32 parts) needs fp32 outputs");
  if (ckpt != nullptr && !aligned16(ckpt)) return fail(VMSCAN_ERR_ALIGN, "ckpt is not 16-byte aligned");
  ScanGeom g;
  VM_TRY(make_geom(batch, seqlen, d_inner, dir, g));
  VM_TRY(ensure_context(u));
  using Cfg = BwdCfg<T>;
  const int ndt = int((d_inner + Cfg::DT - 1) / Cfg::DT);
  const BwdWorkspace wl = bwd_layout(g, ndt, ckpt == nullptr);
  if (workspace == nullptr || workspace_bytes < wl.total || !aligned16(workspace)) return VMSCAN_ERR_WORKSPACE;
  char* ws = static_cast<char*>(workspace);
  float* wpart = reinterpret_cast<float*>(ws + wl.part);
  float* wA = reinterpret_cast<float*>(ws + wl.wA);
  float* wD = reinterpret_cast<float*>(ws + wl.wD);
  CUtensorMap mu, mdt, mz, mdy, mB, mC;
  VM_TRY(encode_map(&mu, "u", u, d_inner, Cfg::DT, su, g, ES));
  VM_TRY(encode_map(&mdt, "delta", delta, d_inner, Cfg::DT, sdelta, g, ES));
  if (z != nullptr) {
    VM_TRY(encode_map(&mz, "z", z, d_inner, Cfg::DT, sz, g, ES));
  } else {
    mz = mu;
  }
  VM_TRY(encode_map(&mdy, "dy", dy, d_inner, Cfg::DT, sdy, g, ES));
  VM_TRY(encode_map(&mB, "B", B, NS, NS, sB, g, ES));
  VM_TRY(encode_map(&mC, "C", C, NS, NS, sC, g, ES));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const float* ck = ckpt;
  if (ck == nullptr) {
    // Rebuild the checkpoints (the reference VJP also recomputes the forward),
    // chunked over L like vmscan_fwd; the forward gets its own maps.
    using FC = FwdCfg<kFwdNCW, T>;
    CUtensorMap fu, fdt, fB;
    VM_TRY(encode_map(&fu, "u", u, d_inner, FC::DT, su, g, ES));
    VM_TRY(encode_map(&fdt, "delta", delta, d_inner, FC::DT, sdelta, g, ES));
    VM_TRY(encode_map(&fB, "B", B, NS, NS, sB, g, ES));
    float* ckw = reinterpret_cast<float*>(ws + wl.ck);
    VM_TRY((launch_fwd<T, false, true, false>(fu, fdt, fu, fB, fB, static_cast<T*>(nullptr), vmscan_strides{0, 0},
                                              nullptr, A, D, ckw, ws + wl.fws, wl.total - wl.fws, g, s)));
    ck = ckw;
  }
  const BwdOut<T> o{du, sdu, ddelta, sddelta, dz, sdz, z != nullptr ? dz_lo : nullptr};
  if (z != nullptr) {
    VM_TRY((launch_bwd<T, true>(mu, mdt, mz, mdy, mB, mC, o, A, D, ck, wpart, wA, wD, wl, ws, g, s)));
  } else {
    VM_TRY((launch_bwd<T, false>(mu, mdt, mz, mdy, mB, mC, o, A, D, ck, wpart, wA, wD, wl, ws, g, s)));
  }
  reduce_dbc_kernel<T><<<dim3(unsigned(g.nboxes), unsigned(g.batch)), TMAX * kPartRow, 0, s>>>(
      wpart, dB, sdB.batch, sdB.seq, dC, sdC.batch, sdC.seq, g, ndt);
  VM_TRY(check_launch());
  const int nA = int(d_inner * NS);
  reduce_dad_kernel<<<unsigned((nA + 255) / 256), 256, 0, s>>>(wA, wD, dA, dD, int(batch) * wl.nc, int(d_inner));
  return check_launch();
}

}  // namespace

namespace {

template <bool BWD>
int launch_dt_softplus(int64_t ntok, int64_t dt_rank, int64_t d_inner, const float* x, int64_t ldx,
                       const float* weight, const float* bias, const float* gin, int64_t ldg, float* out,
                       int64_t ldo, float* out_lo, float* bpart, vmscan_stream_t stream) {
  if (x == nullptr || weight == nullptr || bias == nullptr || out == nullptr || (BWD && gin == nullptr))
    return VMSCAN_ERR_NULL;
  if (ntok <= 0 || d_inner <= 0 || d_inner > INT32_MAX || dt_rank < 1 || dt_rank > DTP_RMAX)
    return fail(VMSCAN_ERR_SHAPE, "dt_softplus: ntok %lld, dt_rank %lld (1..%d), d_inner %lld",
                (long long)ntok, (long long)dt_rank, DTP_RMAX, (long long)d_inner);
  if (ldx < dt_rank || ldo < d_inner || (BWD && ldg < d_inner))
    return fail(VMSCAN_ERR_SHAPE, "dt_softplus: row strides shorter than the rows");
  if ((ntok + DTP_TOKENS - 1) / DTP_TOKENS > 65535)
    return fail(VMSCAN_ERR_SHAPE, "dt_softplus: %lld tokens exceed the launch grid", (long long)ntok);
  VM_TRY(ensure_context(x));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int R = int(dt_rank), D = int(d_inner);
  const unsigned ty = unsigned((ntok + DTP_TOKENS - 1) / DTP_TOKENS);
#define VM_DTP(RP)                                                                                           \
  dt_softplus_kernel<RP, BWD>                                                                                \
      <<<dim3(unsigned((d_inner + DTP_THREADS * dtp_channels(RP) - 1) / (DTP_THREADS * dtp_channels(RP))), ty), \
         DTP_THREADS, 0, s>>>(x, ldx, R, weight, bias, gin, ldg, out, ldo, out_lo, bpart, ntok, D)
  if (R <= 8)
    VM_DTP(8);
  else if (R <= 16)
    VM_DTP(16);
  else if (R <= 24)
    VM_DTP(24);
  else if (R <= 32)
    VM_DTP(32);
  else if (R <= 48)
    VM_DTP(48);
  else
    VM_DTP(64);
#undef VM_DTP
  return check_launch();
}

}  // namespace

namespace {

// Output tile width: the narrowest of 32, 64, 128 columns that covers N
// (the skinny x_proj / dt_proj products), 128 otherwise.
int gemm_bn(int64_t N) { return N <= 32 ? 32 : (N <= 64 ? 64 : 128); }

// 2-D tensor map of a row-major (rows x cols) fp32 matrix with row stride ld
// (elements): box {32, box_rows}, zero fill outside, 128-byte swizzle of
// 16-byte chunks (K-major operand tiles) or of 32-byte chunks (mn: MN-major).
int encode_gemm_map(CUtensorMap* m, const char* what, const float* p, int64_t cols, int64_t rows, int64_t ld,
                    int box_rows, bool mn) {
  if (p == nullptr) return fail(VMSCAN_ERR_NULL, "gemm: %s is NULL", what);
  if (!aligned16(p) || ld % 4 != 0 || ld < cols)
    return fail(VMSCAN_ERR_ALIGN, "gemm: %s (base %p, row stride %lld for %lld columns) must be 16-byte aligned "
                "with a row stride that is a multiple of 4 elements", what, p, (long long)ld, (long long)cols);
  auto fn = encode_fn();
  if (fn == nullptr) return fail(VMSCAN_ERR_DRIVER, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 4};
  cuuint32_t box[2] = {32u, cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        mn ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(VMSCAN_ERR_DRIVER, "cuTensorMapEncodeTiled(gemm %s) -> CUresult %d; dims {%lld, %lld} ld %lld",
                what, int(r), (long long)cols, (long long)rows, (long long)ld);
  return VMSCAN_OK;
}

// K splits of a GEMM: 1 while the output tiles fill the SMs, otherwise enough
// splits to fill them with at least 4 k-blocks each (at most 32 splits; the
// skinny weight gradients have a handful of tiles and K of 10^4).
//
// CTA pairs (256-row work items, cta_group::2 MMAs, 4 ring stages instead of
// 3) for 128-column tiles with an MN-major A (the weight gradients, A = dY^T,
// whose k-blocks arrive as 4 + 4 TMA boxes) when M is a multiple of 256, so
// no pair has an empty half; the pairs then play the role of the SMs in the
// split count.  Measured on one B200 (A/B, bench.py --gemm): in_proj weight
// gradient (M 6144, N 384, K 12544) 0.408 -> 0.324 ms; with a K-major A the
// pairs were 2-6 % slower (in_proj / out_proj forward and input gradients:
// the two SMs wait for each other at every chain and tile hand-over).
struct GemmPlan {
  int bn, tiles_n, tiles_m, splits, kb_per_split;
  bool pair;
  size_t ws_bytes;
};

#ifndef VMSCAN_GEMM_PAIR
#define VMSCAN_GEMM_PAIR 1
#endif

GemmPlan gemm_plan(int64_t M, int64_t N, int64_t K, bool a_mn) {
  GemmPlan p;
  p.bn = gemm_bn(N);
  p.pair = VMSCAN_GEMM_PAIR && a_mn && p.bn == 128 && M % (2 * GM_BM) == 0;
  p.tiles_n = int((N + p.bn - 1) / p.bn);
  p.tiles_m = int((M + GM_BM - 1) / GM_BM) / (p.pair ? 2 : 1);
  const int nkb = int((K + GM_BK - 1) / GM_BK);
  const int64_t tiles = int64_t(p.tiles_n) * p.tiles_m;
  const int sms = sm_count() / (p.pair ? 2 : 1);
  int s = 1;
  if (tiles < sms) s = int(std::min<int64_t>({int64_t(sms) / tiles, int64_t(nkb / 4), 32}));
  s = std::max(s, 1);
  p.kb_per_split = (nkb + s - 1) / s;
  p.splits = (nkb + p.kb_per_split - 1) / p.kb_per_split;  // no empty split
  p.ws_bytes = p.splits > 1 ? align256(size_t(p.splits) * size_t(M) * size_t(N) * 4) : 0;
  return p;
}

template <int BN, bool A_MN, bool B_MN, bool PAIR = false>
int launch_gemm(const CUtensorMap& ahi, const CUtensorMap& alo, const CUtensorMap& bhi, const CUtensorMap& blo,
                const GemmPlan& p, const GemmArgs& a, cudaStream_t s) {
  using Cfg = GemmCfg<BN, PAIR>;
  auto kern = gemm_tf32x3_kernel<BN, A_MN, B_MN, PAIR>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Cfg::SMEM_BYTES)) != cudaSuccess)
    return fail(VMSCAN_ERR_LAUNCH, "cudaFuncSetAttribute(gemm_tf32x3_kernel) failed");
  int* st = status_ptr();
  if (st == nullptr) return fail(VMSCAN_ERR_LAUNCH, "status symbol unavailable");
  const int64_t items = int64_t(p.tiles_n) * p.tiles_m * p.splits;
  if constexpr (PAIR) {
    // clusters of 2 CTAs, one pair per work item up to one pair per 2 SMs
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2u * unsigned(std::min<int64_t>(items, sm_count() / 2)));
    cfg.blockDim = dim3(GM_THREADS);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ahi, alo, bhi, blo, a, st);
    if (e != cudaSuccess) return fail(VMSCAN_ERR_LAUNCH, "gemm (CTA pairs) launch: %s", cudaGetErrorString(e));
  } else {
    const unsigned grid = unsigned(std::min<int64_t>(items, sm_count()));
    kern<<<grid, GM_THREADS, Cfg::SMEM_BYTES, s>>>(ahi, alo, bhi, blo, a, st);
  }
  return check_launch();
}

template <bool A_MN, bool B_MN>
int launch_gemm_bn(const CUtensorMap& ahi, const CUtensorMap& alo, const CUtensorMap& bhi, const CUtensorMap& blo,
                   const GemmPlan& p, const GemmArgs& a, cudaStream_t s) {
  if (p.bn == 32) return launch_gemm<32, A_MN, B_MN>(ahi, alo, bhi, blo, p, a, s);
  if (p.bn == 64) return launch_gemm<64, A_MN, B_MN>(ahi, alo, bhi, blo, p, a, s);
  if constexpr (A_MN)
    if (p.pair) return launch_gemm<128, A_MN, B_MN, true>(ahi, alo, bhi, blo, p, a, s);
  return launch_gemm<128, A_MN, B_MN>(ahi, alo, bhi, blo, p, a, s);
}

}  // namespace

// The failure path of every bounded wait, exercised on purpose: one warp
// waits on an mbarrier that nothing arrives on, gives up after `tries`
// polls, records VMSCAN_ERR_TIMEOUT in the sticky status and returns; no
// fault, no trap, and the context stays usable.
__global__ void wait_timeout_selftest_kernel(uint32_t tries, int* status) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) (void)mbar_wait(&bar, 0u, &abort_flag, status, tries);
}

namespace {

int ln_chunks(int64_t dim) { return int((dim / 4 + 31) / 32); }

bool ln_shape_ok(int64_t rows, int64_t dim) {
  return rows > 0 && rows <= INT32_MAX && dim > 0 && dim % 4 == 0 && dim <= LN_MAX_DIM;
}

template <int NC>
void launch_ln_fwd(int rows, int dim, const float* x, int64_t ldx, const float* w, const float* b, float eps,
                   float* y, int64_t ldy, float* mean, float* rstd, cudaStream_t s) {
  layernorm_fwd_kernel<NC><<<unsigned((rows + LN_WARPS - 1) / LN_WARPS), LN_WARPS * 32, 0, s>>>(
      x, ldx, w, b, eps, y, ldy, mean, rstd, rows, dim);
}

template <int NC>
int launch_ln_bwd(int rows, int dim, const float* x, int64_t ldx, const float* w, const float* mean,
                  const float* rstd, const float* dy, int64_t lddy, float* dx, int64_t lddx, float* part,
                  cudaStream_t s) {
  const int per = LN_WARPS * LN_ROWS_PER_WARP;
  const size_t smem = size_t(LN_WARPS) * 2 * size_t(dim) * 4;
  auto kern = layernorm_bwd_kernel<NC>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return fail(VMSCAN_ERR_LAUNCH, "cudaFuncSetAttribute(layernorm_bwd_kernel) failed");
  kern<<<unsigned((rows + per - 1) / per), LN_WARPS * 32, smem, s>>>(x, ldx, w, mean, rstd, dy, lddy, dx, lddx,
                                                                    part, rows, dim);
  return VMSCAN_OK;
}

}  // namespace

extern "C" {

int vmscan_version(void) { return 100; }

const char* vmscan_strerror(int status) {
  switch (status) {
    case VMSCAN_OK: return "ok";
    case VMSCAN_ERR_NULL: return "a required pointer is NULL";
    case VMSCAN_ERR_SHAPE: return "a size is out of range";
    case VMSCAN_ERR_DSTATE: return "d_state must be 16";
    case VMSCAN_ERR_ALIGN: return "pointer or stride breaks the 16-byte TMA alignment rules (channel stride 1, "
                                  "16-byte base, strides multiple of 4 elements)";
    case VMSCAN_ERR_DIRECTION: return "bad direction descriptor (grid product != seqlen, axes not a permutation, "
                                      "or more than 3 non-mergeable scan dims)";
    case VMSCAN_ERR_WORKSPACE: return "workspace missing or too small";
    case VMSCAN_ERR_DRIVER: return "the CUDA driver refused the tensor map";
    case VMSCAN_ERR_LAUNCH: return "kernel launch failed";
    case VMSCAN_ERR_TIMEOUT: return "a device-side wait ran out; the kernel returned early";
    case VMSCAN_ERR_CONV: return "conv kernel size must be 1..8 and channels a multiple of 4";
    case VMSCAN_ERR_SCRATCH: return "problem needs more scratch than vmscan_bwd_noalloc's static 32 MiB array; "
                                    "use vmscan_bwd with a caller-provided workspace";
    default: return "unknown vmscan status";
  }
}

int64_t vmscan_ckpt_elems(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state,
                          const vmscan_direction* dir) {
  if (d_state != NS) return -VMSCAN_ERR_DSTATE;
  ScanGeom g;
  const int rc = make_geom(batch, seqlen, d_inner, dir, g);
  if (rc != VMSCAN_OK) return -rc;
  return int64_t(batch) * g.nboxes * d_inner * NS;
}

int vmscan_fwd(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state, const float* u, vmscan_strides su,
               const float* delta, vmscan_strides sdelta, const float* A, const float* B, vmscan_strides sB,
               const float* C, vmscan_strides sC, const float* D, const float* z, vmscan_strides sz, float* y,
               vmscan_strides sy, float* y_lo, float* ckpt, const vmscan_direction* dir, void* workspace,
               size_t workspace_bytes, vmscan_stream_t stream) {
  return fwd_impl<float>(batch, seqlen, d_inner, d_state, u, su, delta, sdelta, A, B, sB, C, sC, D, z, sz, y, sy,
                         y_lo, ckpt, dir, workspace, workspace_bytes, stream);
}

int vmscan_fwd_bf16(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state, const void* u,
                    vmscan_strides su, const void* delta, vmscan_strides sdelta, const float* A, const void* B,
                    vmscan_strides sB, const void* C, vmscan_strides sC, const float* D, const void* z,
                    vmscan_strides sz, void* y, vmscan_strides sy, float* ckpt, const vmscan_direction* dir,
                    void* workspace, size_t workspace_bytes, vmscan_stream_t stream) {
  using T = __nv_bfloat16;
  return fwd_impl<T>(batch, seqlen, d_inner, d_state, static_cast<const T*>(u), su, static_cast<const T*>(delta),
                     sdelta, A, static_cast<const T*>(B), sB, static_cast<const T*>(C), sC, D,
                     static_cast<const T*>(z), sz, static_cast<T*>(y), sy, nullptr, ckpt, dir, workspace,
                     workspace_bytes, stream);
}

int64_t vmscan_fwd_workspace_bytes(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state,
                                   const vmscan_direction* dir) {
  if (d_state != NS) return -VMSCAN_ERR_DSTATE;
  ScanGeom g;
  const int rc = make_geom(batch, seqlen, d_inner, dir, g);
  if (rc != VMSCAN_OK) return -rc;
  return int64_t(fwd_chunk_plan(g).bytes);
}

int64_t vmscan_bwd_workspace_bytes(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state,
                                   const vmscan_direction* dir, int recompute_ckpt) {
  if (d_state != NS) return -VMSCAN_ERR_DSTATE;
  ScanGeom g;
  const int rc = make_geom(batch, seqlen, d_inner, dir, g);
  if (rc != VMSCAN_OK) return -rc;
  const int ndt = int((d_inner + BwdCfg<>::DT - 1) / BwdCfg<>::DT);
  return int64_t(bwd_layout(g, ndt, recompute_ckpt != 0).total);
}

int vmscan_bwd(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state, const float* u, vmscan_strides su,
               const float* delta, vmscan_strides sdelta, const float* A, const float* B, vmscan_strides sB,
               const float* C, vmscan_strides sC, const float* D, const float* z, vmscan_strides sz,
               const float* ckpt, const float* dy, vmscan_strides sdy, float* du, vmscan_strides sdu,
               float* ddelta, vmscan_strides sddelta, float* dA, float* dB, vmscan_strides sdB, float* dC,
               vmscan_strides sdC, float* dD, float* dz, vmscan_strides sdz, float* dz_lo,
               const vmscan_direction* dir, void* workspace, size_t workspace_bytes, vmscan_stream_t stream) {
  return bwd_impl<float>(batch, seqlen, d_inner, d_state, u, su, delta, sdelta, A, B, sB, C, sC, D, z, sz, ckpt, dy,
                         sdy, du, sdu, ddelta, sddelta, dA, dB, sdB, dC, sdC, dD, dz, sdz, dz_lo, dir, workspace,
                         workspace_bytes, stream);
}

int vmscan_bwd_bf16(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state, const void* u,
                    vmscan_strides su, const void* delta, vmscan_strides sdelta, const float* A, const void* B,
                    vmscan_strides sB, const void* C, vmscan_strides sC, const float* D, const void* z,
                    vmscan_strides sz, const float* ckpt, const void* dy, vmscan_strides sdy, void* du,
                    vmscan_strides sdu, void* ddelta, vmscan_strides sddelta, float* dA, void* dB,
                    vmscan_strides sdB, void* dC, vmscan_strides sdC, float* dD, void* dz, vmscan_strides sdz,
                    const vmscan_direction* dir, void* workspace, size_t workspace_bytes, vmscan_stream_t stream) {
  using T = __nv_bfloat16;
  return bwd_impl<T>(batch, seqlen, d_inner, d_state, static_cast<const T*>(u), su, static_cast<const T*>(delta),
                     sdelta, A, static_cast<const T*>(B), sB, static_cast<const T*>(C), sC, D,
                     static_cast<const T*>(z), sz, ckpt, static_cast<const T*>(dy), sdy, static_cast<T*>(du), sdu,
                     static_cast<T*>(ddelta), sddelta, dA, static_cast<T*>(dB), sdB, static_cast<T*>(dC), sdC, dD,
                     static_cast<T*>(dz), sdz, nullptr, dir, workspace, workspace_bytes, stream);
}

int vmscan_dt_softplus_fwd(int64_t ntok, int64_t dt_rank, int64_t d_inner, const float* x, int64_t ldx,
                           const float* weight, const float* bias, float* delta, int64_t ld_delta,
                           vmscan_stream_t stream) {
  return launch_dt_softplus<false>(ntok, dt_rank, d_inner, x, ldx, weight, bias, nullptr, 0, delta, ld_delta,
                                   nullptr, nullptr, stream);
}

int64_t vmscan_dt_softplus_bias_rows(int64_t ntok) {
  if (ntok <= 0) return -VMSCAN_ERR_SHAPE;
  return (ntok + DTP_TOKENS - 1) / DTP_TOKENS;
}


int vmscan_layernorm_fwd(int64_t rows, int64_t dim, const float* x, int64_t ldx, const float* weight,
                         const float* bias, float eps, float* y, int64_t ldy, float* mean, float* rstd,
                         vmscan_stream_t stream) {
  if (!ln_shape_ok(rows, dim) || ldx < dim || ldy < dim) return VMSCAN_ERR_SHAPE;
  if (x == nullptr || weight == nullptr || bias == nullptr || y == nullptr || mean == nullptr || rstd == nullptr)
    return VMSCAN_ERR_NULL;
  if (!aligned16(x) || !aligned16(y) || !aligned16(weight) || !aligned16(bias) || ldx % 4 || ldy % 4)
    return VMSCAN_ERR_ALIGN;
  VM_TRY(ensure_context(x));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int r = int(rows), d = int(dim);
  switch (ln_chunks(dim)) {
    case 1: launch_ln_fwd<1>(r, d, x, ldx, weight, bias, eps, y, ldy, mean, rstd, s); break;
    case 2: launch_ln_fwd<2>(r, d, x, ldx, weight, bias, eps, y, ldy, mean, rstd, s); break;
    case 3: launch_ln_fwd<3>(r, d, x, ldx, weight, bias, eps, y, ldy, mean, rstd, s); break;
    case 4: launch_ln_fwd<4>(r, d, x, ldx, weight, bias, eps, y, ldy, mean, rstd, s); break;
    default: launch_ln_fwd<8>(r, d, x, ldx, weight, bias, eps, y, ldy, mean, rstd, s); break;
  }
  return check_launch();
}

int64_t vmscan_layernorm_bwd_workspace_bytes(int64_t rows, int64_t dim) {
  if (!ln_shape_ok(rows, dim)) return -VMSCAN_ERR_SHAPE;
  const int64_t per = LN_WARPS * LN_ROWS_PER_WARP;
  return int64_t(align256(size_t((rows + per - 1) / per) * 2 * size_t(dim) * 4));
}

int vmscan_layernorm_bwd(int64_t rows, int64_t dim, const float* x, int64_t ldx, const float* weight,
                         const float* mean, const float* rstd, const float* dy, int64_t lddy, float* dx,
                         int64_t lddx, float* dweight, float* dbias, void* workspace, size_t workspace_bytes,
                         vmscan_stream_t stream) {
  if (!ln_shape_ok(rows, dim) || ldx < dim || lddy < dim || lddx < dim) return VMSCAN_ERR_SHAPE;
  if (x == nullptr || weight == nullptr || mean == nullptr || rstd == nullptr || dy == nullptr || dx == nullptr ||
      dweight == nullptr || dbias == nullptr)
    return VMSCAN_ERR_NULL;
  if (!aligned16(x) || !aligned16(dy) || !aligned16(dx) || !aligned16(weight) || ldx % 4 || lddy % 4 || lddx % 4)
    return VMSCAN_ERR_ALIGN;
  const int64_t need = vmscan_layernorm_bwd_workspace_bytes(rows, dim);
  if (workspace == nullptr || int64_t(workspace_bytes) < need || !aligned16(workspace)) return VMSCAN_ERR_WORKSPACE;
  VM_TRY(ensure_context(x));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int r = int(rows), d = int(dim);
  float* part = static_cast<float*>(workspace);
  switch (ln_chunks(dim)) {
    case 1: VM_TRY(launch_ln_bwd<1>(r, d, x, ldx, weight, mean, rstd, dy, lddy, dx, lddx, part, s)); break;
    case 2: VM_TRY(launch_ln_bwd<2>(r, d, x, ldx, weight, mean, rstd, dy, lddy, dx, lddx, part, s)); break;
    case 3: VM_TRY(launch_ln_bwd<3>(r, d, x, ldx, weight, mean, rstd, dy, lddy, dx, lddx, part, s)); break;
    case 4: VM_TRY(launch_ln_bwd<4>(r, d, x, ldx, weight, mean, rstd, dy, lddy, dx, lddx, part, s)); break;
    default: VM_TRY(launch_ln_bwd<8>(r, d, x, ldx, weight, mean, rstd, dy, lddy, dx, lddx, part, s)); break;
  }
  VM_TRY(check_launch());
  const int64_t per = LN_WARPS * LN_ROWS_PER_WARP;
  const int prow = int((rows + per - 1) / per);
  const dim3 g(unsigned((dim + kSumRowsCols - 1) / kSumRowsCols));
  sum_rows_kernel<<<g, kSumRowsCols * kSumRowsGroups, 0, s>>>(part, dweight, prow, d, 2 * dim);
  VM_TRY(check_launch());
  sum_rows_kernel<<<g, kSumRowsCols * kSumRowsGroups, 0, s>>>(part + dim, dbias, prow, d, 2 * dim);
  return check_launch();
}

int vmscan_sum_rows(int64_t rows, int64_t cols, const float* part, float* out, vmscan_stream_t stream) {
  if (rows <= 0 || cols <= 0 || rows > INT32_MAX || cols > INT32_MAX) return VMSCAN_ERR_SHAPE;
  if (part == nullptr || out == nullptr) return VMSCAN_ERR_NULL;
  VM_TRY(ensure_context(part));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  sum_rows_kernel<<<unsigned((cols + kSumRowsCols - 1) / kSumRowsCols), kSumRowsCols * kSumRowsGroups, 0, s>>>(
      part, out, int(rows), int(cols), cols);
  return check_launch();
}

int vmscan_dt_softplus_bwd(int64_t ntok, int64_t dt_rank, int64_t d_inner, const float* x, int64_t ldx,
                           const float* weight, const float* bias, const float* ddelta, int64_t ld_ddelta,
                           float* dpre, int64_t ld_dpre, float* dpre_lo, float* dbias_part, vmscan_stream_t stream) {
  return launch_dt_softplus<true>(ntok, dt_rank, d_inner, x, ldx, weight, bias, ddelta, ld_ddelta, dpre, ld_dpre,
                                  dpre_lo, dbias_part, stream);
}

int vmscan_conv1d_silu_fwd(int64_t batch, int64_t seqlen, int64_t channels, int64_t ksize, const float* x,
                           vmscan_strides sx, const float* weight, const float* bias, float* out,
                           vmscan_strides sout, float* out_hi, float* out_lo, const vmscan_direction* dir,
                           vmscan_stream_t stream) {
  if (x == nullptr || weight == nullptr || bias == nullptr || out == nullptr) return VMSCAN_ERR_NULL;
  if ((out_hi == nullptr) != (out_lo == nullptr)) return VMSCAN_ERR_NULL;
  if (out_hi != nullptr && (!aligned16(out_hi) || !aligned16(out_lo))) return VMSCAN_ERR_ALIGN;
  if (ksize < 1 || ksize > CONV_KMAX || channels % 4 != 0) return VMSCAN_ERR_CONV;
  ScanGeom g;
  VM_TRY(make_geom(batch, seqlen, channels, dir, g));
  VM_TRY(ensure_context(x));
  if (!aligned16(x) || !aligned16(out) || !aligned16(bias) || sx.seq % 4 || sx.batch % 4 || sout.seq % 4 ||
      sout.batch % 4)
    return VMSCAN_ERR_ALIGN;
  const dim3 grid(unsigned((channels / 4 + CONV_THREADS - 1) / CONV_THREADS),
                  unsigned((seqlen + CONV_CHUNK - 1) / CONV_CHUNK), unsigned(batch));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool split = out_hi != nullptr;
  auto kern = ksize <= 4 ? (split ? conv_silu_fwd_kernel<4, true> : conv_silu_fwd_kernel<4, false>)
                         : (split ? conv_silu_fwd_kernel<8, true> : conv_silu_fwd_kernel<8, false>);
  kern<<<grid, CONV_THREADS, 0, s>>>(x, sx.batch, sx.seq, weight, bias, out, sout.batch, sout.seq, out_hi, out_lo,
                                     int(channels), int(ksize), g);
  return check_launch();
}

int64_t vmscan_conv1d_bwd_workspace_bytes(int64_t batch, int64_t seqlen, int64_t channels, int64_t ksize) {
  if (batch <= 0 || seqlen <= 0 || channels <= 0) return -VMSCAN_ERR_SHAPE;
  if (ksize < 1 || ksize > CONV_KMAX) return -VMSCAN_ERR_CONV;
  const int64_t nchunk = (seqlen + CONV_CHUNK - 1) / CONV_CHUNK;
  return int64_t(align256(size_t(batch) * nchunk * channels * (CONV_KMAX + 1) * 4) +
                 align256(size_t(CONV_RGROUPS) * channels * (CONV_KMAX + 1) * 4));
}

int vmscan_conv1d_silu_bwd(int64_t batch, int64_t seqlen, int64_t channels, int64_t ksize, const float* x,
                           vmscan_strides sx, const float* weight, const float* bias, const float* dout,
                           vmscan_strides sdout, float* dx, vmscan_strides sdx, float* dx_lo, float* dweight,
                           float* dbias, const vmscan_direction* dir, void* workspace, size_t workspace_bytes,
                           vmscan_stream_t stream) {
  if (x == nullptr || weight == nullptr || bias == nullptr || dout == nullptr || dx == nullptr ||
      dweight == nullptr || dbias == nullptr)
    return VMSCAN_ERR_NULL;
  if (ksize < 1 || ksize > CONV_KMAX || channels % 4 != 0) return VMSCAN_ERR_CONV;
  ScanGeom g;
  VM_TRY(make_geom(batch, seqlen, channels, dir, g));
  VM_TRY(ensure_context(x));
  if (!aligned16(x) || !aligned16(dout) || !aligned16(dx) || !aligned16(bias) || sx.seq % 4 || sx.batch % 4 ||
      sdout.seq % 4 || sdout.batch % 4 || sdx.seq % 4 || sdx.batch % 4 || (dx_lo != nullptr && !aligned16(dx_lo)))
    return VMSCAN_ERR_ALIGN;
  const int64_t need = vmscan_conv1d_bwd_workspace_bytes(batch, seqlen, channels, ksize);
  if (workspace == nullptr || int64_t(workspace_bytes) < need) return VMSCAN_ERR_WORKSPACE;
  const int nchunk = int((seqlen + CONV_CHUNK - 1) / CONV_CHUNK);
  const dim3 grid(unsigned((channels / 4 + CONV_THREADS - 1) / CONV_THREADS), unsigned(nchunk), unsigned(batch));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float* wpart = static_cast<float*>(workspace);
  const bool split = dx_lo != nullptr;
  auto kern = ksize <= 4 ? (split ? conv_silu_bwd_kernel<4, true> : conv_silu_bwd_kernel<4, false>)
                         : (split ? conv_silu_bwd_kernel<8, true> : conv_silu_bwd_kernel<8, false>);
  kern<<<grid, CONV_THREADS, 0, s>>>(x, sx.batch, sx.seq, weight, bias, dout, sdout.batch, sdout.seq, dx, sdx.batch,
                                     sdx.seq, dx_lo, wpart, int(channels), int(ksize), g);
  VM_TRY(check_launch());
  const int n = int(channels * (ksize + 1));
  const int nrows = int(batch) * nchunk;
  const int ngroups = std::min(CONV_RGROUPS, nrows);
  float* gpart = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                          align256(size_t(batch) * nchunk * channels * (CONV_KMAX + 1) * 4));
  conv_reduce_kernel<<<dim3(unsigned((n + 255) / 256), unsigned(ngroups)), 256, 0, s>>>(wpart, gpart, nrows,
                                                                                       int(channels), int(ksize));
  VM_TRY(check_launch());
  conv_reduce2_kernel<<<unsigned((n + 255) / 256), 256, 0, s>>>(gpart, dweight, dbias, ngroups, int(channels),
                                                               int(ksize));
  return check_launch();
}

int vmscan_scan_order(int64_t seqlen, const vmscan_direction* dir, int mode, int64_t* tokens, int64_t* geom) {
  if (tokens == nullptr) return VMSCAN_ERR_NULL;
  ScanGeom g;
  VM_TRY(make_geom(1, seqlen, 1, dir, g));
  if (geom != nullptr) {
    const int64_t v[16] = {g.nsd,  g.size[0], g.size[1], g.size[2], g.tstride[0], g.tstride[1],
                           g.tstride[2], g.j, g.bj, g.nj, g.P, g.T, g.nboxes, g.reverse, 0, 0};
    for (int i = 0; i < 16; ++i) geom[i] = v[i];
  }
  if (mode == 1) {
    for (int64_t p = 0; p < seqlen; ++p) tokens[p] = scan_pos_token(g, int(p));
    return VMSCAN_OK;
  }
  int64_t q = 0;
  for (int i = 0; i < g.nboxes; ++i) {
    const int k = g.reverse ? g.nboxes - 1 - i : i;
    int c[3], nv;
    box_coords(g, k, c, nv);
    for (int s = 0; s < nv; ++s) {
      const int r = g.reverse ? nv - 1 - s : s;
      if (q >= seqlen) return VMSCAN_ERR_SHAPE;
      tokens[q++] = box_row_token(g, c, r);
    }
  }
  return q == seqlen ? VMSCAN_OK : VMSCAN_ERR_SHAPE;
}

const char* vmscan_last_error(void) { return g_last_error; }

namespace {
// Address of g_vmscan_noalloc_scratch in the CUDA context that is current for
// this call.  The address belongs to a context (not to a device index): a
// thread may bind a non-primary context, and a context can be destroyed and
// created again.  So it is looked up on every call, as status_ptr() does for
// the status word, never cached.
int noalloc_scratch_addr(const void* devbuf, void** out) {
  VM_TRY(ensure_context(devbuf));
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return fail(VMSCAN_ERR_LAUNCH, "cudaGetDevice failed");
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, devbuf) != cudaSuccess || attr.device != dev)
    return fail(VMSCAN_ERR_LAUNCH, "the current device (%d) does not own the input buffers", dev);
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_vmscan_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr)
    return fail(VMSCAN_ERR_LAUNCH, "cudaGetSymbolAddress(scratch) on device %d failed: %s", dev,
                cudaGetErrorString(e));
  *out = p;
  return VMSCAN_OK;
}
}  // namespace

int vmscan_bwd_noalloc(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state, const float* u,
                       vmscan_strides su, const float* delta, vmscan_strides sdelta, const float* A, const float* B,
                       vmscan_strides sB, const float* C, vmscan_strides sC, const float* D, const float* z,
                       vmscan_strides sz, const float* ckpt, const float* dy, vmscan_strides sdy, float* du,
                       vmscan_strides sdu, float* ddelta, vmscan_strides sddelta, float* dA, float* dB,
                       vmscan_strides sdB, float* dC, vmscan_strides sdC, float* dD, float* dz, vmscan_strides sdz,
                       const vmscan_direction* dir, vmscan_stream_t stream) {
  if (u == nullptr) return VMSCAN_ERR_NULL;
  const int64_t need = vmscan_bwd_workspace_bytes(batch, seqlen, d_inner, d_state, dir, ckpt == nullptr ? 1 : 0);
  if (need < 0) return int(-need);
  if (need > int64_t(VMSCAN_NOALLOC_SCRATCH_BYTES))
    return fail(VMSCAN_ERR_SCRATCH, "needs %lld bytes of scratch, the static array holds %u", (long long)need,
                VMSCAN_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  VM_TRY(noalloc_scratch_addr(u, &scratch));
  return vmscan_bwd(batch, seqlen, d_inner, d_state, u, su, delta, sdelta, A, B, sB, C, sC, D, z, sz, ckpt, dy, sdy,
                    du, sdu, ddelta, sddelta, dA, dB, sdB, dC, sdC, dD, dz, sdz, nullptr, dir, scratch,
                    size_t(VMSCAN_NOALLOC_SCRATCH_BYTES), stream);
}

int vmscan_tf32_split(int64_t n, const float* x, float* hi, float* lo, vmscan_stream_t stream) {
  if (n == 0) return VMSCAN_OK;
  if (x == nullptr || hi == nullptr || lo == nullptr) return VMSCAN_ERR_NULL;
  if (n < 0 || n % 4 != 0) return fail(VMSCAN_ERR_SHAPE, "tf32_split: n = %lld must be a multiple of 4", (long long)n);
  if (!aligned16(x) || !aligned16(hi) || !aligned16(lo))
    return fail(VMSCAN_ERR_ALIGN, "tf32_split: buffers must be 16-byte aligned");
  VM_TRY(ensure_context(x));
  const int64_t n4 = n / 4;
  const unsigned blocks = unsigned(std::min<int64_t>((n4 + 255) / 256, int64_t(sm_count()) * 8));
  tf32_split_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(hi), reinterpret_cast<float4*>(lo), n4);
  return check_launch();
}

int vmscan_tf32_split_multi(int count, const float* const* x, float* const* hi, float* const* lo, const int64_t* n,
                            vmscan_stream_t stream) {
  if (count == 0) return VMSCAN_OK;
  if (count < 0 || count > kSplitMaxTensors)
    return fail(VMSCAN_ERR_SHAPE, "tf32_split_multi: %d tensors (1..%d)", count, kSplitMaxTensors);
  if (x == nullptr || hi == nullptr || lo == nullptr || n == nullptr) return VMSCAN_ERR_NULL;
  SplitTable t{};
  int64_t most = 0;
  for (int k = 0; k < count; ++k) {
    if (x[k] == nullptr || hi[k] == nullptr || lo[k] == nullptr) return VMSCAN_ERR_NULL;
    if (n[k] < 0 || n[k] % 4 != 0)
      return fail(VMSCAN_ERR_SHAPE, "tf32_split_multi: tensor %d has %lld floats (a multiple of 4)", k,
                  (long long)n[k]);
    if (!aligned16(x[k]) || !aligned16(hi[k]) || !aligned16(lo[k]))
      return fail(VMSCAN_ERR_ALIGN, "tf32_split_multi: tensor %d is not 16-byte aligned", k);
    t.x[k] = reinterpret_cast<const float4*>(x[k]);
    t.hi[k] = reinterpret_cast<float4*>(hi[k]);
    t.lo[k] = reinterpret_cast<float4*>(lo[k]);
    t.n4[k] = n[k] / 4;
    most = std::max(most, n[k] / 4);
  }
  if (most == 0) return VMSCAN_OK;
  VM_TRY(ensure_context(x[0]));
  const unsigned bx = unsigned(std::min<int64_t>((most + 255) / 256, int64_t(sm_count()) * 2));
  tf32_split_multi_kernel<<<dim3(bx, unsigned(count)), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(t);
  return check_launch();
}

int64_t vmscan_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return -VMSCAN_ERR_SHAPE;
  // enough for either operand layout of A (CTA pairs may split K differently)
  return int64_t(std::max(gemm_plan(M, N, K, false).ws_bytes, gemm_plan(M, N, K, true).ws_bytes));
}

int vmscan_gemm_tf32x3(int64_t M, int64_t N, int64_t K, const float* a_hi, const float* a_lo, int64_t lda,
                       int a_mn_major, const float* b_hi, const float* b_lo, int64_t ldb, int b_mn_major, float* c,
                       int64_t ldc, int accumulate, void* workspace, int64_t workspace_bytes,
                       vmscan_stream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(VMSCAN_ERR_SHAPE, "gemm: M %lld, N %lld, K %lld", (long long)M, (long long)N, (long long)K);
  if (c == nullptr) return VMSCAN_ERR_NULL;
  if (ldc < N) return fail(VMSCAN_ERR_SHAPE, "gemm: ldc %lld < N %lld", (long long)ldc, (long long)N);
  if ((M + GM_BM - 1) / GM_BM * ((N + 31) / 32) * 8 > INT32_MAX)
    return fail(VMSCAN_ERR_SHAPE, "gemm: M %lld x N %lld has too many tiles", (long long)M, (long long)N);
  VM_TRY(ensure_context(c));
  CUtensorMap ahi, alo, bhi, blo;
  // A(m, k): K-major a[m * lda + k] (rows M), MN-major a[k * lda + m] (rows K)
  const int64_t acols = a_mn_major ? M : K, arows = a_mn_major ? K : M;
  const int64_t bcols = b_mn_major ? N : K, brows = b_mn_major ? K : N;
  const GemmPlan p = gemm_plan(M, N, K, a_mn_major != 0);
  // B box: the rows of B one CTA loads (half the tile's columns for a CTA pair)
  const int abox = a_mn_major ? 32 : GM_BM, bbox = b_mn_major ? 32 : (p.pair ? p.bn / 2 : p.bn);
  VM_TRY(encode_gemm_map(&ahi, "a_hi", a_hi, acols, arows, lda, abox, a_mn_major != 0));
  VM_TRY(encode_gemm_map(&alo, "a_lo", a_lo, acols, arows, lda, abox, a_mn_major != 0));
  VM_TRY(encode_gemm_map(&bhi, "b_hi", b_hi, bcols, brows, ldb, bbox, b_mn_major != 0));
  VM_TRY(encode_gemm_map(&blo, "b_lo", b_lo, bcols, brows, ldb, bbox, b_mn_major != 0));
  if (p.splits > 1 && (workspace == nullptr || workspace_bytes < int64_t(p.ws_bytes)))
    return fail(VMSCAN_ERR_WORKSPACE, "gemm: %d K splits need %zu bytes of workspace", p.splits, p.ws_bytes);
  if (p.splits > 1 && !aligned16(workspace)) return fail(VMSCAN_ERR_ALIGN, "gemm: workspace not 16-byte aligned");
  GemmArgs a;
  a.M = int(M);
  a.N = int(N);
  a.K = int(K);
  a.splits = p.splits;
  a.kb_per_split = p.kb_per_split;
  a.accumulate = (accumulate && p.splits == 1) ? 1 : 0;
  a.C = p.splits > 1 ? static_cast<float*>(workspace) : c;
  a.ldc = p.splits > 1 ? N : ldc;
  a.split_stride = M * N;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int rc;
  if (a_mn_major && b_mn_major)
    rc = launch_gemm_bn<true, true>(ahi, alo, bhi, blo, p, a, s);
  else if (a_mn_major)
    rc = launch_gemm_bn<true, false>(ahi, alo, bhi, blo, p, a, s);
  else if (b_mn_major)
    rc = launch_gemm_bn<false, true>(ahi, alo, bhi, blo, p, a, s);
  else
    rc = launch_gemm_bn<false, false>(ahi, alo, bhi, blo, p, a, s);
  if (rc != VMSCAN_OK || p.splits == 1) return rc;
  const int64_t total = M * N;
  const unsigned blocks = unsigned(std::min<int64_t>((total + 255) / 256, int64_t(sm_count()) * 8));
  gemm_splitk_reduce_kernel<<<blocks, 256, 0, s>>>(static_cast<const float*>(workspace), c, ldc, int(M), int(N),
                                                   p.splits, M * N, accumulate ? 1 : 0);
  return check_launch();
}

int vmscan_wait_timeout_selftest(uint32_t tries, vmscan_stream_t stream) {
  if (tries == 0 || tries > kWaitLimit) return fail(VMSCAN_ERR_SHAPE, "tries must be in 1..%u", kWaitLimit);
  int* st = status_ptr();
  if (st == nullptr) return fail(VMSCAN_ERR_LAUNCH, "status symbol unavailable");
  wait_timeout_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(tries, st);
  return check_launch();
}

int vmscan_device_status(vmscan_stream_t stream, int clear) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return VMSCAN_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_vmscan_status, sizeof(int)) != cudaSuccess) return VMSCAN_ERR_LAUNCH;
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_vmscan_status, &zero, sizeof(int)) != cudaSuccess) return VMSCAN_ERR_LAUNCH;
  }
  return v;
}

}  // extern "C"
