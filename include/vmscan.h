/*
 * vmscan.h — C ABI of the B200 (sm_100a) selective-scan library `libvmscan.so`.
 *
 * This is the drop-in boundary for the selective-scan (S6) hot path of
 * mlx-vision-mamba.  Every entry point takes plain device pointers, element
 * strides, sizes and a CUDA stream; none allocates memory, none synchronises
 * the stream, and none holds state between calls (thread-safe).  Each returns
 * an `int` status (VMSCAN_OK == 0) that `vmscan_strerror` turns into text.
 *
 * Reference interfaces replaced (paths inside the mlx-vision-mamba project):
 *   - scan forward  : `selective_scan(x, delta, A, B, C, D) -> y`
 *                     mlx_vision_mamba/mamba_block.py:20-74 (semantics), and the fused
 *                     Metal launch `_launch_fused_fwd`
 *                     mlx_vision_mamba/mamba_metal_fused.py:148-179 (kernel :21-63)
 *   - scan VJP      : `_fused_scan_core_vjp` + `_launch_fused_bwd`
 *                     mlx_vision_mamba/mamba_metal_fused.py:182-250 (kernel :66-145,
 *                     reductions :213-224)
 *   - gate          : `y * silu(z)` in MambaBlock.__call__, mamba_block.py:190
 *   - directions    : permute/flip/unpermute helpers mamba_block.py:244-338 and
 *                     `MultiDirectionalMambaBlock._apply_direction` :407-534, folded
 *                     into the scan's (and the conv's) index maths
 *   - conv1d + SiLU : `self.conv1d(x)[:, :L]` then `nn.silu`, mamba_block.py:129-132,170-171
 *
 * Layouts.  Sequence tensors are (batch, seq, channel) views with channel
 * stride 1 and element strides {batch, seq} given by `vmscan_strides`;
 * B, C, dB, dC are (batch, seq, d_state) views of the same kind.  A / dA are
 * contiguous (d_inner, d_state); D / dD are contiguous (d_inner).  All data is
 * fp32.  Sequence views must start on a 16-byte boundary and have strides that
 * are multiples of 4 elements (TMA tensor-map rules); otherwise the call
 * returns VMSCAN_ERR_ALIGN.  d_state must be 16 (the reference hard-codes a
 * 16-float state, mamba_metal_fused.py:28).
 */
#ifndef VMSCAN_H
#define VMSCAN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream; NULL means the legacy default stream. */
typedef struct CUstream_st* vmscan_stream_t;

enum vmscan_status {
  VMSCAN_OK = 0,
  VMSCAN_ERR_NULL = 1,       /* a required pointer is NULL */
  VMSCAN_ERR_SHAPE = 2,      /* a size is <= 0 or out of range */
  VMSCAN_ERR_DSTATE = 3,     /* d_state != 16 */
  VMSCAN_ERR_ALIGN = 4,      /* pointer / stride breaks the 16-byte TMA rules */
  VMSCAN_ERR_DIRECTION = 5,  /* bad direction descriptor */
  VMSCAN_ERR_WORKSPACE = 6,  /* workspace missing or too small */
  VMSCAN_ERR_DRIVER = 7,     /* tensor-map encoding refused by the driver */
  VMSCAN_ERR_LAUNCH = 8,     /* kernel launch failed */
  VMSCAN_ERR_TIMEOUT = 9,    /* a device-side wait ran out (see vmscan_device_status) */
  VMSCAN_ERR_CONV = 10,      /* conv kernel size unsupported (1..8) */
  VMSCAN_ERR_SCRATCH = 11    /* problem too large for vmscan_bwd_noalloc's static scratch */
};

/*
 * Scan direction.  The sequence of `seqlen` tokens is laid out row-major on
 * `grid[0..ndim)`.  The scan visits tokens in the order of
 * `transpose(grid, axes)` flattened row-major, reversed when `reverse` != 0.
 * ndim == 0 means plain sequence order (grid/axes ignored).  This is the
 * reference's `_permute_*` + `[:, ::-1, :]` pair (mamba_block.py:244-338,
 * :443-534) without moving any data.
 */
typedef struct vmscan_direction {
  int32_t ndim;
  int32_t grid[4];
  int32_t axes[4];
  int32_t reverse;
} vmscan_direction;

/* Element strides of a (batch, seq, channel) view; channel stride is 1. */
typedef struct vmscan_strides {
  int64_t batch;
  int64_t seq;
} vmscan_strides;

/* Library ABI version (major*100 + minor). */
int vmscan_version(void);

/* Static text for a status code. */
const char* vmscan_strerror(int status);

/*
 * Detail of the last failed call on this thread (which argument, the driver's
 * CUresult, the tensor-map dims/strides...); "" if none.  Thread-local.
 */
const char* vmscan_last_error(void);

/*
 * Number of fp32 elements of the checkpoint buffer written by vmscan_fwd and
 * read by vmscan_bwd: the recurrent state (d_state floats per channel) at the
 * end of every scan box of at most 16 steps.  Negative on a bad argument.
 */
int64_t vmscan_ckpt_elems(int64_t batch, int64_t seqlen, int64_t d_inner,
                          int64_t d_state, const vmscan_direction* dir);

/*
 * Workspace of vmscan_fwd: the chunk carries of a scan chunked over L (used
 * when batch x channel tiles would leave most SMs idle); 0 when the scan is
 * not chunked.  Negative on a bad argument.
 */
int64_t vmscan_fwd_workspace_bytes(int64_t batch, int64_t seqlen, int64_t d_inner,
                                   int64_t d_state, const vmscan_direction* dir);

/*
 * Fused forward: y = (selective_scan(u, delta, A, B, C, D)) * silu(z).
 * z == NULL drops the gate (plain reference `selective_scan` output).
 * y_lo != NULL (same strides as y) writes the output as its TF32 hi part into
 * y and lo part into y_lo, the operand form vmscan_gemm_tf32x3 reads (the
 * block's out_proj GEMM), instead of y itself.
 * ckpt == NULL skips the checkpoints (inference); otherwise ckpt must hold
 * vmscan_ckpt_elems(...) floats.  workspace (16-byte aligned) of at least
 * vmscan_fwd_workspace_bytes(...) enables the chunked scan over L; NULL (or
 * too small) runs every sequence in one piece (same results up to rounding).
 * Replaces mamba_metal_fused.py:148-179 (+ the gate at mamba_block.py:190).
 */
int vmscan_fwd(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state,
               const float* u, vmscan_strides su,
               const float* delta, vmscan_strides sdelta,
               const float* A,
               const float* B, vmscan_strides sB,
               const float* C, vmscan_strides sC,
               const float* D,
               const float* z, vmscan_strides sz,
               float* y, vmscan_strides sy,
               float* y_lo,
               float* ckpt,
               const vmscan_direction* dir,
               void* workspace, size_t workspace_bytes,
               vmscan_stream_t stream);

/*
 * Workspace bytes needed by vmscan_bwd.  With recompute_ckpt != 0 the
 * workspace also holds checkpoints that vmscan_bwd rebuilds itself (call
 * vmscan_bwd with ckpt == NULL), matching the reference VJP, which recomputes
 * the forward (mamba_metal_fused.py:241-244).  Negative on a bad argument.
 */
int64_t vmscan_bwd_workspace_bytes(int64_t batch, int64_t seqlen, int64_t d_inner,
                                   int64_t d_state, const vmscan_direction* dir,
                                   int recompute_ckpt);

/*
 * Fused VJP.  dy is the cotangent of the forward output (gated if z != NULL).
 * Writes du, ddelta, dA, dB, dC, dD and (when z != NULL) dz; all outputs are
 * overwritten, not accumulated.  dz_lo != NULL (same strides as dz) writes dz
 * as its TF32 hi part into dz and lo part into dz_lo (the operand form of
 * vmscan_gemm_tf32x3 for the in_proj gradient GEMMs).  Replaces mamba_metal_fused.py:182-250,
 * including the host-side reductions at :213-224, which run on the device in
 * a fixed order (deterministic).
 */
int vmscan_bwd(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state,
               const float* u, vmscan_strides su,
               const float* delta, vmscan_strides sdelta,
               const float* A,
               const float* B, vmscan_strides sB,
               const float* C, vmscan_strides sC,
               const float* D,
               const float* z, vmscan_strides sz,
               const float* ckpt,
               const float* dy, vmscan_strides sdy,
               float* du, vmscan_strides sdu,
               float* ddelta, vmscan_strides sddelta,
               float* dA,
               float* dB, vmscan_strides sdB,
               float* dC, vmscan_strides sdC,
               float* dD,
               float* dz, vmscan_strides sdz,
               float* dz_lo,
               const vmscan_direction* dir,
               void* workspace, size_t workspace_bytes,
               vmscan_stream_t stream);

/*
 * bf16 I/O variants of vmscan_fwd / vmscan_bwd.  The sequence tensors
 * (u, delta, B, C, z, y; dy and du, ddelta, dB, dC, dz) are bf16, passed as
 * void* so that the header needs no CUDA include; A, D, dA, dD and the
 * checkpoints stay fp32, and every operation inside the kernels runs in fp32
 * (loads widen bf16 to fp32, stores round to nearest even).  Strides must be
 * multiples of 8 elements (16 bytes).  Checkpoint and workspace sizes are the
 * fp32 calls' (vmscan_ckpt_elems, vmscan_fwd_workspace_bytes,
 * vmscan_bwd_workspace_bytes).  The reference computes in fp32 only; these
 * halve the scan's HBM traffic for a caller that keeps activations in bf16.
 */
int vmscan_fwd_bf16(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state,
                    const void* u, vmscan_strides su,
                    const void* delta, vmscan_strides sdelta,
                    const float* A,
                    const void* B, vmscan_strides sB,
                    const void* C, vmscan_strides sC,
                    const float* D,
                    const void* z, vmscan_strides sz,
                    void* y, vmscan_strides sy,
                    float* ckpt,
                    const vmscan_direction* dir,
                    void* workspace, size_t workspace_bytes,
                    vmscan_stream_t stream);

int vmscan_bwd_bf16(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state,
                    const void* u, vmscan_strides su,
                    const void* delta, vmscan_strides sdelta,
                    const float* A,
                    const void* B, vmscan_strides sB,
                    const void* C, vmscan_strides sC,
                    const float* D,
                    const void* z, vmscan_strides sz,
                    const float* ckpt,
                    const void* dy, vmscan_strides sdy,
                    void* du, vmscan_strides sdu,
                    void* ddelta, vmscan_strides sddelta,
                    float* dA,
                    void* dB, vmscan_strides sdB,
                    void* dC, vmscan_strides sdC,
                    float* dD,
                    void* dz, vmscan_strides sdz,
                    const vmscan_direction* dir,
                    void* workspace, size_t workspace_bytes,
                    vmscan_stream_t stream);

/*
 * Size of the device array behind vmscan_bwd_noalloc: 32 MiB, reserved on
 * every GPU that loads libvmscan.so, for as long as the library stays loaded.
 */
#define VMSCAN_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

/*
 * vmscan_bwd without a workspace argument, for callers that cannot allocate
 * device memory: for example a C or FFI binding that is handed raw input and
 * output buffers by a host framework and has no device allocator of its own,
 * or a serving process that budgets all device memory at start-up and forbids
 * allocator calls afterwards.  It has no counterpart in the reference, whose
 * VJP lets MLX allocate its outputs and (B, L, D, N) partials.
 *
 * The scratch is a file-scope device array of VMSCAN_NOALLOC_SCRATCH_BYTES;
 * a problem whose vmscan_bwd_workspace_bytes(..., recompute_ckpt = (ckpt ==
 * NULL)) exceeds it returns VMSCAN_ERR_SCRATCH without launching anything.
 * Inputs and outputs are the caller's, exactly as for vmscan_bwd.  The call
 * allocates and frees nothing.  Every call looks up the array's address in
 * the CUDA context current for the call (cudaGetSymbolAddress, as the other
 * entry points do for the status word), so nothing is cached across contexts.
 * All calls on a device share the one array
 * and it keeps the previous call's contents; nothing in it needs to start at
 * zero (every byte read is written earlier in the same call), but calls whose
 * kernels overlap on the GPU (different streams, or another thread) race on
 * it and corrupt each other's results: serialise them.
 */
int vmscan_bwd_noalloc(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state,
                       const float* u, vmscan_strides su,
                       const float* delta, vmscan_strides sdelta,
                       const float* A,
                       const float* B, vmscan_strides sB,
                       const float* C, vmscan_strides sC,
                       const float* D,
                       const float* z, vmscan_strides sz,
                       const float* ckpt,
                       const float* dy, vmscan_strides sdy,
                       float* du, vmscan_strides sdu,
                       float* ddelta, vmscan_strides sddelta,
                       float* dA,
                       float* dB, vmscan_strides sdB,
                       float* dC, vmscan_strides sdC,
                       float* dD,
                       float* dz, vmscan_strides sdz,
                       const vmscan_direction* dir,
                       vmscan_stream_t stream);

/*
 * Depthwise causal conv1d along the scan order, fused with SiLU:
 *   out[tok(p)] = silu(bias + sum_k w[c, k] * x[tok(p - K + 1 + k)])
 * where p is the scan position and tok() the direction's token map.  The
 * weight uses MLX's Conv1d layout (channels, K, 1).  Replaces
 * `silu(conv1d(x)[:, :L])`, mamba_block.py:129-132,170-171, on the permuted
 * sequence of mamba_block.py:443-534.  K in 1..8; channels % 4 == 0.
 * out_hi / out_lo (both or neither; 16-byte aligned, laid out like out)
 * also receive the TF32 hi / lo parts of out that vmscan_gemm_tf32x3 reads
 * (the x_proj GEMM's operand), so no separate vmscan_tf32_split pass is needed.
 */
int vmscan_conv1d_silu_fwd(int64_t batch, int64_t seqlen, int64_t channels, int64_t ksize,
                           const float* x, vmscan_strides sx,
                           const float* weight, const float* bias,
                           float* out, vmscan_strides sout,
                           float* out_hi, float* out_lo,
                           const vmscan_direction* dir,
                           vmscan_stream_t stream);

int64_t vmscan_conv1d_bwd_workspace_bytes(int64_t batch, int64_t seqlen, int64_t channels,
                                          int64_t ksize);

/*
 * VJP of vmscan_conv1d_silu_fwd.  dweight / dbias are overwritten.  dx_lo !=
 * NULL (16-byte aligned, laid out like dx) writes dx as its TF32 hi part into
 * dx and lo part into dx_lo (the in_proj gradient GEMMs' operand form).
 */
int vmscan_conv1d_silu_bwd(int64_t batch, int64_t seqlen, int64_t channels, int64_t ksize,
                           const float* x, vmscan_strides sx,
                           const float* weight, const float* bias,
                           const float* dout, vmscan_strides sdout,
                           float* dx, vmscan_strides sdx,
                           float* dx_lo,
                           float* dweight, float* dbias,
                           const vmscan_direction* dir,
                           void* workspace, size_t workspace_bytes,
                           vmscan_stream_t stream);

/*
 * dt_proj + bias + softplus producing the scan's delta
 * (mamba_block.py:177-181: `delta = log(1 + exp(dt_proj(x_dbc[..., :dt_rank])))`):
 *   delta[t, d] = log(1 + exp(bias[d] + sum_r x[t, r] * weight[d, r]))
 * for ntok tokens t (rows of x every ldx floats, rows of delta every
 * ld_delta floats) and d < d_inner; weight is nn.Linear's (d_inner, dt_rank)
 * row-major matrix.  dt_rank in 1..64.
 */
int vmscan_dt_softplus_fwd(int64_t ntok, int64_t dt_rank, int64_t d_inner,
                           const float* x, int64_t ldx,
                           const float* weight, const float* bias,
                           float* delta, int64_t ld_delta,
                           vmscan_stream_t stream);

/*
 * Softplus part of the VJP of vmscan_dt_softplus_fwd: dpre = ddelta *
 * sigmoid(pre) with pre recomputed from x, weight, bias (the gradient the
 * reference's autograd forms through log(1 + exp(.))).  dx = dpre weight and
 * dweight = dpre^T x are left to the caller (GEMMs).  When dpre_lo is not
 * NULL, dpre receives the TF32 hi part of dpre and dpre_lo (same row stride)
 * the lo part, the operand form of vmscan_gemm_tf32x3, instead of dpre
 * itself.  When dbias_part is not NULL it receives, as
 * vmscan_dt_softplus_bias_rows(ntok) x d_inner contiguous floats, the column
 * sums of dpre (fp32) over consecutive groups of tokens; dbias is the sum of
 * its rows (a small reduction for the caller).
 */
int vmscan_dt_softplus_bwd(int64_t ntok, int64_t dt_rank, int64_t d_inner,
                           const float* x, int64_t ldx,
                           const float* weight, const float* bias,
                           const float* ddelta, int64_t ld_ddelta,
                           float* dpre, int64_t ld_dpre, float* dpre_lo,
                           float* dbias_part,
                           vmscan_stream_t stream);

/* Rows of the dbias_part array of vmscan_dt_softplus_bwd for ntok tokens. */
int64_t vmscan_dt_softplus_bias_rows(int64_t ntok);

/*
 * Column sums of a row-major (rows x cols) fp32 array, added in a fixed
 * order (deterministic): out[c] = sum_r part[r * cols + c].  Finishes dbias of
 * vmscan_dt_softplus_bwd from its dbias_part rows (the reference's dt_proj
 * bias gradient, mamba_block.py:180 through nn.Linear's autograd).
 */
int vmscan_sum_rows(int64_t rows, int64_t cols, const float* part, float* out, vmscan_stream_t stream);

/*
 * LayerNorm over the last dimension of a (rows x dim) fp32 array (row strides
 * ld*, multiples of 4; 16-byte aligned x, y, dy, dx, weight, bias), as MLX's
 * nn.LayerNorm in the reference's blocks and encoder (mamba_block.py:201,222,
 * 401, vision_mamba.py:192): y = (x - mean) rstd weight + bias, rstd = 1 /
 * sqrt(var + eps) with the biased variance.  dim % 4 == 0 and dim <= 1024
 * (VMSCAN_ERR_SHAPE otherwise).  The forward also writes each row's mean and
 * rstd (rows floats each) for the VJP.  The VJP writes dx and the weight /
 * bias gradients (summed over rows in a fixed order: deterministic), with
 * vmscan_layernorm_bwd_workspace_bytes(rows, dim) bytes of workspace.
 */
int vmscan_layernorm_fwd(int64_t rows, int64_t dim, const float* x, int64_t ldx, const float* weight,
                         const float* bias, float eps, float* y, int64_t ldy, float* mean, float* rstd,
                         vmscan_stream_t stream);
int64_t vmscan_layernorm_bwd_workspace_bytes(int64_t rows, int64_t dim);
int vmscan_layernorm_bwd(int64_t rows, int64_t dim, const float* x, int64_t ldx, const float* weight,
                         const float* mean, const float* rstd, const float* dy, int64_t lddy, float* dx,
                         int64_t lddx, float* dweight, float* dbias, void* workspace, size_t workspace_bytes,
                         vmscan_stream_t stream);

/*
 * Projection GEMMs of the block on the tensor cores with fp32 accuracy
 * (in_proj and out_proj, mamba_block.py:165,191, the out_proj over the
 * concatenated directions performing the sum of :562-566, and their input
 * and weight gradients).
 *
 * vmscan_tf32_split writes hi = tf32(x) and lo = tf32(x - hi) (round to
 * nearest) for n floats (n % 4 == 0, 16-byte aligned buffers); x = hi + lo to
 * about 2^-22 |x|.
 *
 * vmscan_gemm_tf32x3 computes C[m, n] = sum_k A(m, k) B(n, k) for row-major C
 * (row stride ldc) from the split operands:
 *   A(m, k) = a[m * lda + k] (a_mn_major == 0) or a[k * lda + m] (!= 0),
 *   B(n, k) = b[n * ldb + k] (b_mn_major == 0) or b[k * ldb + n] (!= 0),
 * as A_hi B_hi + (A_hi B_lo + A_lo B_hi) with the large and the correction
 * products in separate fp32 accumulators.  lda, ldb: multiples of 4, all
 * operand pointers 16-byte aligned.  accumulate != 0 adds the product to C
 * (C += A B^T).  When the output tiles would not fill the GPU, K is split and
 * the partials are summed in a fixed order; that needs
 * vmscan_gemm_workspace_bytes(M, N, K) bytes of workspace (0: none; the size
 * covers either operand layout).  With an MN-major A, N > 64 and M a
 * multiple of 256 (the weight gradients) the kernel runs as clusters of two
 * CTAs; the call stays stream-ordered, synchronisation- and allocation-free.
 */
int vmscan_tf32_split(int64_t n, const float* x, float* hi, float* lo, vmscan_stream_t stream);
/* The same split for up to 16 tensors in one launch (x[k], hi[k], lo[k] of
 * n[k] floats each): a block's weights before its GEMMs. */
int vmscan_tf32_split_multi(int count, const float* const* x, float* const* hi, float* const* lo,
                            const int64_t* n, vmscan_stream_t stream);
int64_t vmscan_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);
int vmscan_gemm_tf32x3(int64_t M, int64_t N, int64_t K,
                       const float* a_hi, const float* a_lo, int64_t lda, int a_mn_major,
                       const float* b_hi, const float* b_lo, int64_t ldb, int b_mn_major,
                       float* c, int64_t ldc, int accumulate, void* workspace, int64_t workspace_bytes,
                       vmscan_stream_t stream);

/*
 * Host-only introspection (no CUDA call): writes the token index visited at
 * every scan step of `dir` into tokens[0..seqlen), computed the way the
 * kernels compute it.  mode 0 enumerates the TMA boxes (box coordinates +
 * row -> token, as the scan kernels and the dB/dC scatter do); mode 1 maps
 * each scan position directly (as the conv kernels do).  geom (may be NULL)
 * receives 16 int64 values: nsd, size[3], tstride[3], j, bj, nj, P, T,
 * nboxes, reverse, 0, 0.  No reference counterpart: it exists so the index
 * arithmetic of the direction fold is testable without a GPU.
 */
int vmscan_scan_order(int64_t seqlen, const vmscan_direction* dir, int mode, int64_t* tokens,
                      int64_t* geom);

/*
 * Exercises the device-side wait failure path: a one-warp kernel waits on an
 * mbarrier that nothing arrives on, gives up after `tries` polls (each polls
 * for at most ~1 us), sets the sticky status to VMSCAN_ERR_TIMEOUT and
 * returns.  Nothing faults; vmscan_device_status then reports and clears it.
 * No reference counterpart (the reference has no device error reporting).
 */
int vmscan_wait_timeout_selftest(uint32_t tries, vmscan_stream_t stream);

/*
 * Synchronises `stream` and returns the sticky device-side status (0 or
 * VMSCAN_ERR_TIMEOUT, set when a kernel's bounded wait ran out and the kernel
 * returned early); clears it when `clear` != 0.
 */
int vmscan_device_status(vmscan_stream_t stream, int clear);

#ifdef __cplusplus
}
#endif

#endif /* VMSCAN_H */
