/*
 * ma_api.h -- C ABI of the B200 MonarchAttention forward (libmonarch_attn.so).
 *
 * The reference exposes this path as one Python function,
 *   monarch_attention_torch(q, k, v, attn_mask, T, B, pre_pad)
 *     (djmmoss/monarch-attention, ma/ma_torch.py:65-73)
 * called from the MonarchAttention module's forward
 *     (ma/monarch_attention.py:39-58).
 * ma_fwd() replaces that function one for one: the same tensors (as device
 * pointers plus 4-D element strides), the same mask convention (nonzero =
 * valid, shape (E, N)), the same T / block size / pre-pad arguments and the
 * same output (a dense (E, H, N, Dv) tensor in the value dtype).
 *
 * Contract
 *   - All pointers are device pointers on the current CUDA device.
 *   - Nothing allocates and nothing synchronises: the caller provides the
 *     output, a workspace of ma_workspace_bytes() bytes and a 4-byte device
 *     status word, and the work is enqueued on `stream` (a cudaStream_t;
 *     NULL = legacy default stream).
 *   - Return value: 0 = enqueued; > 0 = invalid argument, detected on the host
 *     before anything was launched; < 0 = CUDA launch error.
 *   - Device-side failures (a bounded wait that ran out) are reported through
 *     the status word, which the kernels only ever OR bits into.  Read it with
 *     ma_read_status() after the stream has finished.
 *   - Inputs are never written.  Calls on different streams with different
 *     workspaces may run concurrently; one workspace serves one call at a time.
 */
#ifndef MONARCH_ATTN_MA_API_H_
#define MONARCH_ATTN_MA_API_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MA_API_VERSION 2

/* Element types of q / k / v / out. */
typedef enum {
  MA_DTYPE_F32 = 0,
  MA_DTYPE_F16 = 1,
  MA_DTYPE_BF16 = 2,
  MA_DTYPE_E4M3 = 3 /* q/k/v only: float8 e4m3 with per-(e,h) scales; out is bf16 */
} ma_dtype_t;

/* Element types accepted for the (E, N) attention mask; nonzero = valid,
 * exactly the truth value the reference takes with logical_and
 * (ma/ma_torch.py:96-98). */
typedef enum {
  MA_MASK_NONE = 0,
  MA_MASK_BOOL = 1, /* 1 byte: bool / uint8 / int8 */
  MA_MASK_I32 = 2,
  MA_MASK_I64 = 3,
  MA_MASK_F32 = 4,
  MA_MASK_F16 = 5,
  MA_MASK_BF16 = 6
} ma_mask_dtype_t;

/* Kernel family selection (MA_IMPL_AUTO picks the fastest that supports the
 * shape). */
typedef enum {
  MA_IMPL_AUTO = 0,
  MA_IMPL_GENERIC = 1, /* any shape/dtype: phase kernels, SIMT fp32 math   */
  MA_IMPL_TC = 2,      /* tcgen05/TMEM kernels (b, M in {32, 64, 128}, D in
                          {64, 128}; b = M = 256, D = 128)                 */
  MA_IMPL_SMALL = 3    /* fused per-head kernels (b, M <= 32): mma.sync for
                          16-bit, FFMA for fp32                            */
} ma_impl_t;

/* Return codes. */
enum {
  MA_OK = 0,
  MA_ERR_NULL_POINTER = 1,
  MA_ERR_BAD_SHAPE = 2,
  MA_ERR_BAD_DTYPE = 3,
  MA_ERR_BAD_STRIDE = 4,
  MA_ERR_BAD_MASK = 5,
  MA_ERR_WORKSPACE = 6,
  MA_ERR_UNSUPPORTED = 7,
  MA_ERR_INJECTED = 8, /* MA_FAULT_INJECT=1 in the environment */
  MA_ERR_BAD_PARAMS = 9,
  MA_ERR_CUDA = -1,
  MA_ERR_DEVICE = -2
};

/* Bits of the device status word. */
#define MA_STATUS_WAIT_TIMEOUT 0x1u /* a dependency wait exceeded its bound */
#define MA_STATUS_TMEM_FAIL 0x2u    /* tensor-memory allocation failed      */
#define MA_STATUS_BAD_ITEM 0x4u     /* scheduler produced an out-of-range item */

typedef struct {
  uint32_t struct_size; /* sizeof(ma_fwd_params): ABI guard              */
  /* tensors: q, k (E, H, N, D); v (E, H, N, Dv); out (E, H, N, Dv) */
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int64_t q_stride[4]; /* element strides of the (E, H, N, D) views      */
  int64_t k_stride[4];
  int64_t v_stride[4];
  int64_t o_stride[4];
  /* optional key/query validity mask (E, N); mask == NULL -> no mask     */
  const void* mask;
  int64_t mask_stride[2];
  int32_t mask_dtype; /* ma_mask_dtype_t                                  */
  /* sizes and algorithm arguments (ma/ma_torch.py:65-73)                 */
  int32_t E, H, N, D, Dv;
  int32_t block_size; /* B: tokens per Monarch block                      */
  int32_t num_steps;  /* T >= 1                                           */
  int32_t pre_pad;    /* 1: pad the front of the sequence                 */
  int32_t dtype;      /* ma_dtype_t of q, k, v                            */
  int32_t out_dtype;  /* = dtype; MA_DTYPE_BF16 for E4M3; F32 with v_f32  */
  /* E4M3 only: per-(e,h) dequantisation scales, E*H floats each          */
  const float* q_scale;
  const float* k_scale;
  const float* v_scale;
  /* scratch                                                              */
  void* workspace;
  size_t workspace_bytes;
  uint32_t* status; /* device word; bits MA_STATUS_* are OR-ed in          */
  int32_t impl;     /* ma_impl_t                                          */
  /* 1: v and out are fp32 while q, k are fp16 / bf16 (the reference's
   * get_matrix passes an fp32 identity as the values whatever the query
   * dtype, ma/monarch_attention.py:60-70): y and the output step then run in
   * fp32 (generic kernels).  0: v and out in the q / k dtype.              */
  int32_t v_f32;
  /* optional (NULL = none): a word of page-locked host memory that the
   * device can write (cudaHostAlloc / cudaMallocHost, same address on host
   * and device).  A kernel that sets a status bit also stores that bit here
   * with a plain store, so the host sees "a failure happened" without a
   * device read; the exact bits stay in *status.  Nothing is written on
   * success.  (API version 2; older callers leave it zero.)               */
  uint32_t* status_host;
  int32_t reserved[4];
} ma_fwd_params;

/* Bytes of workspace ma_fwd() needs for these params (0 on bad params).
 * The size depends on the kernel ma_fwd() selects (the persistent tcgen05
 * kernel cycles through a few head slots only), so pass the same params,
 * pointers included, that ma_fwd() will get; a workspace that is too small
 * for the kernel actually selected is rejected with MA_ERR_WORKSPACE. */
size_t ma_workspace_bytes(const ma_fwd_params* p);

/* Enqueue one MonarchAttention forward on `stream`
 * (replaces monarch_attention_torch, ma/ma_torch.py:65-108). */
int ma_fwd(const ma_fwd_params* p, void* stream);

/* Same forward as ma_fwd(), for callers that cannot allocate device memory
 * (e.g. a runtime whose memory pool forbids foreign allocations, or a
 * serving loop with a fixed device-memory budget where an allocation could
 * block or fail): the scratch comes from a 64 MiB
 * array compiled into the library instead of p->workspace, which is ignored.
 * This entry point has no counterpart in the reference.
 *   - Runs the persistent tcgen05 kernel only: head dim 128, block size =
 *     number of blocks = 64 or 128, bf16 / fp16, no mask; other shapes, and
 *     shapes whose scratch exceeds 64 MiB, return MA_ERR_UNSUPPORTED before
 *     anything runs.
 *   - Every GPU that loads the library keeps the 64 MiB until process exit.
 *   - All calls on a device share the array: calls that overlap on the GPU
 *     race.  The array keeps the previous call's contents; each call clears
 *     the part that must start at zero.
 *   - The first call on a device performs a one-time set-up
 *     (cudaGetSymbolAddress); make it before any stream capture.
 *   - p->status may be NULL (device-side failures are then not reported). */
int ma_fwd_noalloc(const ma_fwd_params* p, void* stream);

/* ------------------------------------------------------------------------
 * Backward pass.  The reference trains through PyTorch autograd over
 * monarch_attention_torch (ma/ma_torch.py:65-108; BART fine-tuning,
 * bart/run_summarization.py); ma_bwd() computes the same gradients
 * d<out, dout>/d(q, k, v) with CUDA kernels: the forward is recomputed with
 * every step's intermediates kept (same rounding points as ma_fwd's generic
 * kernels), then each phase is differentiated in reverse order.
 *   - fwd: the forward call's parameters (q, k, v, mask, sizes, dtype f32 /
 *     f16 / bf16; fwd.out, fwd.workspace and fwd.impl are not used).
 *   - dout: the gradient of the (E, H, N, Dv) output, element strides.
 *   - dq, dk, dv: receive the gradients in the input dtype, element strides.
 *   - Nothing allocates; the workspace is ma_bwd_workspace_bytes() bytes.
 * ------------------------------------------------------------------------ */
typedef struct {
  uint32_t struct_size; /* sizeof(ma_bwd_params)                          */
  ma_fwd_params fwd;
  const void* dout;
  int64_t dout_stride[4];
  void* dq;
  void* dk;
  void* dv;
  int64_t dq_stride[4];
  int64_t dk_stride[4];
  int64_t dv_stride[4];
  void* workspace;
  size_t workspace_bytes;
  int32_t reserved[8];
} ma_bwd_params;

/* Bytes of workspace ma_bwd() needs (0 on bad params). */
size_t ma_bwd_workspace_bytes(const ma_bwd_params* p);

/* Enqueue the backward pass on `stream`; return codes as ma_fwd(). */
int ma_bwd(const ma_bwd_params* p, void* stream);

/* Which implementation ma_fwd() would run for these params
 * (MA_IMPL_GENERIC, MA_IMPL_TC or MA_IMPL_SMALL), or a negative error code. */
int ma_select_impl(const ma_fwd_params* p);

/* Static description of a return code. */
const char* ma_error_string(int code);

/* Detail of the last error raised on the calling thread ("" if none). */
const char* ma_last_error_detail(void);

/* Copy the device status word to *status_out (synchronous on `stream`). */
int ma_read_status(const uint32_t* status_dev, void* stream, uint32_t* status_out);

/* Kernels launched by the most recent successful ma_fwd() on this thread. */
int ma_last_launch_count(void);

/* MA_API_VERSION of the built library. */
int ma_api_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MONARCH_ATTN_MA_API_H_ */
