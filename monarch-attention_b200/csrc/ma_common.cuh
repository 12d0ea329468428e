// Shared device helpers and host-side descriptions for the MonarchAttention
// kernels (generic phase kernels in ma_generic.cu, tcgen05 kernels in ma_tc.cu
// and ma_tc256.cu, small-block kernel in ma_small.cu, e4m3 conversion in
// ma_convert.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ma_api.h"

namespace ma {

// ---------------------------------------------------------------------------
// constants of the reference algorithm (ma/ma_torch.py)
// ---------------------------------------------------------------------------
constexpr float kEps = 1e-12f;                 // ma_torch.py:10, 38
constexpr float kTiny = 1.17549435082228750797e-38f;  // torch.finfo(float32).tiny, :18

// ---------------------------------------------------------------------------
// problem description shared by host and device code
// ---------------------------------------------------------------------------
struct Shape {
  int E, H, N, D, Dv, b, M, Np, T, pre_pad, pad_off;
  float sm_scale;
};

// Byte offsets of the intermediate arrays inside the workspace.  Every array
// holds all E*H heads back to back; per head:
//   al [b][M][D]  (storage dtype)   -- R-step output, L/out-step input
//   y  [b][M][Dv] (storage dtype)   -- final R-step output
//   ar [M][b][D]  (storage dtype)   -- L-step output, R-step input
//   cl [b][M] fp32, cr [M][b] fp32  -- row/column statistics
//   clx [b][M] x 16 bytes           -- cl as a 16-bit (hi, lo) pair padded to
//                                      16 bytes (tcgen05 kernel, b = 64 / 128:
//                                      the operand of the GEMM step that
//                                      subtracts cl; 0 = not used)
//   lsex [b][M] x 16 bytes          -- the b = 256 kernel's L-step
//                                      log-sum-exp in the same form
//   lmax, lsum [b][M] fp32          -- L-step softmax statistics (generic path)
//   valid [E][N / 32] u32           -- token validity bitmap of a masked call
//                                      (tcgen05 kernel; 0 = not used)
//   ctrl                            -- dependency counters (tcgen05 path)
//   xq, xk, xv                      -- bf16 copies of e4m3 q / k / v for the
//                                      tensor-core kernels (0 = not used)
//   tc_slots                         -- heads whose al / y / ar / cl / cr
//                                      arrays exist (the tcgen05 kernel's
//                                      slot limit; every head in ma_fwd's
//                                      workspace, fewer in compact ones)
struct WsLayout {
  size_t al, y, ar, cl, cr, clx, lsex, lmax, lsum, valid, ctrl, ctrl_bytes, total;
  size_t xq, xk, xv;
  int tc_slots;
  int store_bytes;  // bytes per element of al / y / ar
};

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---------------------------------------------------------------------------
// element conversion
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <> __device__ __forceinline__ float to_f<__nv_fp8_e4m3>(__nv_fp8_e4m3 x) {
  return static_cast<float>(x);
}

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Round an fp32 value to the precision of T (identity for float).  Used where
// the reference rounds a matmul output or a matmul operand to the input dtype.
template <typename T> __device__ __forceinline__ float rnd(float x) {
  return to_f<T>(from_f<T>(x));
}
template <> __device__ __forceinline__ float rnd<float>(float x) { return x; }

// Mask truth value: nonzero = valid (logical_and semantics, ma_torch.py:96-98).
__device__ __forceinline__ bool mask_value(const void* mask, int dtype, int64_t off) {
  switch (dtype) {
    case MA_MASK_BOOL: return reinterpret_cast<const uint8_t*>(mask)[off] != 0;
    case MA_MASK_I32: return reinterpret_cast<const int32_t*>(mask)[off] != 0;
    case MA_MASK_I64: return reinterpret_cast<const int64_t*>(mask)[off] != 0;
    case MA_MASK_F32: return reinterpret_cast<const float*>(mask)[off] != 0.0f;
    case MA_MASK_F16:
    case MA_MASK_BF16:
      // +0 and -0 are false; everything else (NaN included) is true
      return (reinterpret_cast<const uint16_t*>(mask)[off] & 0x7fffu) != 0;
    default: return true;
  }
}

}  // namespace ma
