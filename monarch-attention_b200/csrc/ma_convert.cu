// e4m3 inputs for the 16-bit tensor-core kernels: dequantise q, k, v with
// their per-(e, h) scales into contiguous bf16 copies (E, H, N, D) in the
// workspace, so that the tcgen05 and small-block kernels (whose tensor-core
// operands are 16-bit) run the problem unchanged.  The reference takes fp32
// or 16-bit inputs only (ma/ma_torch.py:65-76); e4m3 with scales is this
// library's extension, specified as "the fp32 forward of the dequantised
// inputs", and rounding the dequantised value to bf16 is the one extra
// rounding this path adds.  One launch converts all three tensors; it is
// HBM-bound (1 byte read, 2 bytes written per element).
#include "ma_common.cuh"

namespace ma {
namespace conv {

struct ConvParams {
  const uint8_t* src[3];
  int64_t st[3][4];        // element strides of q, k, v
  const float* scale[3];   // per-(e, h) scales
  __nv_bfloat16* dst[3];   // contiguous (E, H, N, X)
  int X[3];                // row length (D for q, k; Dv for v)
  int E, H, N;
};

constexpr int kThreads = 256;

// 8 e4m3 values (one 64-bit word) -> scaled bf16 (one 16-byte word)
__device__ __forceinline__ uint4 convert8(uint32_t lo4, uint32_t hi4, float sc) {
  const uint32_t in[2] = {lo4, hi4};
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t pair = (in[i >> 1] >> (16 * (i & 1))) & 0xffffu;
    __nv_fp8_e4m3 lo, hi;
    lo.__x = (uint8_t)(pair & 0xff);
    hi.__x = (uint8_t)(pair >> 8);
    const __nv_bfloat162 v =
        __floats2bfloat162_rn(static_cast<float>(lo) * sc, static_cast<float>(hi) * sc);
    w[i] = *reinterpret_cast<const uint32_t*>(&v);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Vector path: rows contiguous, 16-byte aligned, X % 16 == 0.  Thread i takes
// 16 elements (one 16-byte load, two 16-byte stores); 32-bit index math
// (the host checks that rows * X / 16 fits).  blockIdx.y selects q / k / v.
__global__ void __launch_bounds__(kThreads) convert_e4m3_vec16(const ConvParams p) {
  const int t = blockIdx.y;
  const int X = p.X[t];
  const int per_row = X >> 4;
  const uint32_t total = (uint32_t)p.E * p.H * p.N * per_row;
  const uint8_t* src = p.src[t];
  const int64_t* st = p.st[t];
  const float* scale = p.scale[t];
  __nv_bfloat16* dst = p.dst[t];
  for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < total; i += gridDim.x * kThreads) {
    const uint32_t row = i / per_row;
    const uint32_t c = i - row * per_row;
    const uint32_t eh = row / p.N;
    const uint32_t n = row - eh * p.N;
    const uint32_t h = eh % p.H, e = eh / p.H;
    const uint8_t* sp = src + (int64_t)e * st[0] + (int64_t)h * st[1] + (int64_t)n * st[2] + c * 16;
    const uint4 raw = *reinterpret_cast<const uint4*>(sp);
    const float sc = scale[eh];
    uint4* dp = reinterpret_cast<uint4*>(dst + (size_t)row * X + c * 16);
    dp[0] = convert8(raw.x, raw.y, sc);
    dp[1] = convert8(raw.z, raw.w, sc);
  }
}

// Row-block path: X / 16 is a power of two dividing the block (D = 128: 8
// threads per row).  Block (head, row block) converts kRowsPerBlock rows of
// one (e, h): the head's scale and base pointer are computed once and each
// thread moves 16 elements per row it visits.
constexpr int kRowsPerBlock = 256;
__global__ void __launch_bounds__(kThreads) convert_e4m3_rows(const ConvParams p) {
  const int t = blockIdx.y;
  const int X = p.X[t];
  const int per_row = X >> 4;
  const int rows_per_step = kThreads / per_row;
  const int blocks_per_head = (p.N + kRowsPerBlock - 1) / kRowsPerBlock;
  const int eh = blockIdx.x / blocks_per_head;
  const int rb = blockIdx.x - eh * blocks_per_head;
  const int h = eh % p.H, e = eh / p.H;
  const int64_t* st = p.st[t];
  const uint8_t* src = p.src[t] + (int64_t)e * st[0] + (int64_t)h * st[1];
  __nv_bfloat16* dst = p.dst[t] + (size_t)eh * p.N * X;
  const float sc = p.scale[t][eh];
  const int c = threadIdx.x % per_row;
  const int n_end = min(p.N, (rb + 1) * kRowsPerBlock);
#pragma unroll 2
  for (int n = rb * kRowsPerBlock + threadIdx.x / per_row; n < n_end; n += rows_per_step) {
    const uint4 raw = *reinterpret_cast<const uint4*>(src + (int64_t)n * st[2] + c * 16);
    uint4* dp = reinterpret_cast<uint4*>(dst + (size_t)n * X + c * 16);
    dp[0] = convert8(raw.x, raw.y, sc);
    dp[1] = convert8(raw.z, raw.w, sc);
  }
}

// Any layout: one element per thread step, 64-bit index math.
__global__ void __launch_bounds__(kThreads) convert_e4m3_any(const ConvParams p) {
  const int t = blockIdx.y;
  const int X = p.X[t];
  const int64_t total = (int64_t)p.E * p.H * p.N * X;
  const uint8_t* src = p.src[t];
  const int64_t* st = p.st[t];
  const float* scale = p.scale[t];
  __nv_bfloat16* dst = p.dst[t];
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * kThreads) {
    const int64_t row = i / X;
    const int c = (int)(i - row * X);
    const int n = (int)(row % p.N);
    const int64_t eh = row / p.N;
    const int h = (int)(eh % p.H), e = (int)(eh / p.H);
    __nv_fp8_e4m3 v;
    v.__x = src[(int64_t)e * st[0] + (int64_t)h * st[1] + (int64_t)n * st[2] + (int64_t)c * st[3]];
    dst[row * X + c] = __float2bfloat16_rn(static_cast<float>(v) * scale[eh]);
  }
}

}  // namespace conv

// Converts q, k, v of an e4m3 problem into the bf16 copies at dq, dk, dv.
cudaError_t run_e4m3_to_bf16(const ma_fwd_params* p, const Shape& s, void* dq, void* dk, void* dv,
                             cudaStream_t st, int* nlaunch) {
  conv::ConvParams cp{};
  const void* src[3] = {p->q, p->k, p->v};
  const int64_t* strides[3] = {p->q_stride, p->k_stride, p->v_stride};
  const float* scales[3] = {p->q_scale, p->k_scale, p->v_scale};
  void* dst[3] = {dq, dk, dv};
  const int X[3] = {s.D, s.D, s.Dv};
  const int xmax = s.D > s.Dv ? s.D : s.Dv;
  const int64_t rows = (int64_t)s.E * s.H * s.N;
  bool vec = rows * (xmax / 16) < 0x7fffffffLL;
  for (int t = 0; t < 3; ++t) {
    cp.src[t] = reinterpret_cast<const uint8_t*>(src[t]);
    for (int i = 0; i < 4; ++i) cp.st[t][i] = strides[t][i];
    cp.scale[t] = scales[t];
    cp.dst[t] = reinterpret_cast<__nv_bfloat16*>(dst[t]);
    cp.X[t] = X[t];
    if (strides[t][3] != 1 || X[t] % 16 != 0 || (reinterpret_cast<uintptr_t>(src[t]) & 15) != 0 ||
        (reinterpret_cast<uintptr_t>(dst[t]) & 15) != 0)
      vec = false;
    for (int i = 0; i < 3; ++i)
      if (strides[t][i] % 16 != 0) vec = false;
  }
  cp.E = s.E; cp.H = s.H; cp.N = s.N;
  int dev = 0, sms = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (err != cudaSuccess) return err;
  const int64_t per_tensor = rows * (vec ? xmax / 16 : xmax);
  int64_t blocks = (per_tensor + conv::kThreads - 1) / conv::kThreads;
  const int64_t cap = (int64_t)sms * 8;  // grid-stride beyond 8 CTAs per SM
  if (blocks > cap) blocks = cap;
  const dim3 grid((unsigned)blocks, 3);
  // row blocks when every tensor's X / 16 is a power of two <= the block
  bool rows_path = vec;
  for (int t = 0; t < 3; ++t) {
    const int pr = X[t] / 16;
    if (pr < 1 || pr > conv::kThreads || (pr & (pr - 1)) != 0) rows_path = false;
  }
  if (rows_path) {
    const int64_t nblk = (int64_t)s.E * s.H * ((s.N + conv::kRowsPerBlock - 1) / conv::kRowsPerBlock);
    if (nblk <= 0x7fffffffLL)
      conv::convert_e4m3_rows<<<dim3((unsigned)nblk, 3), conv::kThreads, 0, st>>>(cp);
    else
      rows_path = false;
  }
  if (!rows_path) {
    if (vec)
      conv::convert_e4m3_vec16<<<grid, conv::kThreads, 0, st>>>(cp);
    else
      conv::convert_e4m3_any<<<grid, conv::kThreads, 0, st>>>(cp);
  }
  err = cudaGetLastError();
  if (err == cudaSuccess) *nlaunch += 1;
  return err;
}

}  // namespace ma
