// C ABI of the MonarchAttention forward: argument validation, workspace
// layout and dispatch between the kernel families -- the persistent tcgen05
// kernel (b = 64, 128), the per-phase tcgen05 kernel (b = 256), the fused
// small-block mma.sync kernel (b, M <= 32) and the generic phase kernels;
// e4m3 inputs reach the tensor-core ones through a conversion launch.
// Replaces monarch_attention_torch (ma/ma_torch.py:65-108).
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>

#include "ma_common.cuh"

namespace ma {
// ma_generic.cu
bool generic_supports(const Shape& s);
cudaError_t run_generic(const ma_fwd_params* p, const Shape& s, const WsLayout& ws,
                        cudaStream_t st, int* nlaunch);
// ma_small.cu
bool small_supports(const ma_fwd_params* p, const Shape& s);
cudaError_t run_small(const ma_fwd_params* p, const Shape& s, const WsLayout& ws,
                      cudaStream_t st, int* nlaunch);
// ma_convert.cu
cudaError_t run_e4m3_to_bf16(const ma_fwd_params* p, const Shape& s, void* dq, void* dk, void* dv,
                             cudaStream_t st, int* nlaunch);
// ma_tc256.cu
bool tc256_supports(const ma_fwd_params* p, const Shape& s);
cudaError_t run_tc256(const ma_fwd_params* p, const Shape& s, const WsLayout& ws,
                      cudaStream_t st, int* nlaunch);
// ma_tc.cu
bool tc_supports(const ma_fwd_params* p, const Shape& s);
int tc_slots(const Shape& s);
bool tc_fp8_direct(const ma_fwd_params* p, const Shape& s);
size_t tc_ctrl_bytes(const Shape& s);
size_t tc_valid_bytes(const ma_fwd_params* p, const Shape& s);
cudaError_t run_tc(const ma_fwd_params* p, const Shape& s, const WsLayout& ws, cudaStream_t st,
                   int* nlaunch);
}  // namespace ma

using namespace ma;

namespace {

thread_local std::string g_detail;
thread_local int g_launches = 0;
thread_local const void* g_host_word_ok = nullptr;  // last status_host that passed

// A status_host word must be page-locked host memory mapped into the device
// address space at the same address (what cudaHostAlloc / cudaMallocHost
// give with unified addressing).
bool host_word_ok(const void* ptr) {
  if (ptr == g_host_word_ok) return true;
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  if (a.type != cudaMemoryTypeHost || a.devicePointer != ptr) return false;
  g_host_word_ok = ptr;
  return true;
}

int fail(int code, const std::string& detail) {
  g_detail = detail;
  return code;
}

int elem_bytes(int dtype) {
  switch (dtype) {
    case MA_DTYPE_F32: return 4;
    case MA_DTYPE_F16: return 2;
    case MA_DTYPE_BF16: return 2;
    case MA_DTYPE_E4M3: return 1;
    default: return 0;
  }
}

Shape make_shape(const ma_fwd_params* p) {
  Shape s{};
  s.E = p->E; s.H = p->H; s.N = p->N; s.D = p->D; s.Dv = p->Dv;
  s.b = p->block_size;
  s.M = (p->N + p->block_size - 1) / p->block_size;
  s.Np = s.M * s.b;
  s.T = p->num_steps;
  s.pre_pad = p->pre_pad ? 1 : 0;
  s.pad_off = s.pre_pad ? s.Np - s.N : 0;
  s.sm_scale = (float)(1.0 / sqrt((double)p->D));  // ma_torch.py:79
  return s;
}

// Workspace layout for the kernel family `impl` (MA_IMPL_*).  conv: reserve
// bf16 copies of e4m3 q / k / v (tensor-core kernels).  The persistent
// tcgen05 kernel (b != 256) cycles through tc_slots() head slots of the
// al / y / ar / cl / cr arrays, needs no lmax / lsum, and takes a token
// validity bitmap of valid_bytes when masked; every other kernel keeps the
// arrays of all E * H heads.
WsLayout make_layout(const Shape& s, int dtype, bool conv, int impl, size_t valid_bytes,
                     bool v_f32) {
  WsLayout w{};
  // intermediates are kept in the input precision; e4m3 inputs use bf16;
  // y is kept in fp32 when the values are fp32 (v_f32)
  w.store_bytes = dtype == MA_DTYPE_F32 ? 4 : 2;
  const int y_bytes = v_f32 ? 4 : w.store_bytes;
  const bool tc = impl == MA_IMPL_TC;
  const bool persistent = tc && s.b != 256;
  const size_t heads = persistent ? (size_t)tc_slots(s) : (size_t)s.E * s.H;
  const size_t bm = (size_t)s.b * s.M;
  size_t off = 0;
  w.al = off; off = align_up(off + heads * bm * s.D * w.store_bytes, 256);
  w.y = off; off = align_up(off + heads * bm * s.Dv * y_bytes, 256);
  w.ar = off; off = align_up(off + heads * bm * s.D * w.store_bytes, 256);
  w.cl = off; off = align_up(off + heads * bm * 4, 256);
  w.cr = off; off = align_up(off + heads * bm * 4, 256);
  if (tc) {
    w.clx = off; off = align_up(off + heads * bm * 16, 256);
    if (s.b == 256) {
      w.lsex = off; off = align_up(off + heads * bm * 16, 256);
    }
  }
  if (persistent && valid_bytes > 0) {
    w.valid = off; off = align_up(off + valid_bytes, 256);
  }
  const size_t lrows = persistent ? 0 : heads * bm;
  w.lmax = off; off = align_up(off + lrows * 4, 256);
  w.lsum = off; off = align_up(off + lrows * 4, 256);
  w.ctrl = off;
  w.ctrl_bytes = tc_ctrl_bytes(s);
  w.tc_slots = (int)heads;
  off = align_up(off + w.ctrl_bytes, 256);
  if (conv) {
    const size_t rows = (size_t)s.E * s.H * (size_t)s.N;
    w.xq = off; off = align_up(off + rows * s.D * 2, 256);
    w.xk = off; off = align_up(off + rows * s.D * 2, 256);
    w.xv = off; off = align_up(off + rows * s.Dv * 2, 256);
  }
  w.total = off;
  return w;
}

// The bf16 problem an e4m3 call is run as on the tensor-core kernels: q, k, v
// replaced by their dequantised contiguous copies in the workspace (null
// pointers when `ws` is null, for shape-only checks).
ma_fwd_params bf16_view(const ma_fwd_params* p, const Shape& s, char* ws, const WsLayout& w) {
  ma_fwd_params v = *p;
  v.dtype = MA_DTYPE_BF16;
  v.out_dtype = MA_DTYPE_BF16;
  v.q = ws ? ws + w.xq : nullptr;
  v.k = ws ? ws + w.xk : nullptr;
  v.v = ws ? ws + w.xv : nullptr;
  if (!ws) v.out = nullptr;
  const int64_t n = s.N;
  const int64_t rq[4] = {(int64_t)s.H * n * s.D, n * s.D, s.D, 1};
  const int64_t rv[4] = {(int64_t)s.H * n * s.Dv, n * s.Dv, s.Dv, 1};
  for (int i = 0; i < 4; ++i) {
    v.q_stride[i] = rq[i];
    v.k_stride[i] = rq[i];
    v.v_stride[i] = rv[i];
  }
  v.q_scale = v.k_scale = v.v_scale = nullptr;
  return v;
}

// Host-side validation; nothing is launched when this fails.
int validate(const ma_fwd_params* p, bool need_buffers) {
  if (p == nullptr) return fail(MA_ERR_NULL_POINTER, "params is NULL");
  if (p->struct_size != sizeof(ma_fwd_params))
    return fail(MA_ERR_BAD_PARAMS, "struct_size " + std::to_string(p->struct_size) +
                                       " != sizeof(ma_fwd_params) " +
                                       std::to_string(sizeof(ma_fwd_params)));
  if (p->E < 1 || p->H < 1 || p->N < 1 || p->D < 1 || p->Dv < 1)
    return fail(MA_ERR_BAD_SHAPE, "E, H, N, D and Dv must all be >= 1");
  if (p->block_size < 1) return fail(MA_ERR_BAD_SHAPE, "block_size must be >= 1");
  if (p->num_steps < 1)
    return fail(MA_ERR_BAD_SHAPE, "num_steps must be >= 1");
  if (elem_bytes(p->dtype) == 0) return fail(MA_ERR_BAD_DTYPE, "unknown q/k/v dtype");
  if (p->v_f32 && p->dtype != MA_DTYPE_F16 && p->dtype != MA_DTYPE_BF16)
    return fail(MA_ERR_BAD_DTYPE, "v_f32 needs fp16 / bf16 q and k");
  const int want_out = p->v_f32 ? MA_DTYPE_F32
                                : (p->dtype == MA_DTYPE_E4M3 ? MA_DTYPE_BF16 : p->dtype);
  if (p->out_dtype != want_out)
    return fail(MA_ERR_BAD_DTYPE, "out_dtype must equal the value dtype (bf16 for e4m3)");
  if (p->mask_dtype < MA_MASK_NONE || p->mask_dtype > MA_MASK_BF16)
    return fail(MA_ERR_BAD_MASK, "unknown mask dtype");
  if (p->mask_dtype != MA_MASK_NONE && p->mask == nullptr)
    return fail(MA_ERR_BAD_MASK, "mask_dtype set but mask is NULL");
  if (p->impl < MA_IMPL_AUTO || p->impl > MA_IMPL_SMALL)
    return fail(MA_ERR_BAD_PARAMS, "unknown impl");
  if (!need_buffers) return MA_OK;
  if (!p->q || !p->k || !p->v || !p->out) return fail(MA_ERR_NULL_POINTER, "q/k/v/out is NULL");
  if (!p->status) return fail(MA_ERR_NULL_POINTER, "status word is NULL");
  if (p->status_host && !host_word_ok(p->status_host))
    return fail(MA_ERR_BAD_PARAMS,
                "status_host is not page-locked host memory the device can write at the "
                "same address");
  if (p->dtype == MA_DTYPE_E4M3 && (!p->q_scale || !p->k_scale || !p->v_scale))
    return fail(MA_ERR_NULL_POINTER, "e4m3 inputs need q/k/v scales");
  const int64_t* st[4] = {p->q_stride, p->k_stride, p->v_stride, p->o_stride};
  for (int t = 0; t < 4; ++t)
    for (int i = 0; i < 4; ++i)
      if (st[t][i] < 0) return fail(MA_ERR_BAD_STRIDE, "negative stride");
  if (p->mask_dtype != MA_MASK_NONE && (p->mask_stride[0] < 0 || p->mask_stride[1] < 0))
    return fail(MA_ERR_BAD_STRIDE, "negative mask stride");
  return MA_OK;
}

// Picks the kernel family; returns MA_OK and sets *impl, or an error code.
// e4m3 problems are checked as their bf16 view (`view`): the tensor-core
// kernels run them after a conversion launch, the generic kernels directly.
int select_impl(const ma_fwd_params* p, const Shape& s, int* impl) {
  if (p->v_f32) {  // fp32 values with 16-bit q / k: the generic kernels only
    if (p->impl == MA_IMPL_TC || p->impl == MA_IMPL_SMALL)
      return fail(MA_ERR_UNSUPPORTED, "fp32 values with 16-bit q / k run on the generic kernels");
    if (!generic_supports(s))
      return fail(MA_ERR_UNSUPPORTED, "shape exceeds the generic kernel's limits");
    *impl = MA_IMPL_GENERIC;
    return MA_OK;
  }
  if (p->dtype == MA_DTYPE_E4M3 && p->impl != MA_IMPL_GENERIC) {
    const ma_fwd_params v = bf16_view(p, s, nullptr, WsLayout{});
    // the view has no buffers yet; the output pointer is the caller's
    ma_fwd_params vo = v;
    vo.out = p->out;
    // (tc_supports checks the output alignment only together with q / k / v)
    const bool out16 = p->out == nullptr || (reinterpret_cast<uintptr_t>(p->out) & 15) == 0;
    const bool tc = (tc_supports(&vo, s) || tc256_supports(&vo, s)) && out16;
    const bool sm = small_supports(&vo, s);
    if (p->impl == MA_IMPL_TC && !tc)
      return fail(MA_ERR_UNSUPPORTED, "the tcgen05 kernel does not support this shape");
    if (p->impl == MA_IMPL_SMALL && !sm)
      return fail(MA_ERR_UNSUPPORTED, "the small-block kernel does not support this shape");
    if (p->impl == MA_IMPL_TC || (p->impl == MA_IMPL_AUTO && tc)) {
      *impl = MA_IMPL_TC;
      return MA_OK;
    }
    if (p->impl == MA_IMPL_SMALL || (p->impl == MA_IMPL_AUTO && sm)) {
      *impl = MA_IMPL_SMALL;
      return MA_OK;
    }
  }
  const bool tc = tc_supports(p, s) || tc256_supports(p, s);
  if (p->impl == MA_IMPL_TC) {
    if (!tc) return fail(MA_ERR_UNSUPPORTED, "the tcgen05 kernel does not support this shape");
    *impl = MA_IMPL_TC;
    return MA_OK;
  }
  if (p->impl == MA_IMPL_AUTO && tc) {
    *impl = MA_IMPL_TC;
    return MA_OK;
  }
  const bool sm = small_supports(p, s);
  if (p->impl == MA_IMPL_SMALL) {
    if (!sm) return fail(MA_ERR_UNSUPPORTED, "the small-block kernel does not support this shape");
    *impl = MA_IMPL_SMALL;
    return MA_OK;
  }
  if (p->impl == MA_IMPL_AUTO && sm) {
    *impl = MA_IMPL_SMALL;
    return MA_OK;
  }
  if (!generic_supports(s))
    return fail(MA_ERR_UNSUPPORTED, "shape exceeds the generic kernel's limits");
  *impl = MA_IMPL_GENERIC;
  return MA_OK;
}

}  // namespace

namespace ma {
// Let the allocation-free entry point (ma_noalloc.cu) report through
// ma_last_error_detail() and ma_last_launch_count().
void set_error_detail(const std::string& detail) { g_detail = detail; }
void set_launch_count(int n) { g_launches = n; }
}  // namespace ma

extern "C" {

size_t ma_workspace_bytes(const ma_fwd_params* p) {
  if (validate(p, false) != MA_OK) return 0;
  const Shape s = make_shape(p);
  int impl = 0;
  const std::string keep = g_detail;
  const int rc = select_impl(p, s, &impl);
  g_detail = keep;
  if (rc != MA_OK) return 0;
  const bool conv = p->dtype == MA_DTYPE_E4M3 && impl != MA_IMPL_GENERIC && !tc_fp8_direct(p, s);
  return make_layout(s, p->dtype, conv, impl, tc_valid_bytes(p, s), p->v_f32 != 0).total;
}

int ma_select_impl(const ma_fwd_params* p) {
  int rc = validate(p, false);
  if (rc != MA_OK) return -rc;
  int impl = 0;
  rc = select_impl(p, make_shape(p), &impl);
  return rc != MA_OK ? -rc : impl;
}

int ma_fwd(const ma_fwd_params* p, void* stream) {
  g_detail.clear();
  const char* inj = getenv("MA_FAULT_INJECT");
  if (inj && inj[0] == '1') return fail(MA_ERR_INJECTED, "MA_FAULT_INJECT=1");
  int rc = validate(p, true);
  if (rc != MA_OK) return rc;
  const Shape s = make_shape(p);
  int impl = 0;
  rc = select_impl(p, s, &impl);
  if (rc != MA_OK) return rc;
  // e4m3: the persistent tcgen05 kernel reads the e4m3 tiles itself where it
  // can; otherwise a conversion launch writes bf16 copies first
  const bool direct = p->dtype == MA_DTYPE_E4M3 && impl == MA_IMPL_TC && tc_fp8_direct(p, s);
  const bool conv = p->dtype == MA_DTYPE_E4M3 && impl != MA_IMPL_GENERIC && !direct;
  const WsLayout ws = make_layout(s, p->dtype, conv, impl, tc_valid_bytes(p, s), p->v_f32 != 0);
  if (p->workspace == nullptr || p->workspace_bytes < ws.total)
    return fail(MA_ERR_WORKSPACE, "workspace needs " + std::to_string(ws.total) + " bytes, got " +
                                      std::to_string(p->workspace_bytes));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int n = 0;
  cudaError_t err = cudaSuccess;
  ma_fwd_params view;
  const ma_fwd_params* run = p;
  if (conv) {  // dequantise into the bf16 copies, then run the bf16 problem
    char* w = reinterpret_cast<char*>(p->workspace);
    view = bf16_view(p, s, w, ws);
    run = &view;
    err = run_e4m3_to_bf16(p, s, w + ws.xq, w + ws.xk, w + ws.xv, st, &n);
  }
  if (err == cudaSuccess)
    err = impl == MA_IMPL_TC      ? (s.b == 256 ? run_tc256(run, s, ws, st, &n)
                                                  : run_tc(run, s, ws, st, &n))
          : impl == MA_IMPL_SMALL ? run_small(run, s, ws, st, &n)
                                  : run_generic(run, s, ws, st, &n);
  if (err != cudaSuccess)
    return fail(MA_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorName(err) + ": " +
                                 cudaGetErrorString(err));
  g_launches = n;
  return MA_OK;
}

const char* ma_error_string(int code) {
  switch (code) {
    case MA_OK: return "ok";
    case MA_ERR_NULL_POINTER: return "a required pointer is NULL";
    case MA_ERR_BAD_SHAPE: return "invalid shape or algorithm argument";
    case MA_ERR_BAD_DTYPE: return "invalid or inconsistent dtype";
    case MA_ERR_BAD_STRIDE: return "invalid stride";
    case MA_ERR_BAD_MASK: return "invalid attention mask";
    case MA_ERR_WORKSPACE: return "workspace missing or too small";
    case MA_ERR_UNSUPPORTED: return "shape not supported by the selected kernel";
    case MA_ERR_INJECTED: return "injected failure (MA_FAULT_INJECT)";
    case MA_ERR_BAD_PARAMS: return "malformed parameter block";
    case MA_ERR_CUDA: return "CUDA launch error";
    case MA_ERR_DEVICE: return "device-side failure reported through the status word";
    default: return "unknown error";
  }
}

const char* ma_last_error_detail(void) { return g_detail.c_str(); }

int ma_read_status(const uint32_t* status_dev, void* stream, uint32_t* status_out) {
  if (!status_dev || !status_out) return MA_ERR_NULL_POINTER;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t err = cudaMemcpyAsync(status_out, status_dev, sizeof(uint32_t),
                                    cudaMemcpyDeviceToHost, st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(st);
  if (err != cudaSuccess)
    return fail(MA_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorName(err));
  return MA_OK;
}

int ma_last_launch_count(void) { return g_launches; }

int ma_api_version(void) { return MA_API_VERSION; }

}  // extern "C"
