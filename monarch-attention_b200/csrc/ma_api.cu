// C ABI of the MonarchAttention forward: argument validation, workspace
// layout and dispatch between the generic phase kernels and the persistent
// tcgen05 kernel.  Replaces monarch_attention_torch (ma/ma_torch.py:65-108).
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
// ma_tc.cu
bool tc_supports(const ma_fwd_params* p, const Shape& s);
size_t tc_ctrl_bytes(const Shape& s);
cudaError_t run_tc(const ma_fwd_params* p, const Shape& s, const WsLayout& ws, cudaStream_t st,
                   int* nlaunch);
}  // namespace ma

using namespace ma;

namespace {

thread_local std::string g_detail;
thread_local int g_launches = 0;

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

WsLayout make_layout(const Shape& s, int dtype) {
  WsLayout w{};
  // intermediates are kept in the input precision; e4m3 inputs use bf16
  w.store_bytes = dtype == MA_DTYPE_F32 ? 4 : 2;
  const size_t heads = (size_t)s.E * s.H;
  const size_t bm = (size_t)s.b * s.M;
  size_t off = 0;
  w.al = off; off = align_up(off + heads * bm * s.D * w.store_bytes, 256);
  w.y = off; off = align_up(off + heads * bm * s.Dv * w.store_bytes, 256);
  w.ar = off; off = align_up(off + heads * bm * s.D * w.store_bytes, 256);
  w.cl = off; off = align_up(off + heads * bm * 4, 256);
  w.cr = off; off = align_up(off + heads * bm * 4, 256);
  w.lmax = off; off = align_up(off + heads * bm * 4, 256);
  w.lsum = off; off = align_up(off + heads * bm * 4, 256);
  w.ctrl = off;
  w.ctrl_bytes = tc_ctrl_bytes(s);
  off = align_up(off + w.ctrl_bytes, 256);
  w.total = off;
  return w;
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
  const int want_out = p->dtype == MA_DTYPE_E4M3 ? MA_DTYPE_BF16 : p->dtype;
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
int select_impl(const ma_fwd_params* p, const Shape& s, int* impl) {
  const bool tc = tc_supports(p, s);
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
// Lets the allocation-free entry point (ma_noalloc.cu) report through
// ma_last_error_detail().
void set_error_detail(const std::string& detail) { g_detail = detail; }
}  // namespace ma

extern "C" {

size_t ma_workspace_bytes(const ma_fwd_params* p) {
  if (validate(p, false) != MA_OK) return 0;
  return make_layout(make_shape(p), p->dtype).total;
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
  const WsLayout ws = make_layout(s, p->dtype);
  if (p->workspace == nullptr || p->workspace_bytes < ws.total)
    return fail(MA_ERR_WORKSPACE, "workspace needs " + std::to_string(ws.total) + " bytes, got " +
                                      std::to_string(p->workspace_bytes));
  int impl = 0;
  rc = select_impl(p, s, &impl);
  if (rc != MA_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int n = 0;
  cudaError_t err = impl == MA_IMPL_TC      ? run_tc(p, s, ws, st, &n)
                    : impl == MA_IMPL_SMALL ? run_small(p, s, ws, st, &n)
                                            : run_generic(p, s, ws, st, &n);
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
