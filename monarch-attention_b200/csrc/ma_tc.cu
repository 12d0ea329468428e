// Host side of the persistent tcgen05 MonarchAttention kernel
// (ma_tc_kernel.cuh): shape support, workspace slots, tensor maps, the
// validity bitmap of masked calls, and dispatch to the compiled (b, M, D)
// instantiations (ma_tc_inst_*.cu).  Replaces the phases of
// monarch_attention_torch (ma/ma_torch.py:100-105) for those shapes.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ma_common.cuh"
#include "ma_tc_kernel.cuh"

namespace ma {
namespace tc {

// explicit instantiations live in ma_tc_inst_*.cu
#define MA_TC_DECLARE(BB, MM, DD)                                                          \
  extern template cudaError_t launch_tc<true, BB, MM, DD, false, false>(const TcParams&,    \
                                                                        int, cudaStream_t); \
  extern template cudaError_t launch_tc<false, BB, MM, DD, false, false>(const TcParams&,   \
                                                                         int, cudaStream_t);\
  extern template cudaError_t launch_tc<true, BB, MM, DD, true, false>(const TcParams&, int, \
                                                                       cudaStream_t);       \
  extern template cudaError_t launch_tc<false, BB, MM, DD, true, false>(const TcParams&, int,\
                                                                        cudaStream_t);
MA_TC_SHAPES(MA_TC_DECLARE)
#undef MA_TC_DECLARE
// e4m3 inputs read directly (f16 arithmetic): head dim 128, b = M = 64 or 128
#define MA_TC_FP8_SHAPES(X) \
  X(128, 128, 128)          \
  X(64, 64, 128)
#define MA_TC_DECLARE8(BB, MM, DD)                                                          \
  extern template cudaError_t launch_tc<false, BB, MM, DD, false, true>(const TcParams&,    \
                                                                        int, cudaStream_t); \
  extern template cudaError_t launch_tc<false, BB, MM, DD, true, true>(const TcParams&, int, \
                                                                       cudaStream_t);
MA_TC_FP8_SHAPES(MA_TC_DECLARE8)
#undef MA_TC_DECLARE8

static bool shape_compiled(int b, int M, int D) {
#define MA_TC_MATCH(BB, MM, DD) \
  if (b == BB && M == MM && D == DD) return true;
  MA_TC_SHAPES(MA_TC_MATCH)
#undef MA_TC_MATCH
  return false;
}

static cudaError_t dispatch(bool bf16, bool fp8, int b, int M, int D, const TcParams& tp,
                            int grid, cudaStream_t st) {
  const bool masked = tp.valid != nullptr;
  if (fp8) {
#define MA_TC_CALL8(BB, MM, DD)                                                  \
  if (b == BB && M == MM && D == DD)                                             \
    return masked ? launch_tc<false, BB, MM, DD, true, true>(tp, grid, st)       \
                  : launch_tc<false, BB, MM, DD, false, true>(tp, grid, st);
    MA_TC_FP8_SHAPES(MA_TC_CALL8)
#undef MA_TC_CALL8
    return cudaErrorInvalidValue;
  }
#define MA_TC_CALL(BB, MM, DD)                                                              \
  if (b == BB && M == MM && D == DD) {                                                      \
    if (masked)                                                                             \
      return bf16 ? launch_tc<true, BB, MM, DD, true, false>(tp, grid, st)                  \
                  : launch_tc<false, BB, MM, DD, true, false>(tp, grid, st);                \
    return bf16 ? launch_tc<true, BB, MM, DD, false, false>(tp, grid, st)                   \
                : launch_tc<false, BB, MM, DD, false, false>(tp, grid, st);                 \
  }
  MA_TC_SHAPES(MA_TC_CALL)
#undef MA_TC_CALL
  return cudaErrorInvalidValue;
}

// Validity of every (e, token): the caller's mask (nonzero = valid) as a
// bitmap of 32-token words; one warp per word.
__global__ void valid_bits_kernel(const void* mask, int mask_dtype, int64_t ms0, int64_t ms1,
                                  int E, int N, uint32_t* out) {
  const int words = N / 32;
  const int w = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= E * words) return;
  const int e = w / words, tok = (w - e * words) * 32 + lane;
  const bool v = mask_value(mask, mask_dtype, (int64_t)e * ms0 + (int64_t)tok * ms1);
  const uint32_t bits = __ballot_sync(0xFFFFFFFFu, v);
  if (lane == 0) out[w] = bits;
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

static bool encode(CUtensorMap* tm, CUtensorMapDataType dt, int rank, const void* base,
                   const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box) {
  auto fn = get_encode();
  if (!fn) return false;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  cuuint64_t gd[5], gs[4];
  cuuint32_t bx[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
  CUresult r = fn(tm, dt, (cuuint32_t)rank, const_cast<void*>(base), gd, gs, bx, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace tc

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

bool tc_supports(const ma_fwd_params* p, const Shape& s) {
  const char* off = getenv("MA_DISABLE_TC");
  if (off && off[0] == '1') return false;
  if (p->dtype != MA_DTYPE_BF16 && p->dtype != MA_DTYPE_F16) return false;
  if (s.D != s.Dv || s.N != s.Np) return false;
  if (!tc::shape_compiled(s.b, s.M, s.D)) return false;
  const int64_t* st[4] = {p->q_stride, p->k_stride, p->v_stride, p->o_stride};
  for (int t = 0; t < 4; ++t) {
    if (st[t][3] != 1) return false;
    for (int i = 0; i < 3; ++i)
      if ((st[t][i] * 2) % 16 != 0 || st[t][i] <= 0) return false;
  }
  if (p->q && !(aligned16(p->q) && aligned16(p->k) && aligned16(p->v) && aligned16(p->out)))
    return false;
  return true;
}

// e4m3 calls the persistent kernel reads directly (no bf16 copies): head dim
// 128, b = M = 64 or 128, q / k / v rows of 128 bytes at 16-byte aligned
// addresses.  MA_FP8_CONVERT=1 forces the conversion path instead.
bool tc_fp8_direct(const ma_fwd_params* p, const Shape& s) {
  if (p->dtype != MA_DTYPE_E4M3) return false;
  const char* conv = getenv("MA_FP8_CONVERT");
  if (conv && conv[0] == '1') return false;
  const char* off = getenv("MA_DISABLE_TC");
  if (off && off[0] == '1') return false;
  if (s.D != 128 || s.Dv != 128 || s.N != s.Np || s.b != s.M || (s.b != 64 && s.b != 128))
    return false;
  const int64_t* st[3] = {p->q_stride, p->k_stride, p->v_stride};
  for (int t = 0; t < 3; ++t) {
    if (st[t][3] != 1) return false;
    for (int i = 0; i < 3; ++i)
      if (st[t][i] % 16 != 0 || st[t][i] <= 0) return false;
  }
  const int64_t* os = p->o_stride;  // bf16 output
  if (os[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if ((os[i] * 2) % 16 != 0 || os[i] <= 0) return false;
  if (p->q && !(aligned16(p->q) && aligned16(p->k) && aligned16(p->v) && aligned16(p->out)))
    return false;
  return true;
}

// Heads per wavefront phase slot of the persistent kernel: more heads in
// flight give a longer distance between dependent tiles (a round is
// 2T * hgroup * tiles tiles).  Measured best on B200 for b = M = 128
// (1: 856 us, 2: 785 us, 3: 808 us, 4: 803 us): rounds of 256 tiles per
// phase, the same round length for the other shapes.  A call with no more
// heads than that group's slots (a shard of a few heads per GPU) runs them
// as two groups instead: the wavefront then has P + 1 rounds, and every
// round is a dependent step on the critical path (8 heads of b = M = 128:
// groups of 1: 132 us, 2: 116 us, 4: 107 us).  MA_TC_GROUP overrides it.
int tc_hgroup(const Shape& s) {
  const int nheads = s.E * s.H;
  const int tiles = s.b * s.M / tc::kT;
  int hgroup = 256 / tiles > 1 ? 256 / tiles : 1;
  if (nheads <= hgroup * (2 * s.T + 1) && (nheads + 1) / 2 > hgroup) hgroup = (nheads + 1) / 2;
  const char* hg = getenv("MA_TC_GROUP");
  if (hg) hgroup = atoi(hg);
  if (hgroup < 1) hgroup = 1;
  if (hgroup > nheads) hgroup = nheads;
  return hgroup;
}

// Workspace head slots the persistent kernel cycles through: a slot is
// reused by head h + slots once head h's output phase is done, so a group of
// hgroup heads needs hgroup * (2T + 1) slots for every dependency to point
// to an earlier round of the wavefront.
int tc_slots(const Shape& s) {
  const int nheads = s.E * s.H;
  const int want = tc_hgroup(s) * (2 * s.T + 1);
  return want < nheads ? want : nheads;
}

size_t tc_ctrl_bytes(const Shape& s) {
  return sizeof(uint32_t) * (tc::kCtrlDone + (size_t)s.E * s.H * 2 * s.T) + 256;
}

// bytes of the validity bitmap of a masked call (0 without a mask)
size_t tc_valid_bytes(const ma_fwd_params* p, const Shape& s) {
  if (p->mask_dtype == MA_MASK_NONE) return 0;
  return sizeof(uint32_t) * (size_t)s.E * (s.N / 32);
}

cudaError_t run_tc(const ma_fwd_params* p, const Shape& s, const WsLayout& ws, cudaStream_t st,
                   int* nlaunch) {
  using namespace tc;
  TcParams tp;
  memset(&tp, 0, sizeof(tp));
  // e4m3 inputs (read directly): byte tiles of q / k / v, f16 intermediates,
  // bf16 output
  const bool fp8 = p->dtype == MA_DTYPE_E4M3;
  const CUtensorMapDataType dt =
      p->dtype == MA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUtensorMapDataType dt_in = fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : dt;
  const CUtensorMapDataType dt_out = fp8 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : dt;
  const uint64_t esz = fp8 ? 1 : 2;          // bytes per q / k / v element
  const uint32_t in_box = fp8 ? 128u : 64u;  // elements per 128-byte row of a tile
  const int nheads = s.E * s.H;
  const int P = 2 * s.T;
  const int tiles = s.b * s.M / kT;  // tiles per (head, phase)
  int hgroup = tc_hgroup(s);
  // The workspace holds the arrays of ws.tc_slots heads (tc_slots() for
  // ma_fwd's layout): shrink the group to what exists.  When every head has
  // a slot of its own, no slot is reused and any group size is safe.
  const int max_slots = ws.tc_slots > 0 && ws.tc_slots < nheads ? ws.tc_slots : nheads;
  if (max_slots < nheads && hgroup * (2 * s.T + 1) > max_slots)
    hgroup = max_slots / (2 * s.T + 1) > 1 ? max_slots / (2 * s.T + 1) : 1;
  int slots = hgroup * (2 * s.T + 1);
  if (slots > max_slots) slots = max_slots;
  const uint32_t box_blk[4] = {in_box, kT, 1, 1};
  const uint32_t box_str[5] = {in_box, 1, (uint32_t)s.M, 1, 1};
  const uint32_t box_ws[2] = {64, kT};
  bool ok = true;
  auto tok_map = [&](CUtensorMap* tm, const void* base, const int64_t* es) {
    const uint64_t dims[4] = {(uint64_t)s.D, (uint64_t)s.N, (uint64_t)s.H, (uint64_t)s.E};
    const uint64_t str[3] = {(uint64_t)es[2] * esz, (uint64_t)es[1] * esz,
                             (uint64_t)es[0] * esz};
    ok = ok && encode(tm, dt_in, 4, base, dims, str, box_blk);
  };
  tok_map(&tp.tm_qblk, p->q, p->q_stride);
  tok_map(&tp.tm_kblk, p->k, p->k_stride);
  tok_map(&tp.tm_vblk, p->v, p->v_stride);
  {
    const int64_t* es = p->q_stride;
    const uint64_t dims[5] = {(uint64_t)s.D, (uint64_t)s.b, (uint64_t)s.M, (uint64_t)s.H,
                              (uint64_t)s.E};
    const uint64_t str[4] = {(uint64_t)es[2] * esz, (uint64_t)es[2] * esz * s.b,
                             (uint64_t)es[1] * esz, (uint64_t)es[0] * esz};
    ok = ok && encode(&tp.tm_qstr, dt_in, 5, p->q, dims, str, box_str);
  }
  char* w = reinterpret_cast<char*>(p->workspace);
  const uint64_t rows = (uint64_t)slots * s.b * s.M;
  {
    const uint64_t dims[2] = {(uint64_t)s.D, rows};
    const uint64_t str[1] = {(uint64_t)s.D * 2};
    ok = ok && encode(&tp.tm_al, dt, 2, w + ws.al, dims, str, box_ws);
    ok = ok && encode(&tp.tm_ar, dt, 2, w + ws.ar, dims, str, box_ws);
    const uint64_t dimy[2] = {(uint64_t)s.Dv, rows};
    const uint64_t stry[1] = {(uint64_t)s.Dv * 2};
    ok = ok && encode(&tp.tm_y, dt, 2, w + ws.y, dimy, stry, box_ws);
  }
  {
    // store views: 64 x 1 x b (al, y) and 64 x 1 x M (ar, out) boxes of strided rows
    const uint32_t box_b[3] = {64, 1, (uint32_t)s.b};
    const uint32_t box_m[3] = {64, 1, (uint32_t)s.M};
    const uint64_t dal[3] = {(uint64_t)s.D, (uint64_t)s.M, (uint64_t)slots * s.b};
    const uint64_t sal[2] = {(uint64_t)s.D * 2, (uint64_t)s.M * s.D * 2};
    ok = ok && encode(&tp.tm_al_st, dt, 3, w + ws.al, dal, sal, box_b);
    const uint64_t dy[3] = {(uint64_t)s.Dv, (uint64_t)s.M, (uint64_t)slots * s.b};
    const uint64_t sy[2] = {(uint64_t)s.Dv * 2, (uint64_t)s.M * s.Dv * 2};
    ok = ok && encode(&tp.tm_y_st, dt, 3, w + ws.y, dy, sy, box_b);
    const uint64_t dar[3] = {(uint64_t)s.D, (uint64_t)s.b, (uint64_t)slots * s.M};
    const uint64_t sar[2] = {(uint64_t)s.D * 2, (uint64_t)s.b * s.D * 2};
    ok = ok && encode(&tp.tm_ar_st, dt, 3, w + ws.ar, dar, sar, box_m);
    const int64_t* os = p->o_stride;
    const uint64_t dout[5] = {(uint64_t)s.Dv, (uint64_t)s.b, (uint64_t)s.M, (uint64_t)s.H,
                              (uint64_t)s.E};
    const uint64_t sout[4] = {(uint64_t)os[2] * 2, (uint64_t)os[2] * 2 * s.b,
                              (uint64_t)os[1] * 2, (uint64_t)os[0] * 2};
    const uint32_t box5[5] = {64, 1, (uint32_t)s.M, 1, 1};
    ok = ok && encode(&tp.tm_out_st, dt_out, 5, p->out, dout, sout, box5);
  }
  if (!ok) return cudaErrorInvalidValue;
  tp.al = w + ws.al;
  tp.ar = w + ws.ar;
  tp.y = w + ws.y;
  if (ws.clx == 0) return cudaErrorInvalidValue;  // the layout has no cl rows for this shape
  tp.clx = reinterpret_cast<uint4*>(w + ws.clx);
  tp.cr = reinterpret_cast<float*>(w + ws.cr);
  tp.ctrl = reinterpret_cast<uint32_t*>(w + ws.ctrl);
  tp.status = p->status;
  tp.status_host = p->status_host;
  if (fp8) {
    tp.qsc = p->q_scale;
    tp.ksc = p->k_scale;
    tp.vsc = p->v_scale;
  }
  tp.stall_head = tp.stall_phase = -1;
  const char* stall = getenv("MA_TEST_STALL_DEP");  // "head,phase" (tests only)
  if (stall) {
    int sh = -1, sp = -1;
    if (sscanf(stall, "%d,%d", &sh, &sp) == 2 && sh >= 0 && sh < nheads && sp >= 1 && sp < P) {
      tp.stall_head = sh;
      tp.stall_phase = sp;
    }
  }
  tp.N = s.N;
  tp.H = s.H;
  tp.nheads = nheads;
  tp.T = s.T;
  tp.P = P;
  tp.slots = slots;
  tp.hgroup = hgroup;
  const char* ea = getenv("MA_TC_EARLY");  // default on (measured faster with hgroup 2)
  tp.early = (ea && ea[0] == '0') ? 0 : 1;
  tp.claim = 2;
  const char* cl = getenv("MA_TC_CLAIM");
  if (cl) tp.claim = atoi(cl);
  if (tp.claim < 1) tp.claim = 1;
  if (tp.claim > 16) tp.claim = 16;
  tp.sm_scale = s.sm_scale;
  tp.timeout_ns = 2000000000ull;  // 2 s per bounded wait
  const char* tmo = getenv("MA_WAIT_TIMEOUT_NS");
  if (tmo) tp.timeout_ns = strtoull(tmo, nullptr, 10);
#ifdef MA_TC_TRACE
  const char* trc = getenv("MA_TC_TRACE_PTR");  // device buffer of grid x 256 x 16 u64
  if (trc) tp.trace = reinterpret_cast<unsigned long long*>(strtoull(trc, nullptr, 0));
#endif

  int dev = 0, sms = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (err != cudaSuccess) return err;
  err = cudaMemsetAsync(tp.ctrl, 0, ws.ctrl_bytes, st);
  if (err != cudaSuccess) return err;
  if (p->mask_dtype != MA_MASK_NONE) {
    if (ws.valid == 0) return cudaErrorInvalidValue;  // the layout has no bitmap
    uint32_t* vb = reinterpret_cast<uint32_t*>(w + ws.valid);
    const int words = s.E * (s.N / 32);
    valid_bits_kernel<<<(words + 7) / 8, 256, 0, st>>>(p->mask, p->mask_dtype, p->mask_stride[0],
                                                       p->mask_stride[1], s.E, s.N, vb);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    *nlaunch += 1;
    tp.valid = vb;
  }
  const int64_t items = (int64_t)nheads * P * tiles;
  const int grid = (int)(items < sms ? items : sms);
  err = dispatch(p->dtype == MA_DTYPE_BF16, fp8, s.b, s.M, s.D, tp, grid, st);
  if (err == cudaSuccess) *nlaunch += 1;
  return err;
}

}  // namespace ma
