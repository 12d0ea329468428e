// Allocation-free entry point: the persistent tcgen05 kernel driven from a
// scratch array that lives in the library itself.
//
// Who needs it: callers that cannot call cudaMalloc (or any allocator) on the
// path that runs the attention -- e.g. an embedding runtime whose memory pool
// is owned elsewhere and forbids foreign allocations, or a real-time serving
// loop with a fixed device-memory budget where an allocation could block or
// fail.  They pass q / k / v / out and nothing else; the
// kernel's scratch (the workspace slots of its intermediates and its control
// counters) comes from g_ma_noalloc_scratch below.
//
// Limits and sharing rules:
//   * the array holds kNoAllocScratchBytes (64 MiB); a shape whose scratch
//     does not fit is rejected with MA_ERR_UNSUPPORTED before anything runs;
//   * every GPU that loads this module keeps the array until the process
//     exits;
//   * every call on a device uses the same array: calls whose kernels overlap
//     on the GPU (different streams, no ordering between them) race and give
//     wrong results -- serialise them (one stream, or events);
//   * the array keeps the last call's contents; the only part that must start
//     at zero, the control counters, is cleared by every call on its stream;
//   * the first call on a device looks the array's device address up
//     (cudaGetSymbolAddress, once per device, with that device current); make
//     that first call before any stream capture that includes it.
#include <math.h>

#include <mutex>
#include <string>

#include "ma_common.cuh"

namespace ma {
// ma_tc.cu
bool tc_supports(const ma_fwd_params* p, const Shape& s);
size_t tc_ctrl_bytes(const Shape& s);
cudaError_t run_tc(const ma_fwd_params* p, const Shape& s, const WsLayout& ws, cudaStream_t st,
                   int* nlaunch);
// ma_api.cu
void set_error_detail(const std::string& detail);
void set_launch_count(int n);
}  // namespace ma

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;  // 64 MiB
constexpr int kMaxDevices = 64;

// The scratch itself.  In host code this name is only a host-side stand-in:
// host code must use the address cudaGetSymbolAddress returns for it.
static __device__ __align__(256) unsigned char g_ma_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_dev[kMaxDevices] = {};

// Device address of the scratch on the current device (set-up on first use).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_dev[dev] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_ma_noalloc_scratch);
    if (err != cudaSuccess) return err;
    g_scratch_dev[dev] = ptr;
  }
  *out = g_scratch_dev[dev];
  return cudaSuccess;
}

ma::Shape shape_of(const ma_fwd_params* p) {
  ma::Shape s{};
  s.E = p->E; s.H = p->H; s.N = p->N; s.D = p->D; s.Dv = p->Dv;
  s.b = p->block_size;
  s.M = (p->N + p->block_size - 1) / p->block_size;
  s.Np = s.M * s.b;
  s.T = p->num_steps;
  s.pre_pad = p->pre_pad ? 1 : 0;
  s.pad_off = s.pre_pad ? s.Np - s.N : 0;
  s.sm_scale = (float)(1.0 / sqrt((double)p->D));
  return s;
}

// Compact scratch layout: only the 2T+1 workspace slots the tcgen05 kernel
// cycles through (the ma_fwd workspace holds every head), then a status word
// used when the caller passes none, then the control block.
ma::WsLayout compact_layout(const ma::Shape& s, int slots, size_t* status_off) {
  ma::WsLayout w{};
  w.store_bytes = 2;
  const size_t bm = (size_t)s.b * s.M;
  size_t off = 0;
  w.al = off; off = ma::align_up(off + slots * bm * s.D * 2, 256);
  w.y = off; off = ma::align_up(off + slots * bm * s.Dv * 2, 256);
  w.ar = off; off = ma::align_up(off + slots * bm * s.D * 2, 256);
  w.cl = off; off = ma::align_up(off + slots * bm * 4, 256);
  w.cr = off; off = ma::align_up(off + slots * bm * 4, 256);
  w.clx = off; off = ma::align_up(off + slots * bm * 16, 256);
  w.tc_slots = slots;
  w.lmax = w.lsum = off;  // unused by the tcgen05 kernel
  *status_off = off; off = ma::align_up(off + 4, 256);
  w.ctrl = off;
  w.ctrl_bytes = ma::tc_ctrl_bytes(s);
  off = ma::align_up(off + w.ctrl_bytes, 256);
  w.total = off;
  return w;
}

}  // namespace

extern "C" int ma_fwd_noalloc(const ma_fwd_params* p, void* stream) {
  ma::set_error_detail("");
  const int sel = ma_select_impl(p);  // validates the parameter block
  if (sel < 0) return -sel;
  // e4m3 inputs reach the tcgen05 kernel only through bf16 copies in a
  // caller workspace, which this entry point does not have
  if (sel != MA_IMPL_TC || (p->dtype != MA_DTYPE_BF16 && p->dtype != MA_DTYPE_F16)) {
    ma::set_error_detail(
        "ma_fwd_noalloc runs the persistent tcgen05 kernel only (block size = number of "
        "blocks = 64 or 128, head dim 128, bf16/fp16, no mask); use ma_fwd for this shape");
    return MA_ERR_UNSUPPORTED;
  }
  if (!p->q || !p->k || !p->v || !p->out) {
    ma::set_error_detail("q/k/v/out is NULL");
    return MA_ERR_NULL_POINTER;
  }
  const ma::Shape s = shape_of(p);
  // the b = 256 kernel needs every head's arrays; masked calls need a bitmap
  // the static array does not hold
  if (!ma::tc_supports(p, s) || s.D != 128 || s.b != s.M || (s.b != 64 && s.b != 128) ||
      p->mask_dtype != MA_MASK_NONE) {
    ma::set_error_detail(
        "ma_fwd_noalloc runs the persistent tcgen05 kernel only (block size = number of "
        "blocks = 64 or 128, head dim 128, bf16/fp16, no mask); use ma_fwd for this shape");
    return MA_ERR_UNSUPPORTED;
  }
  const int nheads = s.E * s.H;
  const int slots = 2 * s.T + 1 < nheads ? 2 * s.T + 1 : nheads;
  size_t status_off = 0;
  const ma::WsLayout ws = compact_layout(s, slots, &status_off);
  if (ws.total > kNoAllocScratchBytes) {
    ma::set_error_detail("ma_fwd_noalloc needs " + std::to_string(ws.total) +
                         " bytes of scratch for this shape; its static array holds " +
                         std::to_string(kNoAllocScratchBytes));
    return MA_ERR_UNSUPPORTED;
  }
  void* scratch = nullptr;
  cudaError_t err = scratch_address(&scratch);
  if (err != cudaSuccess) {
    ma::set_error_detail(std::string("cudaGetSymbolAddress: ") + cudaGetErrorName(err));
    return MA_ERR_CUDA;
  }
  ma_fwd_params q = *p;
  q.workspace = scratch;
  q.workspace_bytes = ws.total;
  if (q.status == nullptr)
    q.status = reinterpret_cast<uint32_t*>(static_cast<char*>(scratch) + status_off);
  int n = 0;
  err = ma::run_tc(&q, s, ws, reinterpret_cast<cudaStream_t>(stream), &n);
  if (err != cudaSuccess) {
    ma::set_error_detail(std::string("CUDA error: ") + cudaGetErrorName(err));
    return MA_ERR_CUDA;
  }
  ma::set_launch_count(n);
  return MA_OK;
}
