// Persistent tcgen05/TMEM MonarchAttention kernel (large blocks).
#include "ma_common.cuh"

namespace ma {

bool tc_supports(const ma_fwd_params*, const Shape&) { return false; }
size_t tc_ctrl_bytes(const Shape&) { return 256; }
cudaError_t run_tc(const ma_fwd_params*, const Shape&, const WsLayout&, cudaStream_t, int*) {
  return cudaErrorNotSupported;
}

}  // namespace ma
