// Persistent tcgen05 kernel (ma_tc_kernel.cuh) compiled for block size
// b = 128, 128 blocks, head dim 64 (one translation unit per shape, so the
// shapes build in parallel).
#include "ma_tc_kernel.cuh"

namespace ma {
namespace tc {
template cudaError_t launch_tc<true, 128, 128, 64, false, false>(const TcParams&, int, cudaStream_t);
template cudaError_t launch_tc<true, 128, 128, 64, true, false>(const TcParams&, int, cudaStream_t);
template cudaError_t launch_tc<false, 128, 128, 64, false, false>(const TcParams&, int, cudaStream_t);
template cudaError_t launch_tc<false, 128, 128, 64, true, false>(const TcParams&, int, cudaStream_t);
}  // namespace tc
}  // namespace ma
