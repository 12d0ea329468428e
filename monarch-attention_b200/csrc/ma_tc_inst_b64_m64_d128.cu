// Persistent tcgen05 kernel (ma_tc_kernel.cuh) compiled for block size
// b = 64, 64 blocks, head dim 128 (one translation unit per shape, so the
// shapes build in parallel).
#include "ma_tc_kernel.cuh"

namespace ma {
namespace tc {
template cudaError_t launch_tc<true, 64, 64, 128, false, false>(const TcParams&, int, cudaStream_t);
template cudaError_t launch_tc<true, 64, 64, 128, true, false>(const TcParams&, int, cudaStream_t);
template cudaError_t launch_tc<false, 64, 64, 128, false, false>(const TcParams&, int, cudaStream_t);
template cudaError_t launch_tc<false, 64, 64, 128, true, false>(const TcParams&, int, cudaStream_t);
template cudaError_t launch_tc<false, 64, 64, 128, false, true>(const TcParams&, int, cudaStream_t);
template cudaError_t launch_tc<false, 64, 64, 128, true, true>(const TcParams&, int, cudaStream_t);
}  // namespace tc
}  // namespace ma
