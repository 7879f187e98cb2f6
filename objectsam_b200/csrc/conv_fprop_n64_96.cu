// Instantiations of the forward-convolution launcher (conv_fprop.cuh) for GEMM N tiles of 64, 96 columns.
#include "conv_fprop.cuh"

namespace osam {
template cudaError_t launch_mode<64, 64>(const ConvLaunch& L, cudaStream_t st, bool prime);
template cudaError_t launch_mode<32, 64>(const ConvLaunch& L, cudaStream_t st, bool prime);
template cudaError_t launch_mode<64, 96>(const ConvLaunch& L, cudaStream_t st, bool prime);
template cudaError_t launch_mode<32, 96>(const ConvLaunch& L, cudaStream_t st, bool prime);
}  // namespace osam
