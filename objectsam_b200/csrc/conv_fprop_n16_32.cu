// Instantiations of the forward-convolution launcher (conv_fprop.cuh) for GEMM N tiles of 16, 32 columns.
#include "conv_fprop.cuh"

namespace osam {
template cudaError_t launch_mode<64, 16>(const ConvLaunch& L, cudaStream_t st, bool prime);
template cudaError_t launch_mode<32, 16>(const ConvLaunch& L, cudaStream_t st, bool prime);
template cudaError_t launch_mode<64, 32>(const ConvLaunch& L, cudaStream_t st, bool prime);
template cudaError_t launch_mode<32, 32>(const ConvLaunch& L, cudaStream_t st, bool prime);
}  // namespace osam
