// Instantiations of the forward-convolution launcher (conv_fprop.cuh) for GEMM N tiles of 256 columns.
#include "conv_fprop.cuh"

namespace osam {
template cudaError_t launch_mode<64, 256>(const ConvLaunch& L, cudaStream_t st, bool prime);
template cudaError_t launch_mode<32, 256>(const ConvLaunch& L, cudaStream_t st, bool prime);
}  // namespace osam
