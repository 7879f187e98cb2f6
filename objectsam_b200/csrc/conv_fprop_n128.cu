// Instantiations of the forward-convolution launcher (conv_fprop.cuh) for GEMM N tiles of 128 columns.
#include "conv_fprop.cuh"

namespace osam {
template cudaError_t launch_mode<64, 128>(const ConvLaunch& L, cudaStream_t st, bool prime);
template cudaError_t launch_mode<32, 128>(const ConvLaunch& L, cudaStream_t st, bool prime);
}  // namespace osam
