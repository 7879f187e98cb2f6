// Instantiations of the forward-convolution launcher (conv_fprop.cuh) for GEMM N tiles of 192, 224 columns.
#include "conv_fprop.cuh"

namespace osam {
template cudaError_t launch_mode<64, 192>(const ConvLaunch& L, cudaStream_t st, bool prime);
template cudaError_t launch_mode<32, 192>(const ConvLaunch& L, cudaStream_t st, bool prime);
template cudaError_t launch_mode<64, 224>(const ConvLaunch& L, cudaStream_t st, bool prime);
template cudaError_t launch_mode<32, 224>(const ConvLaunch& L, cudaStream_t st, bool prime);
}  // namespace osam
