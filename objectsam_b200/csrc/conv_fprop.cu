// Forward convolution: the GEMM N tile dispatch over the instantiated launch_mode<BK, BN> (the kernel and
// its launchers are in conv_fprop.cuh), and the transposed conv's weight re-layout.
#include "conv_internal.h"

namespace osam {

// defined in conv_fprop.cuh, instantiated in conv_fprop_n*.cu
template <int BK, int BN>
cudaError_t launch_mode(const ConvLaunch& L, cudaStream_t st, bool prime);

template <int BK>
static cudaError_t launch_bn(const ConvLaunch& L, cudaStream_t st, bool prime) {
  switch (L.BN) {
    case 16: return launch_mode<BK, 16>(L, st, prime);
    case 32: return launch_mode<BK, 32>(L, st, prime);
    case 64: return launch_mode<BK, 64>(L, st, prime);
    case 96: return launch_mode<BK, 96>(L, st, prime);
    case 128: return launch_mode<BK, 128>(L, st, prime);
    case 192: return launch_mode<BK, 192>(L, st, prime);
    case 224: return launch_mode<BK, 224>(L, st, prime);
    case 256: return launch_mode<BK, 256>(L, st, prime);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_conv_fprop(const ConvLaunch& L, cudaStream_t st, bool prime_only) {
  if (L.BK == 64) return launch_bn<64>(L, st, prime_only);
  if (L.BK == 32) return launch_bn<32>(L, st, prime_only);
  return cudaErrorInvalidValue;
}

// (C, RS, K) → (RS·K, C): transposed-conv weights into the K-major B operand of its GEMM.
__global__ void k_convt_weight_relayout(const __half* __restrict__ src, __half* __restrict__ dst, int C, int RS,
                                        int K) {
  const long long n = (long long)C * RS * K;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const long long j = i / C;  // (rs, k) row of dst
    dst[i] = src[(long long)c * RS * K + j];
  }
}

cudaError_t launch_convt_weight_relayout(const __half* src, __half* dst, int C, int RS, int K, cudaStream_t st) {
  const long long n = (long long)C * RS * K;
  int grid = (int)((n + 255) / 256);
  if (grid > 4096) grid = 4096;
  k_convt_weight_relayout<<<grid, 256, 0, st>>>(src, dst, C, RS, K);
  return cudaGetLastError();
}

}  // namespace osam
