// SPPF pooling (YOLOv8 SPPF block): cv1's output sits in channels [0,c) of the concat buffer; the
// three chained 5×5 / stride 1 / pad 2 max-pools go to slices 1, 2, 3 (reference src/misc.cu:32-46,
// :149-153, which runs three launches over global memory).
//
// Here one CTA owns one image × one 32-channel group: it stages the slice in shared memory once and
// runs the three pools there as separable row/column maxima (max is exact, so the separable and the
// 5×5-window forms agree bit for bit, and the window is clipped at the border exactly like padding
// with −inf).  HBM traffic is the minimum: read slice 0 once, write slices 1–3 once.
#include "conv_internal.h"
#include "sm100.cuh"

namespace osam {

constexpr int kSppfCG = 32;  // channels per CTA (4 × 16-byte vectors per pixel)

__global__ void __launch_bounds__(256) k_sppf(__half* __restrict__ cat, int H, int W, int c) {
  extern __shared__ uint4 sppf_smem[];
  const int HW = H * W, V = kSppfCG / 8;  // 16-byte vectors per pixel in the group
  uint4* cur = sppf_smem;                  // [HW][V]
  uint4* tmp = sppf_smem + HW * V;         // [HW][V]
  const int n = blockIdx.y, g0 = blockIdx.x * kSppfCG;
  const long long ctot = 4LL * c;
  __half* img = cat + (long long)n * HW * ctot;

  for (int i = threadIdx.x; i < HW * V; i += blockDim.x) {
    const int px = i / V, v = i - px * V;
    cur[i] = *reinterpret_cast<const uint4*>(img + px * ctot + g0 + v * 8);
  }
  __syncthreads();
  for (int slice = 1; slice <= 3; slice++) {
    // rows: tmp[h][w] = max_{|dw|≤2} cur[h][w+dw]
    for (int i = threadIdx.x; i < HW * V; i += blockDim.x) {
      const int px = i / V, v = i - px * V, h = px / W, w = px - h * W;
      const int w0 = w - 2 < 0 ? 0 : w - 2, w1 = w + 2 >= W ? W - 1 : w + 2;
      uint4 m = cur[(h * W + w0) * V + v];
      __half2* mh = reinterpret_cast<__half2*>(&m);
      for (int x = w0 + 1; x <= w1; x++) {
        uint4 t = cur[(h * W + x) * V + v];
        const __half2* th = reinterpret_cast<const __half2*>(&t);
#pragma unroll
        for (int k = 0; k < 4; k++) mh[k] = __hmax2(mh[k], th[k]);
      }
      tmp[i] = m;
    }
    __syncthreads();
    // columns: cur[h][w] = max_{|dh|≤2} tmp[h+dh][w]; also the output of this slice
    for (int i = threadIdx.x; i < HW * V; i += blockDim.x) {
      const int px = i / V, v = i - px * V, h = px / W, w = px - h * W;
      const int h0 = h - 2 < 0 ? 0 : h - 2, h1 = h + 2 >= H ? H - 1 : h + 2;
      uint4 m = tmp[(h0 * W + w) * V + v];
      __half2* mh = reinterpret_cast<__half2*>(&m);
      for (int y = h0 + 1; y <= h1; y++) {
        uint4 t = tmp[(y * W + w) * V + v];
        const __half2* th = reinterpret_cast<const __half2*>(&t);
#pragma unroll
        for (int k = 0; k < 4; k++) mh[k] = __hmax2(mh[k], th[k]);
      }
      cur[i] = m;
      *reinterpret_cast<uint4*>(img + px * ctot + slice * c + g0 + v * 8) = m;
    }
    __syncthreads();
  }
}

cudaError_t sppf_prime() {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_sppf, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  return cudaSuccess;
}

cudaError_t launch_sppf(__half* cat, int N, int H, int W, int c, cudaStream_t st) {
  const size_t smem = size_t(2) * H * W * kSppfCG * sizeof(__half);
  cudaError_t e = sppf_prime();
  if (e != cudaSuccess) return e;
  dim3 grid(c / kSppfCG, N);
  k_sppf<<<grid, 256, smem, st>>>(cat, H, W, c);
  return cudaGetLastError();
}

}  // namespace osam
