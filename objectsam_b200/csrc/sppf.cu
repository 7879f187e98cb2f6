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
  // programmatic dependent launch: wait for the conv that wrote slice 0, let the next conv be scheduled
  grid_dep_wait();
  grid_dep_launch();
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

// SPPF backward (reference sppf_pool_bwd, src/misc.cu:48-73, :155-166): with the gradients of all four
// slices in dcat, route slice 3's gradient through pool(slice 2), add slice 2's own gradient, route that
// through pool(slice 1), add slice 1's, route through pool(slice 0) and add the result into dcat slice 0.
// Each output position sends its gradient to the FIRST maximum of its clipped 5×5 window in row-major scan
// order (strict >, the PyTorch rule).  One CTA per image × 8-channel group keeps slices 0–2, the argmax codes
// and the fp32 gradients in shared memory; routing is a gather (each input position sums, in row-major order,
// the gradients of the window positions whose argmax is itself), so the result is deterministic and no
// fp32 scratch goes through HBM.
constexpr int kSppfBwdCG = 8;

size_t sppf_bwd_smem_bytes(int H, int W) { return (size_t)H * W * (3 * 16 + 2 * kSppfBwdCG * 4 + 2 * kSppfBwdCG); }

__global__ void __launch_bounds__(256) k_sppf_bwd(const __half* __restrict__ cat, __half* __restrict__ dcat, int H,
                                                  int W, int c) {
  extern __shared__ uint4 sppfb_smem[];
  const int HW = H * W;
  const uint4* S = sppfb_smem;                                   // [3][HW] 8 fp16 values of slices 0..2
  float* G = reinterpret_cast<float*>(sppfb_smem + 3 * HW);      // [HW][8] gradient of the pool output
  float* Acc = G + HW * kSppfBwdCG;                              // [HW][8] gradient routed to the pool input
  uint8_t* arg = reinterpret_cast<uint8_t*>(Acc + HW * kSppfBwdCG);  // [HW][8] argmax code (dy+2)·5 + (dx+2)
  uint8_t* rx = arg + HW * kSppfBwdCG;                                   // [HW][8] first column of a row maximum
  const int n = blockIdx.y, g0 = blockIdx.x * kSppfBwdCG;
  const long long ctot = 4LL * c;
  const __half* img = cat + (long long)n * HW * ctot;
  __half* dimg = dcat + (long long)n * HW * ctot;
  uint4* Sw = sppfb_smem;
  for (int i = threadIdx.x; i < 3 * HW; i += blockDim.x) {
    const int k = i / HW, px = i - k * HW;
    Sw[i] = *reinterpret_cast<const uint4*>(img + px * ctot + k * c + g0);
  }
  for (int px = threadIdx.x; px < HW; px += blockDim.x) {
    float v[8];
    ld8h(dimg + px * ctot + 3 * c + g0, v);
#pragma unroll
    for (int k = 0; k < 8; k++) G[px * 8 + k] = v[k];
  }
  __syncthreads();
  for (int L = 2; L >= 0; L--) {
    const __half* SL = reinterpret_cast<const __half*>(S + L * HW);
    // First maximum of each clipped 5×5 window in row-major order, separably: per (row, column) the row
    // segment's maximum and its first column (strict >), then per output the first row whose segment
    // maximum is the largest (strict > again) — the same position as the row-major scan.  The row maxima
    // use Acc, which holds nothing live until this level's gather below.
    float* rmax = Acc;
    for (int i = threadIdx.x; i < HW * 8; i += blockDim.x) {
      const int o = i >> 3, ch = i & 7, h = o / W, w = o - h * W;
      const int x0 = w - 2 < 0 ? 0 : w - 2, x1 = w + 2 >= W ? W - 1 : w + 2;
      float best = -INFINITY;
      int bx = 255;
      for (int x = x0; x <= x1; x++) {
        const float v = __half2float(SL[(h * W + x) * 8 + ch]);
        if (v > best) {
          best = v;
          bx = x;
        }
      }
      rmax[i] = best;
      rx[i] = (uint8_t)(bx == 255 ? 255 : bx - w + 2);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < HW * 8; i += blockDim.x) {
      const int o = i >> 3, ch = i & 7, h = o / W, w = o - h * W;
      const int y0 = h - 2 < 0 ? 0 : h - 2, y1 = h + 2 >= H ? H - 1 : h + 2;
      float best = -INFINITY;
      int a = 255;
      for (int y = y0; y <= y1; y++) {
        const int j = (y * W + w) * 8 + ch;
        if (rmax[j] > best) {
          best = rmax[j];
          a = (y - h + 2) * 5 + rx[j];
        }
      }
      arg[i] = (uint8_t)a;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < HW * 8; i += blockDim.x) {
      const int p = i >> 3, h = p / W, w = p - h * W;
      // the 5 × 5 neighbours o = p + (dy, dx) in row-major order; o sends its gradient here when its argmax
      // code is that of offset (−dy, −dx): a constant per unrolled step
      float acc = 0.f;
#pragma unroll
      for (int dy = -2; dy <= 2; dy++) {
        const bool row_in = h + dy >= 0 && h + dy < H;
#pragma unroll
        for (int dx = -2; dx <= 2; dx++) {
          const int j = i + (dy * W + dx) * 8;
          if (row_in && w + dx >= 0 && w + dx < W && arg[j] == (2 - dy) * 5 + (2 - dx)) acc += G[j];
        }
      }
      Acc[i] = acc;
    }
    __syncthreads();
    if (L > 0) {
      for (int px = threadIdx.x; px < HW; px += blockDim.x) {
        float v[8];
        ld8h(dimg + px * ctot + L * c + g0, v);
#pragma unroll
        for (int k = 0; k < 8; k++) G[px * 8 + k] = Acc[px * 8 + k] + v[k];
      }
      __syncthreads();
    }
  }
  for (int px = threadIdx.x; px < HW; px += blockDim.x) {
    float v[8];
    __half* d = dimg + px * ctot + g0;
    ld8h(d, v);
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] += Acc[px * 8 + k];
    st8h(d, v);
  }
}

cudaError_t launch_sppf_bwd(const __half* cat, __half* dcat, int N, int H, int W, int c, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_sppf_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  k_sppf_bwd<<<dim3(c / kSppfBwdCG, N), 256, sppf_bwd_smem_bytes(H, W), st>>>(cat, dcat, H, W, c);
  return cudaGetLastError();
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
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(c / kSppfCG, N);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_sppf, cat, H, W, c);
}

}  // namespace osam
