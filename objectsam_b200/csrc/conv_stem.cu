// Convolution with a tiny reduction (R·S·C ≤ 32, e.g. the 3×3/s2 RGB stem, C = 3) on the tensor cores.
//
// The reference runs this layer through cuDNN, which cannot use tensor cores at C = 3 (its own note,
// src/misc.cu:194-196, measures 4.7 TFLOP/s for the wgrad of this layer).  Here the im2col row of each
// output pixel (R·S·C taps, zero-padded to 32 fp16 = one 64-byte row) is gathered by its own thread
// straight into the 64-byte-swizzled K-major layout the UMMA descriptor reads; one elected thread
// issues two M=128 × N=BN × K=16 tcgen05 MMAs, and the same four warps run the fused epilogue.
// The layer is HBM-bound (reads 6 B, writes 64 B per output pixel), so the CTA stays small and many
// are resident per SM to hide the gather latency.
#include "epilogue.cuh"

namespace osam {

template <int BN>
__global__ void __launch_bounds__(128) k_conv_stem(const __half* __restrict__ x, const __half* __restrict__ w,
                                                   const ConvDev d) {
  constexpr int TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : 128;
  __shared__ __align__(1024) uint8_t sA[128 * 64];
  __shared__ __align__(1024) uint8_t sB[BN * 64];
  __shared__ uint64_t bar;
  __shared__ uint32_t tslot;
  __shared__ float s_sc[BN], s_sh[BN], s_bi[BN];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int RSC = d.R * d.S * d.C;

  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tslot, TMEM_COLS);
    tmem_relinquish();
  }
  // B operand: row k = the RSC weights of output channel k, zero-padded to 32, 64-byte swizzle.
  for (int i = tid; i < BN * 4; i += 128) {
    const int r = i >> 2, ch = i & 3;
    __align__(16) __half v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const int kk = ch * 8 + e;
      v[e] = (r < d.K && kk < RSC) ? w[(long long)r * RSC + kk] : __float2half(0.f);
    }
    *reinterpret_cast<uint4*>(sB + r * 64 + ((ch ^ ((r >> 1) & 3)) << 4)) = *reinterpret_cast<const uint4*>(v);
  }
  load_epilogue_consts(d.ep, d.gemm_n, 0, BN, tid, 128, s_sc, s_sh, s_bi);
  fence_proxy_async_smem();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  constexpr uint32_t idesc = idesc_f16_f32(128, BN);
  const long long ntiles = (d.M + 127) / 128;
  uint32_t phase = 0;

  for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const long long m = tile * 128 + tid;
    const bool valid = m < d.M;
    const int q = (int)(m % d.Q);
    const long long t = m / d.Q;
    const int p = (int)(t % d.P), n = (int)(t / d.P);
    // gather this pixel's im2col row
    __align__(16) __half row[32];
#pragma unroll
    for (int i = 0; i < 32; i++) row[i] = __float2half(0.f);
    if (valid) {
      for (int r = 0; r < d.R; r++) {
        const int ih = p * d.stride - d.pad + r;
        if (ih < 0 || ih >= d.H) continue;
        for (int s = 0; s < d.S; s++) {
          const int iw = q * d.stride - d.pad + s;
          if (iw < 0 || iw >= d.W) continue;
          const __half* src = x + (((long long)n * d.H + ih) * d.W + iw) * d.C;
          const int k0 = (r * d.S + s) * d.C;
          for (int c = 0; c < d.C; c++) row[k0 + c] = src[c];
        }
      }
    }
    uint8_t* dst = sA + tid * 64;
#pragma unroll
    for (int ch = 0; ch < 4; ch++)
      *reinterpret_cast<uint4*>(dst + ((ch ^ ((tid >> 1) & 3)) << 4)) = reinterpret_cast<const uint4*>(row)[ch];
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      const uint32_t a = smem_u32(sA), b = smem_u32(sB);
      umma_f16(tmem, smem_desc_kmajor(a, 64), smem_desc_kmajor(b, 64), idesc, 0);
      umma_f16(tmem, smem_desc_kmajor(a + 32, 64), smem_desc_kmajor(b + 32, 64), idesc, 1);
      umma_commit(&bar);
    }
    bool ok = mbar_wait(&bar, phase, d.err);
    phase ^= 1;
    if (!__syncthreads_and(ok)) break;
    tc_fence_after();
#pragma unroll 1
    for (int jc = 0; jc < BN / 16; jc++) {
      __syncwarp();
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + jc * 16, v);
      if (!valid) continue;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int col = jc * 16 + h * 8;
        if (col >= d.gemm_n) break;
        const int cnt = d.gemm_n - col < 8 ? d.gemm_n - col : 8;
        float y[8];
#pragma unroll
        for (int i = 0; i < 8; i++) y[i] = v[h * 8 + i];
        epilogue8(d.ep, d.K, d.P, d.Q, y, cnt, col, col, s_sc, s_sh, s_bi, m, n, p, q);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

cudaError_t launch_conv_stem(const __half* x, const __half* w, const ConvDev& d, int BN, cudaStream_t st) {
  const long long ntiles = (d.M + 127) / 128;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long cap = (long long)sms * 8;
  const int grid = (int)(ntiles < cap ? ntiles : cap);
  switch (BN) {
    case 16: k_conv_stem<16><<<grid, 128, 0, st>>>(x, w, d); break;
    case 32: k_conv_stem<32><<<grid, 128, 0, st>>>(x, w, d); break;
    case 64: k_conv_stem<64><<<grid, 128, 0, st>>>(x, w, d); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace osam
