// 3×3 / stride 1 / pad 1 convolution for narrow layers (C, K ∈ {32, 64}) from one shared input window.
//
// The implicit GEMM of conv_fprop.cu fetches one 128-pixel TMA box per tap: for these narrow layers nine
// small boxes per tile leave the tensor cores and HBM mostly idle.  Here the output is indexed in a
// row-flattened space of pitch Wp ≥ W + 2 (W + 2 rounded up to 32): position u = p·Wp + q, columns q ≥ W
// are junk.  With the input indexed the same way after a zero border (X'[p'][q'] = X[p'−1][q'−1], zero for
// q' = 0 and q' > W), tap (r, c) of output u reads input u + r·Wp + c: every tap of a 128-position tile is
// the SAME window of 128 + 2·Wp + 2 input positions read from a fixed offset.  The window is kept in the
// no-swizzle K-major layout — C/8 slabs, each one 16-byte row (8 channels) per position — in which an UMMA
// operand may start at any position, so the nine taps cost nine descriptor offsets and the window is
// loaded once per tile.
//
// One CTA per SM, 13 warps:
//   warps 0–3  window producers: 16-byte cp.async gathers from NHWC (zero-filled border) into two or
//              three rotating window buffers; each thread fences its own copies and arrives on the
//              buffer's barrier once they have landed (two tiles in flight per thread);
//   warp 4     TMEM allocator, weight loader (all nine taps, TMA, once per CTA) and the single-thread
//              tcgen05.mma issuer (M=128, N=K, K=16) into one of two TMEM accumulators;
//   warps 5–12 epilogue: two warps per TMEM lane quadrant taking alternate tiles (accumulator buffer
//              0 or 1); a warp's 32 positions are one output row segment, stored by the TMA-store path of
//              epilogue.cuh (junk columns fall outside the tensor and are clipped); the residual rows of a
//              warp's next tile are prefetched into its own shared buffer while that tile's MMAs run.
// No multicast.  Every wait is bounded (sm100.cuh).
#include "epilogue.cuh"

namespace osam {

constexpr int kWinBuffers = 3;  // at most; the plan picks 2 or 3

template <int C, int K>
struct WinCfg {
  static constexpr int SLABS = C / 8;
  static constexpr int PROD_WARPS = 4;
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 32 * (PROD_WARPS + 1 + EPI_WARPS);
  static constexpr int PROD_THREADS = 32 * PROD_WARPS;
  static constexpr int ACC_COLS = K;               // 32 or 64
  static constexpr int TMEM_COLS = 2 * ACC_COLS;   // double-buffered accumulator (64 or 128)
  static constexpr int PASSES = K / 32;            // 32-column epilogue passes per tile
  static constexpr int RES_BYTES = 32 * K * 2;     // one warp's residual rows (PASSES × 32 × 64 B)
  static constexpr int ROW_BYTES_B = C * 2;        // weight rows: 64 B (SW64) or 128 B (SW128)
  static constexpr int B_TAP_BYTES = K * C * 2;    // one tap's weights (a multiple of 1024)
  static constexpr int B_BYTES = 9 * B_TAP_BYTES;
  static constexpr int STAGE_OUT_BYTES = EPI_WARPS * 32 * 64;
  static constexpr int CONST_BYTES = 2 * 64 * 4;
  static_assert(B_TAP_BYTES % 1024 == 0, "weight taps must stay 1024-byte aligned");
};

size_t win_fixed_smem_bytes(int C, int K) {
  // alignment slack, weights, epilogue stages, residual buffers, epilogue constants, barriers + TMEM slot
  const size_t b = (size_t)9 * K * C * 2;
  return 1024 + b + (size_t)8 * 32 * 64 + (size_t)8 * 32 * K * 2 + 2 * 64 * 4 + (2 * kWinBuffers + 4 + 1) * 8 + 16;
}

template <int C, int K>
__global__ void __launch_bounds__(WinCfg<C, K>::THREADS, 1)
    k_conv_win(const __grid_constant__ CUtensorMap tb, const __grid_constant__ StoreMaps sm, const ConvDev d,
               const __half* __restrict__ x) {
  using Cfg = WinCfg<C, K>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = base;                                  // 9 taps of weights, SW64/SW128 K-major
  uint8_t* sW = sB + Cfg::B_BYTES;                     // kWinBuffers windows
  const int SLAB = d.win_slab, WBYTES = d.win_wbytes, Wp = d.win_wp, LW = d.win_lw, TPI = d.win_tpi;
  const int NWB = d.win_nwb;
  const unsigned MUL = d.win_mul;
  uint8_t* s_stage = sW + NWB * WBYTES;                // epilogue stages (WBYTES % 1024 == 0)
  uint8_t* s_res = s_stage + Cfg::STAGE_OUT_BYTES;     // per-warp residual rows
  float* s_sc = reinterpret_cast<float*>(s_res + 8 * Cfg::RES_BYTES);
  float* s_sh = s_sc + 64;
  uint64_t* wfull = reinterpret_cast<uint64_t*>(s_sh + 64);
  uint64_t* wempty = wfull + kWinBuffers;
  uint64_t* accf = wempty + kWinBuffers;  // [2]
  uint64_t* acce = accf + 2;              // [2]
  uint64_t* bfull = acce + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bfull + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = d.tiles_m;
  const int P = d.P, W = d.W, H = d.H;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NWB; s++) {
      mbar_init(wfull + s, Cfg::PROD_THREADS);
      mbar_init(wempty + s, 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(accf + b, 1);
      mbar_init(acce + b, Cfg::EPI_WARPS / 2);  // the four warps that take buffer b's tiles
    }
    mbar_init(bfull, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tb);
  }
  if (warp == 4) {
    tmem_alloc(tslot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp >= 5)
    load_epilogue_consts(d.ep, d.gemm_n, 0, d.gemm_n, threadIdx.x - 32 * 5, 32 * Cfg::EPI_WARPS, s_sc, s_sh);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp < Cfg::PROD_WARPS) {
    // ---------------------------------------------------------------- window producers
    const int pt = threadIdx.x;
    uint32_t it = 0;
    int prev = -1;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, it++) {
      const int wb = it % NWB;
      if (it >= (uint32_t)NWB) {
        const uint32_t ph = ((it / NWB) - 1) & 1;
        if (!mbar_test(wempty + wb, ph)) {
          // the buffer is still in use: publish the pending window first, so that its MMAs do not wait
          // for this one (with two buffers they would otherwise serialise with the copies)
          if (prev >= 0) {
            cp_async_wait_all();
            fence_proxy_async_smem();
            mbar_arrive(wfull + prev);
            prev = -1;
          }
          if (!mbar_wait(wempty + wb, ph, d.err)) {
            ok = false;
            break;
          }
        }
      }
      const int n = t / TPI, u0 = (t - n * TPI) * 128;
      const uint32_t wbase = smem_u32(sW + wb * WBYTES);
      const __half* xn = x + (long long)n * H * W * C;
      // one window position (all C/8 slabs) per thread and step: a warp reads 32 whole pixels
      for (int k = pt; k < LW; k += Cfg::PROD_THREADS) {
        const int up = u0 + k, pp = (int)__umulhi((unsigned)up, MUL), qp = up - pp * Wp;  // padded coordinates
        const bool in = pp >= 1 && pp <= H && qp >= 1 && qp <= W;
        const __half* src = in ? xn + ((long long)(pp - 1) * W + (qp - 1)) * C : x;
        const uint32_t dst = wbase + k * 16;
#pragma unroll
        for (int g = 0; g < Cfg::SLABS; g++) cp_async16(dst + g * SLAB, in ? src + 8 * g : x, in ? 16u : 0u);
      }
      cp_async_commit();
      if (prev >= 0) {  // the previous window's copies of this thread have landed
        cp_async_wait_1();
        fence_proxy_async_smem();
        mbar_arrive(wfull + prev);
      }
      prev = wb;
    }
    if (prev >= 0) {
      cp_async_wait_all();
      fence_proxy_async_smem();
      mbar_arrive(wfull + prev);
    }
  } else if (warp == 4) {
    // ---------------------------------------------------------------- weights + MMA issuer
    if (lane == 0) {
      mbar_arrive_expect_tx(bfull, Cfg::B_BYTES);
      for (int tap = 0; tap < 9; tap++) tma_load_2d(sB + tap * Cfg::B_TAP_BYTES, &tb, bfull, tap * C, 0);
      constexpr uint32_t idesc = idesc_f16_f32(128, K);
      bool ok = mbar_wait(bfull, 0, d.err);
      uint32_t it = 0;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, it++) {
        const int wb = it % NWB;
        const uint32_t buf = it & 1;
        if (it >= 2 && !mbar_wait(acce + buf, ((it >> 1) - 1) & 1, d.err)) break;
        if (!mbar_wait(wfull + wb, (it / NWB) & 1, d.err)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sW + wb * WBYTES), b0 = smem_u32(sB);
        const uint32_t dt = tmem + buf * Cfg::ACC_COLS;
#pragma unroll
        for (int tap = 0; tap < 9; tap++) {
          const int r = tap / 3, c = tap - r * 3;
          const uint32_t off = (uint32_t)(r * Wp + c) * 16u;
#pragma unroll
          for (int kc = 0; kc < C / 16; kc++)
            umma_f16(dt, smem_desc_kmajor_noswz(a0 + (2 * kc) * SLAB + off, (uint32_t)SLAB, 128u),
                     smem_desc_kmajor(b0 + tap * Cfg::B_TAP_BYTES + kc * 32, Cfg::ROW_BYTES_B), idesc,
                     (tap | kc) != 0);
        }
        umma_commit(wempty + wb);
        umma_commit(accf + buf);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 5..12)
    const EpiDev& e = d.ep;
    const int ew = warp - 5;
    const int quad = warp & 3;
    const int half = ew >> 2;  // takes the tiles of accumulator buffer `half`
    uint8_t* stage = s_stage + ew * (32 * 64);
    uint8_t* rsm = s_res + ew * Cfg::RES_BYTES;
    const bool has_res = e.kind == OSAM_EPI_BN_ACT && e.res != nullptr;
    // the warp's 32 positions of tile t: output row p, columns q0 … q0 + 31 of image n
    auto locate = [&](int t, int& n, int& p, int& q0) {
      n = t / TPI;
      const int uw = (t - n * TPI) * 128 + quad * 32;
      p = (int)__umulhi((unsigned)uw, MUL);
      q0 = uw - p * Wp;
    };
    auto prefetch_res = [&](int t) {  // residual rows of tile t → rsm (PASSES × 32 rows × 64 B)
      int n, p, q0;
      locate(t, n, p, q0);
#pragma unroll
      for (int j = lane; j < 32 * (K / 8); j += 32) {
        const int r = j / (K / 8), ch = j - r * (K / 8);
        const bool in = p < P && q0 + r < W;
        const __half* src = in ? e.res + (((long long)n * P + p) * d.Q + q0 + r) * K + 8 * ch : e.res;
        cp_async16(smem_u32(rsm + (ch >> 2) * 2048 + stage_off(r, ch & 3)), src, in ? 16u : 0u);
      }
      cp_async_commit();
    };
    uint32_t it = half;
    int t = blockIdx.x + half * gridDim.x;
    if (has_res && t < ntiles) prefetch_res(t);
    for (; t < ntiles; t += 2 * gridDim.x, it += 2) {
      int n, p, q0;
      locate(t, n, p, q0);
      const int q = q0 + lane;
      const bool valid = q < W && p < P;
      const bool ok = mbar_wait(accf + half, (it >> 1) & 1, d.err);
      tc_fence_after();
      if (!ok) break;
      if (has_res) cp_async_wait_all();
      __syncwarp();
      const uint32_t dt = tmem + half * Cfg::ACC_COLS + ((uint32_t)(quad * 32) << 16);
      const int passes = (q0 < W && p < P) ? Cfg::PASSES : 0;  // no store for a segment wholly outside
#pragma unroll 1
      for (int ps = 0; ps < passes; ps++) {
        uint32_t r0[16], r1[16];
        tmem_ld16_nowait(dt + ps * 32, r0);
        tmem_ld16_nowait(dt + ps * 32 + 16, r1);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int i = 0; i < 16; i++) {
          v[i] = __uint_as_float(r0[i]);
          v[16 + i] = __uint_as_float(r1[i]);
        }
        epilogue_warp_tma(e, sm, K, P, d.Q, v, ps * 32, s_sc, s_sh, valid, n, p, q, q0, p, n, stage,
                          has_res ? rsm + ps * 2048 : nullptr);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce + half);
      if (has_res && t + 2 * gridDim.x < ntiles) prefetch_res(t + 2 * gridDim.x);
    }
    if (lane == 0) bulk_wait_group0();  // tensor stores complete before the CTA retires
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

template <int C, int K>
static cudaError_t win_launch_one(const ConvLaunch& L, cudaStream_t st, bool prime_only) {
  using Cfg = WinCfg<C, K>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(k_conv_win<C, K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kWinSmemLimit);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  if (prime_only) return cudaSuccess;
  const ConvDev& d = L.d;
  const size_t smem = win_fixed_smem_bytes(C, K) + (size_t)d.win_nwb * d.win_wbytes;
  if (smem > kWinSmemLimit || d.win_nwb < 2 || d.win_nwb > kWinBuffers || d.win_wbytes % 1024 != 0 ||
      d.win_slab % 16 != 0 || d.win_wp % 32 != 0 || !d.ep.tstore ||
      (size_t)d.win_slab * (C / 8) > (size_t)d.win_wbytes || d.win_lw < 128 + 2 * d.win_wp + 2)
    return cudaErrorInvalidValue;
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int grid = L.grid < sms ? L.grid : sms;
  k_conv_win<C, K><<<grid, Cfg::THREADS, smem, st>>>(L.tb, L.sm, L.d, L.x);
  return cudaGetLastError();
}

cudaError_t launch_conv_win(const ConvLaunch& L, cudaStream_t st, bool prime_only) {
  const int C = L.d.C, K = L.d.K;
  if (C == 32 && K == 32) return win_launch_one<32, 32>(L, st, prime_only);
  if (C == 32 && K == 64) return win_launch_one<32, 64>(L, st, prime_only);
  if (C == 64 && K == 32) return win_launch_one<64, 32>(L, st, prime_only);
  if (C == 64 && K == 64) return win_launch_one<64, 64>(L, st, prime_only);
  return cudaErrorInvalidValue;
}

}  // namespace osam
