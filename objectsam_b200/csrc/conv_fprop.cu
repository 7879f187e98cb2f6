// Forward convolution as an implicit GEMM on the sm_100a tensor cores.
//
//   GEMM M = output pixels (a 128-pixel tile: tn images × th rows × tw columns, or 128 consecutive rows
//            of the [N·H·W, C] matrix for 1×1 convs), GEMM N = output channels (BN per tile),
//   GEMM K = taps × input channels, walked as (tap, BK-channel chunk) steps.
//
// Persistent kernel: each CTA walks the tile list (tile = blockIdx.x + i·gridDim.x, output-channel tile
// fastest so neighbouring CTAs share their A windows in L2).  Two CTAs per SM with 6 warps each when
// BN ≤ 128, one CTA with 10 warps for wider tiles:
//   warp 0      TMA producer: per K-step one A box (the input window of this tap, halo = TMA zero fill)
//               and one B box (KRSC weight rows) into a STAGES-deep ring; it runs ahead across tiles;
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16), accumulating into
//               one of TWO TMEM buffers, so the MMAs of tile i+1 overlap the epilogue of tile i;
//   warps 2..   epilogue: one (BN ≤ 128) or two (wider, each taking half of the columns) warps per TMEM
//               lane quadrant:
//               tcgen05.ld, folded BN + SiLU (+ residual) or bias, fp16 conversion and the
//               multi-destination store (channel slices, 2× nearest upsample) — written back through a
//               per-warp shared-memory stage so that each store instruction covers whole pixel rows
//               (epilogue.cuh).  This replaces the reference's separate bn_forward_apply / add_bias passes.
// Operand tiles are K-major with the TMA swizzle (128 B rows for BK = 64, 64 B rows for BK = 32) the UMMA
// shared-memory descriptor expects.  No multicast anywhere.  Every wait is bounded (sm100.cuh).
#include "epilogue.cuh"

namespace osam {

constexpr int kMaxGemmN = 512;  // per-column epilogue constants cached in shared memory

template <int BK, int BN>
struct FpropCfg {
  static constexpr int A_BYTES = 128 * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // ≤ 128 output channels: two CTAs per SM, each with 4 epilogue warps (two independent load/MMA
  // pipelines hide TMA latency better); wider tiles: one CTA per SM with 8 epilogue warps.
  static constexpr int CTAS_PER_SM = BN <= 128 ? 2 : 1;
  static constexpr int EPI_WARPS = BN <= 128 ? 4 : 8;
  static constexpr int RING_BUDGET = BN <= 128 ? 96 * 1024 : 196 * 1024;
  static constexpr int STAGES_RAW = RING_BUDGET / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW < 2 ? 2 : (STAGES_RAW > 8 ? 8 : STAGES_RAW);
  static constexpr int ACC_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr int TMEM_COLS = 2 * ACC_COLS;  // double-buffered accumulator
  static constexpr int ROW_BYTES = BK * 2;
  static constexpr int CONST_BYTES = 2 * kMaxGemmN * 4;
  static constexpr int STAGE_OUT_BYTES = EPI_WARPS * 32 * 64;  // per-warp epilogue stage
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + STAGE_OUT_BYTES + CONST_BYTES + 256;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
};

template <int BK, int BN, int MODE>
__global__ void __launch_bounds__(FpropCfg<BK, BN>::THREADS, FpropCfg<BK, BN>::CTAS_PER_SM)
    k_conv_fprop(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                 const __grid_constant__ StoreMaps sm, const ConvDev d) {
  using Cfg = FpropCfg<BK, BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + STAGES * Cfg::A_BYTES;
  uint8_t* s_stage = base + STAGES * Cfg::STAGE_BYTES;  // 1024-aligned: the TMA store swizzle needs 512
  float* s_sc = reinterpret_cast<float*>(s_stage + Cfg::STAGE_OUT_BYTES);
  float* s_sh = s_sc + kMaxGemmN;
  uint64_t* full = reinterpret_cast<uint64_t*>(s_sh + kMaxGemmN);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;  // [2] accumulator ready (MMA → epilogue)
  uint64_t* acce = accf + 2;        // [2] accumulator drained (epilogue → MMA), one arrival per epilogue warp
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acce + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = d.tiles_m * d.ntn;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(accf + b, 1);
      mbar_init(acce + b, Cfg::EPI_WARPS);
    }
    fence_barrier_init();
    tma_prefetch_desc(&ta);
    tma_prefetch_desc(&tb);
  }
  if (warp == 1) {
    tmem_alloc(tslot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp >= 2)
    load_epilogue_consts(d.ep, d.gemm_n, 0, d.gemm_n, threadIdx.x - 64, 32 * Cfg::EPI_WARPS, s_sc, s_sh);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const int nt = t % d.ntn, mt = t / d.ntn, n0 = nt * BN;
        int q0 = 0, p0 = 0, b0 = 0, m0 = 0;
        if (MODE == A_GEMM) {
          m0 = mt * 128;
        } else {
          const int tq = mt % d.tiles_q, rest = mt / d.tiles_q;
          q0 = tq * d.tw;
          p0 = (rest % d.tiles_p) * d.th;
          b0 = (rest / d.tiles_p) * d.tn;
        }
        for (int kb = 0; kb < d.nk; kb++, it++) {
          const int s = it % STAGES;
          if (it >= STAGES && !mbar_wait(empty + s, ((it / STAGES) - 1) & 1, d.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full + s, Cfg::STAGE_BYTES);
          const int tap = kb / d.nkc, cc = (kb - tap * d.nkc) * BK;
          uint8_t* a = sA + s * Cfg::A_BYTES;
          uint8_t* b = sB + s * Cfg::B_BYTES;
          if (MODE == A_GEMM) {
            tma_load_2d(a, &ta, full + s, cc, m0);
          } else {
            const int r = tap / d.S, c = tap - r * d.S;
            if (MODE == A_S1) {
              tma_load_4d(a, &ta, full + s, cc, q0 + c - d.pad, p0 + r - d.pad, b0);
            } else {
              const int dr = r - d.pad, dc = c - d.pad;
              tma_load_5d(a, &ta, full + s, (dc & 1) * d.C + cc, q0 + (dc >> 1), dr & 1, p0 + (dr >> 1), b0);
            }
          }
          tma_load_2d(b, &tb, full + s, tap * d.C + cc, n0);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, BN);
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, lt++) {
        const uint32_t buf = lt & 1;
        if (lt >= 2 && !mbar_wait(acce + buf, ((lt >> 1) - 1) & 1, d.err)) break;
        tc_fence_after();
        const uint32_t dt = tmem + buf * Cfg::ACC_COLS;
        for (int kb = 0; kb < d.nk; kb++, it++) {
          const int s = it % STAGES;
          if (!mbar_wait(full + s, (it / STAGES) & 1, d.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(sA + s * Cfg::A_BYTES), b = smem_u32(sB + s * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; k++)
            umma_f16(dt, smem_desc_kmajor(a + k * 32, Cfg::ROW_BYTES), smem_desc_kmajor(b + k * 32, Cfg::ROW_BYTES),
                     idesc, (kb | k) != 0);
          umma_commit(empty + s);
        }
        if (ok) umma_commit(accf + buf);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..)
    const EpiDev& e = d.ep;
    const int ew = warp - 2;                 // 0..EPI_WARPS-1
    const int quad = warp & 3;               // TMEM lane quadrant this warp may access
    const int half = ew >> 2;                // which half of the tile's columns (8 epilogue warps)
    const int row = quad * 32 + lane;
    // 8 epilogue warps: the first half takes the leading ceil32(BN/2) columns, the second the rest, so
    // both halves are multiples of 32 for every BN % 32 == 0 (e.g. 224 → 128 + 96).
    constexpr int SPLIT = ((BN / 2 + 31) / 32) * 32;
    const int cols = Cfg::EPI_WARPS == 4 ? BN : (half == 0 ? SPLIT : BN - SPLIT);
    const int cbeg = Cfg::EPI_WARPS == 4 ? 0 : half * SPLIT;
    uint8_t* stage = s_stage + ew * (32 * 64);
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, lt++) {
      const int nt = t % d.ntn, mt = t / d.ntn, n0 = nt * BN;
      bool valid;
      long long pix;
      int n, p, q;
      if (MODE == A_GEMM) {
        const long long m = (long long)mt * 128 + row;
        valid = m < d.M;
        pix = m;
        q = (int)(m % d.Q);
        const long long tt = m / d.Q;
        p = (int)(tt % d.P);
        n = (int)(tt / d.P);
      } else {
        const int tq = mt % d.tiles_q, rest = mt / d.tiles_q;
        const int thw = d.th * d.tw;
        const int ni = row / thw, rr = row - ni * thw, i = rr / d.tw, j = rr - i * d.tw;
        n = (rest / d.tiles_p) * d.tn + ni;
        p = (rest % d.tiles_p) * d.th + i;
        q = tq * d.tw + j;
        valid = n < d.N && p < d.P && q < d.Q;
        pix = ((long long)n * d.P + p) * d.Q + q;
      }
      int bq = 0, bp = 0, bn = 0;  // origin of this warp's 32-row box (TMA-store epilogue)
      if (MODE != A_GEMM) {
        const int tq = mt % d.tiles_q, rest = mt / d.tiles_q;
        const int w0 = quad * 32, thw = d.th * d.tw;
        bq = tq * d.tw + w0 % d.tw;
        bp = (rest % d.tiles_p) * d.th + (w0 / d.tw) % d.th;
        bn = (rest / d.tiles_p) * d.tn + w0 / thw;
      }
      const uint32_t buf = lt & 1;
      const bool ok = mbar_wait(accf + buf, (lt >> 1) & 1, d.err);
      tc_fence_after();
      if (!ok) break;
      const uint32_t dt = tmem + buf * Cfg::ACC_COLS + ((uint32_t)(quad * 32) << 16);
      if (e.tstore) {
#pragma unroll 1
        for (int c = 0; c < cols; c += 32) {
          __syncwarp();
          uint32_t r0[16], r1[16];
          tmem_ld16_nowait(dt + cbeg + c, r0);
          tmem_ld16_nowait(dt + cbeg + c + 16, r1);
          tmem_wait_ld();
          float v[32];
#pragma unroll
          for (int i = 0; i < 16; i++) {
            v[i] = __uint_as_float(r0[i]);
            v[16 + i] = __uint_as_float(r1[i]);
          }
          epilogue_warp_tma(e, sm, d.K, d.P, d.Q, v, n0 + cbeg + c, s_sc, s_sh, valid, n, p, q, bq, bp, bn, stage);
        }
      } else if (e.coop) {
#pragma unroll 1
        for (int c = 0; c < cols;) {
          __syncwarp();
          const int col = n0 + cbeg + c;
          if (cols - c >= 32) {
            uint32_t r0[16], r1[16];
            tmem_ld16_nowait(dt + cbeg + c, r0);
            tmem_ld16_nowait(dt + cbeg + c + 16, r1);
            tmem_wait_ld();
            float v[32];
#pragma unroll
            for (int i = 0; i < 16; i++) {
              v[i] = __uint_as_float(r0[i]);
              v[16 + i] = __uint_as_float(r1[i]);
            }
            epilogue_warp<32>(e, d.K, d.P, d.Q, v, col, s_sc, s_sh, valid, n, p, q, stage);
            c += 32;
          } else {
            uint32_t r0[16];
            tmem_ld16_nowait(dt + cbeg + c, r0);
            tmem_wait_ld();
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r0[i]);
            epilogue_warp<16>(e, d.K, d.P, d.Q, v, col, s_sc, s_sh, valid, n, p, q, stage);
            c += 16;
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < cols; c += 16) {
          __syncwarp();
          float v[16];
          tmem_ld16(dt + cbeg + c, v);
          const int col0 = n0 + cbeg + c;
          if (!valid || col0 >= d.gemm_n) continue;
#pragma unroll
          for (int h = 0; h < 2; h++) {
            const int col = col0 + h * 8;
            if (col >= d.gemm_n) break;
            const int cnt = d.gemm_n - col < 8 ? d.gemm_n - col : 8;
            float y[8];
#pragma unroll
            for (int i = 0; i < 8; i++) y[i] = v[h * 8 + i];
            epilogue8(e, d.K, d.P, d.Q, y, cnt, col, col, s_sc, s_sh, pix, n, p, q);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce + buf);
    }
  }
  if (warp >= 2 && lane == 0) bulk_wait_group0();  // tensor stores complete before the CTA retires
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

template <int BK, int BN, int MODE>
static cudaError_t launch_one(const ConvLaunch& L, cudaStream_t st, bool prime_only) {
  using Cfg = FpropCfg<BK, BN>;
  // The dynamic shared-memory opt-in is set once per process (one device per process) and, through
  // conv_prime(), before any stream capture.
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(k_conv_fprop<BK, BN, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  if (prime_only) return cudaSuccess;
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int cap = sms * Cfg::CTAS_PER_SM;
  const int grid = L.grid < cap ? L.grid : cap;
  k_conv_fprop<BK, BN, MODE><<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, st>>>(L.ta, L.tb, L.sm, L.d);
  return cudaGetLastError();
}

template <int BK, int BN>
static cudaError_t launch_mode(const ConvLaunch& L, cudaStream_t st, bool prime) {
  switch (L.mode) {
    case A_GEMM: return launch_one<BK, BN, A_GEMM>(L, st, prime);
    case A_S1: return launch_one<BK, BN, A_S1>(L, st, prime);
    case A_S2: return launch_one<BK, BN, A_S2>(L, st, prime);
  }
  return cudaErrorInvalidValue;
}

template <int BK>
static cudaError_t launch_bn(const ConvLaunch& L, cudaStream_t st, bool prime) {
  switch (L.BN) {
    case 16: return launch_mode<BK, 16>(L, st, prime);
    case 32: return launch_mode<BK, 32>(L, st, prime);
    case 64: return launch_mode<BK, 64>(L, st, prime);
    case 128: return launch_mode<BK, 128>(L, st, prime);
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
