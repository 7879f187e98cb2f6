// Stride-1 R×S convolution with halo reuse, on the sm_100a tensor cores.
//
// The implicit GEMM of conv_fprop.cu fetches, per K-step, one 128-pixel A box per tap: a 3×3 conv reads
// every input pixel nine times from L2 and spends most of its time waiting on TMA rows.  Here a tile is
// MT = 128·MH output pixels of one image (th rows × tw columns, tw a multiple of 8) and, per channel chunk
// and per column shift c of the filter, ONE box of (th + R − 1) input rows × tw columns is loaded.  The R
// row taps of that column are the same box read from row offset r·tw — a multiple of 8 rows, so each
// UMMA operand still starts on a swizzle-atom boundary and the shift costs nothing but a descriptor
// offset.  A 3×3 tile thus loads 3·(th + 2)·tw pixel rows instead of 9·MT, and with MH = 2 (BN ≤ 128)
// every weight tile feeds two 128-row MMAs (two TMEM accumulators), halving the weight traffic as well.
//
// One CTA per SM (the accumulators fill TMEM: MH × BN columns, double-buffered), 10 warps:
//   warp 0   TMA producer: an A ring (one box per chunk × column shift) and a B ring (one weight box per
//            tap), each with its own full/empty barriers; it runs ahead across tiles;
//   warp 1   TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16) into one of two
//            accumulator sets, so the next tile's MMAs overlap this tile's epilogue;
//   warps 2–9 epilogue through the TMA-store path of epilogue.cuh: with MH = 2 each warp takes 32 rows of
//            one half; with MH = 1 (BN > 128) the two warps of a lane quadrant split the columns.
// Only calls whose every destination allows the TMA-store epilogue come here (conv_prepare decides).
// No multicast.  Every wait is bounded (sm100.cuh).
#include "epilogue.cuh"

namespace osam {

constexpr int kHaloMaxGemmN = 512;
constexpr int kHaloMaxSA = 4, kHaloMaxSB = 8;

template <int BK, int BN>
struct HaloCfg {
  static constexpr int MH = BN <= 128 ? 2 : 1;  // 128-row MMA halves per tile
  static constexpr int ACC_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr int SET_COLS = MH * ACC_COLS;  // one accumulator set (all halves)
  static constexpr int TMEM_COLS = 2 * SET_COLS;  // double-buffered
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int ROW_BYTES = BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;  // a multiple of 1024 for BN % 32 == 0, BK ∈ {32, 64}
  static constexpr int STAGE_OUT_BYTES = EPI_WARPS * 32 * 64;
  static_assert(TMEM_COLS <= 512, "accumulators exceed TMEM");
  static_assert(B_BYTES % 1024 == 0, "B stages must keep 1024-byte alignment");
};

size_t halo_fixed_smem_bytes() {
  // alignment slack, epilogue stages (8 warps × 2 KiB), epilogue constants, barriers + TMEM slot
  return 1024 + (size_t)8 * 32 * 64 + 2 * kHaloMaxGemmN * 4 + (2 * kHaloMaxSA + 2 * kHaloMaxSB + 4) * 8 + 16;
}

template <int BK, int BN>
__global__ void __launch_bounds__(HaloCfg<BK, BN>::THREADS, 1)
    k_conv_halo(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                const __grid_constant__ StoreMaps sm, const ConvDev d) {
  using Cfg = HaloCfg<BK, BN>;
  constexpr int MH = Cfg::MH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int SA = d.halo_sa, SB = d.halo_sb, A_BYTES = d.halo_a_bytes, A_STRIDE = d.halo_a_stride;
  uint8_t* sA = base;
  uint8_t* sB = sA + SA * A_STRIDE;           // A_STRIDE % 1024 == 0
  uint8_t* s_stage = sB + SB * Cfg::B_BYTES;  // 1024-aligned: the TMA-store swizzle needs 512
  float* s_sc = reinterpret_cast<float*>(s_stage + Cfg::STAGE_OUT_BYTES);
  float* s_sh = s_sc + kHaloMaxGemmN;
  uint64_t* afull = reinterpret_cast<uint64_t*>(s_sh + kHaloMaxGemmN);
  uint64_t* aempty = afull + kHaloMaxSA;
  uint64_t* bfull = aempty + kHaloMaxSA;
  uint64_t* bempty = bfull + kHaloMaxSB;
  uint64_t* accf = bempty + kHaloMaxSB;  // [2] accumulator set ready (MMA → epilogue)
  uint64_t* acce = accf + 2;             // [2] accumulator set drained, one arrival per epilogue warp
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acce + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = d.tiles_m * d.ntn;
  const int R = d.R, S = d.S, tw = d.tw, th = d.th;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SA; s++) {
      mbar_init(afull + s, 1);
      mbar_init(aempty + s, 1);
    }
    for (int s = 0; s < SB; s++) {
      mbar_init(bfull + s, 1);
      mbar_init(bempty + s, 1);
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
      uint32_t ia = 0, ib = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const int nt = t % d.ntn, mt = t / d.ntn, n0 = nt * BN;
        const int tq = mt % d.tiles_q, rest = mt / d.tiles_q;
        const int q0 = tq * tw, p0 = (rest % d.tiles_p) * th, img = rest / d.tiles_p;
        for (int kc = 0; kc < d.nkc && ok; kc++) {
          const int cc = kc * BK;
          for (int c = 0; c < S && ok; c++, ia++) {
            const int sa = ia % SA;
            if (ia >= (uint32_t)SA && !mbar_wait(aempty + sa, ((ia / SA) - 1) & 1, d.err)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(afull + sa, A_BYTES);
            // input rows p0 − pad … p0 − pad + th + R − 2, columns q0 + c − pad … (halo = TMA zero fill)
            tma_load_4d(sA + sa * A_STRIDE, &ta, afull + sa, cc, q0 + c - d.pad, p0 - d.pad, img);
            for (int r = 0; r < R; r++, ib++) {
              const int sb = ib % SB;
              if (ib >= (uint32_t)SB && !mbar_wait(bempty + sb, ((ib / SB) - 1) & 1, d.err)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(bfull + sb, Cfg::B_BYTES);
              tma_load_2d(sB + sb * Cfg::B_BYTES, &tb, bfull + sb, (r * S + c) * d.C + cc, n0);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, BN);
      uint32_t ia = 0, ib = 0, lt = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, lt++) {
        const uint32_t buf = lt & 1;
        if (lt >= 2 && !mbar_wait(acce + buf, ((lt >> 1) - 1) & 1, d.err)) break;
        tc_fence_after();
        const uint32_t dt = tmem + buf * Cfg::SET_COLS;
        bool first = true;
        for (int kc = 0; kc < d.nkc && ok; kc++) {
          for (int c = 0; c < S && ok; c++, ia++) {
            const int sa = ia % SA;
            if (!mbar_wait(afull + sa, (ia / SA) & 1, d.err)) {
              ok = false;
              break;
            }
            const uint32_t a0 = smem_u32(sA + sa * A_STRIDE);
            for (int r = 0; r < R; r++, ib++) {
              const int sb = ib % SB;
              if (!mbar_wait(bfull + sb, (ib / SB) & 1, d.err)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t b0 = smem_u32(sB + sb * Cfg::B_BYTES);
              const uint32_t ar = a0 + (uint32_t)(r * tw) * Cfg::ROW_BYTES;  // row tap r: r·tw rows down
#pragma unroll
              for (int k = 0; k < BK / 16; k++) {
#pragma unroll
                for (int h = 0; h < MH; h++)
                  umma_f16(dt + h * Cfg::ACC_COLS,
                           smem_desc_kmajor(ar + h * 128 * Cfg::ROW_BYTES + k * 32, Cfg::ROW_BYTES),
                           smem_desc_kmajor(b0 + k * 32, Cfg::ROW_BYTES), idesc, first ? 0u : 1u);
                first = false;
              }
              umma_commit(bempty + sb);
            }
            if (ok) umma_commit(aempty + sa);
          }
        }
        if (ok) umma_commit(accf + buf);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..9)
    const EpiDev& e = d.ep;
    const int ew = warp - 2;    // 0..7
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int half = ew >> 2;
    // MH = 2: warp (half, quad) owns tile rows half·128 + quad·32 … (all columns).
    // MH = 1: the two warps of a quadrant split the columns: ceil32(BN/2) and the rest.
    constexpr int SPLIT = ((BN / 2 + 31) / 32) * 32;
    const int cols = MH == 2 ? BN : (half == 0 ? SPLIT : BN - SPLIT);
    const int cbeg = MH == 2 ? 0 : half * SPLIT;
    const int m0 = (MH == 2 ? half * 128 : 0) + quad * 32;  // first tile row of this warp
    const int row = m0 + lane;
    const int i = row / tw, j = row - i * tw;      // this lane's pixel inside the tile
    const int bi = m0 / tw, bj = m0 - bi * tw;     // origin of this warp's 32-row store box
    const uint32_t tcol = (MH == 2 ? half * Cfg::ACC_COLS : 0) + cbeg;
    uint8_t* stage = s_stage + ew * (32 * 64);
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, lt++) {
      const int nt = t % d.ntn, mt = t / d.ntn, n0 = nt * BN;
      const int tq = mt % d.tiles_q, rest = mt / d.tiles_q;
      const int q0 = tq * tw, p0 = (rest % d.tiles_p) * th, img = rest / d.tiles_p;
      const int p = p0 + i, q = q0 + j;
      const bool valid = p < d.P && q < d.Q;
      const uint32_t buf = lt & 1;
      const bool ok = mbar_wait(accf + buf, (lt >> 1) & 1, d.err);
      tc_fence_after();
      if (!ok) break;
      const uint32_t dt = tmem + buf * Cfg::SET_COLS + tcol + ((uint32_t)(quad * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < cols; c += 32) {
        __syncwarp();
        uint32_t r0[16], r1[16];
        tmem_ld16_nowait(dt + c, r0);
        tmem_ld16_nowait(dt + c + 16, r1);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int x = 0; x < 16; x++) {
          v[x] = __uint_as_float(r0[x]);
          v[16 + x] = __uint_as_float(r1[x]);
        }
        epilogue_warp_tma(e, sm, d.K, d.P, d.Q, v, n0 + cbeg + c, s_sc, s_sh, valid, img, p, q, q0 + bj, p0 + bi,
                          img, stage);
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

template <int BK, int BN>
static cudaError_t halo_launch_one(const ConvLaunch& L, cudaStream_t st, bool prime_only) {
  using Cfg = HaloCfg<BK, BN>;
  // The dynamic shared-memory opt-in is set once per process and, through conv_prime(), before any capture.
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(k_conv_halo<BK, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kHaloSmemLimit);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  if (prime_only) return cudaSuccess;
  const ConvDev& d = L.d;
  const size_t smem = (size_t)d.halo_sa * d.halo_a_stride + (size_t)d.halo_sb * Cfg::B_BYTES + halo_fixed_smem_bytes();
  if (smem > kHaloSmemLimit || d.halo_sa < 2 || d.halo_sa > kHaloMaxSA || d.halo_sb < 2 || d.halo_sb > kHaloMaxSB ||
      d.halo_a_stride % 1024 != 0)
    return cudaErrorInvalidValue;
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int grid = L.grid < sms ? L.grid : sms;
  k_conv_halo<BK, BN><<<grid, Cfg::THREADS, smem, st>>>(L.ta, L.tb, L.sm, L.d);
  return cudaGetLastError();
}

template <int BK>
static cudaError_t halo_launch_bn(const ConvLaunch& L, cudaStream_t st, bool prime) {
  switch (L.BN) {
    case 32: return halo_launch_one<BK, 32>(L, st, prime);
    case 64: return halo_launch_one<BK, 64>(L, st, prime);
    case 128: return halo_launch_one<BK, 128>(L, st, prime);
    case 224: return halo_launch_one<BK, 224>(L, st, prime);
    case 256: return halo_launch_one<BK, 256>(L, st, prime);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_conv_halo(const ConvLaunch& L, cudaStream_t st, bool prime_only) {
  if (L.BK == 64) return halo_launch_bn<64>(L, st, prime_only);
  if (L.BK == 32) return halo_launch_bn<32>(L, st, prime_only);
  return cudaErrorInvalidValue;
}

}  // namespace osam
