// Weight gradient of a conv on the sm_100a tensor cores (osam_conv_wgrad, replaces ConvOp::wgrad,
// src/conv.cpp:357-366):  dW[k][r][s][c] = Σ_{n,p,q} dz[n][p][q][k] · x[n][p·st + r − pad][q·st + s − pad][c].
//
// For each tap (r, s) this is a GEMM  D[k][c] = Σ_pixels A[k][pixel] · B[c][pixel]  whose reduction runs
// over the output pixels.  In NHWC both operands already have their M / N index contiguous, which is
// the MN-major operand form of tcgen05: a TMA box of [pixels][64 channels] with the 128-byte swizzle
// (32 channels: 64-byte swizzle) is exactly the MN-major canonical layout — rows of 64 channels, one row
// per reduction index, LBO = distance between 64-channel blocks, SBO = distance between 8-row groups.
// The pixel tiles are the forward conv's spatial tiles (tn images × th × tw = 128 output pixels): the dz
// box is the tile itself, the x box is the same tile shifted by the tap (stride 2: the parity view of the
// forward kernel), and TMA zero fill supplies the padding.
//
// Work split: CTA = (tap, 128-row block of K, BN-column block of C, range of pixel tiles).  Each CTA
// accumulates its range in TMEM (M = 128, N = BN, K = 16 pixels per MMA, 8 MMAs per tile), then adds its
// fp32 block into a zeroed fp32 workspace with vector atomics; a last pass writes dW in fp16 (+ beta·dW).
// Warp 0: TMA producer; warp 1: TMEM owner + MMA issuer; warps 2–5: the final read-out.
// No multicast.  Every wait is bounded (sm100.cuh).
#include "conv_internal.h"
#include "sm100.cuh"

namespace osam {

// MN-major operand descriptor: `row_bytes` = 128 (64 channels, SWIZZLE_128B) or 64 (32, SWIZZLE_64B).
__device__ __forceinline__ uint64_t smem_desc_mnmajor(uint32_t saddr, int row_bytes, uint32_t block_bytes) {
  uint64_t d = (saddr & 0x3FFFFu) >> 4;
  d |= uint64_t((block_bytes >> 4) & 0x3FFFu) << 16;      // LBO: next block of 64 (32) M/N elements
  d |= uint64_t(((8 * row_bytes) >> 4) & 0x3FFFu) << 32;  // SBO: next 8 reduction rows
  d |= uint64_t(1) << 46;
  d |= uint64_t(row_bytes == 128 ? 2 : 4) << 61;
  return d;
}

// Instruction descriptor, kind::f16, fp32 accumulator, both operands MN-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32_mn(int M, int N) {
  return (1u << 4) | (1u << 15) | (1u << 16) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

template <int AB, int BB, int BN>
struct WgCfg {
  static constexpr int MBOX = 128 / AB;       // dz boxes per stage (M = 128 output channels)
  static constexpr int NBOX = BN / BB;        // x boxes per stage
  static constexpr int A_BOX = 128 * AB * 2;  // 128 pixels × AB channels
  static constexpr int B_BOX = 128 * BB * 2;
  static constexpr int STAGE_BYTES = MBOX * A_BOX + NBOX * B_BOX;
  static constexpr int STAGES_RAW = (200 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW < 2 ? 2 : (STAGES_RAW > 6 ? 6 : STAGES_RAW);
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr int THREADS = 64 + 128;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
  static_assert(A_BOX % 1024 == 0 && B_BOX % 1024 == 0, "stage parts must stay 1024-byte aligned");
};

template <int AB, int BB, int BN, int MODE>
__global__ void __launch_bounds__(WgCfg<AB, BB, BN>::THREADS, 1)
    k_conv_wgrad(const __grid_constant__ CUtensorMap tdz, const __grid_constant__ CUtensorMap tx, const ConvDev d,
                 float* __restrict__ acc, int nsplit, int tiles_per_split) {
  using Cfg = WgCfg<AB, BB, BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accf + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int taps = d.R * d.S;
  const int mblocks = (d.K + 127) / 128, nblocks = (d.C + BN - 1) / BN;
  // CTA → (split, tap, m block, n block); neighbouring CTAs share their pixel range (L2 reuse of dz, x)
  int rest = blockIdx.x;
  const int nb = rest % nblocks;
  rest /= nblocks;
  const int mb = rest % mblocks;
  rest /= mblocks;
  const int tap = rest % taps;
  const int split = rest / taps;
  const int t0 = split * tiles_per_split, t1 = min(d.tiles_m, t0 + tiles_per_split);
  const int r = tap / d.S, c = tap - r * d.S;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(accf, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tdz);
    tma_prefetch_desc(&tx);
  }
  if (warp == 1) {
    tmem_alloc(tslot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = t0; t < t1; t++, it++) {
        const int s = it % STAGES;
        if (it >= STAGES && !mbar_wait(empty + s, ((it / STAGES) - 1) & 1, d.err)) break;
        const int tq = t % d.tiles_q, rr = t / d.tiles_q;
        const int q0 = tq * d.tw, p0 = (rr % d.tiles_p) * d.th, b0 = (rr / d.tiles_p) * d.tn;
        mbar_arrive_expect_tx(full + s, Cfg::STAGE_BYTES);
        uint8_t* a = base + s * Cfg::STAGE_BYTES;
        uint8_t* b = a + Cfg::MBOX * Cfg::A_BOX;
#pragma unroll
        for (int j = 0; j < Cfg::MBOX; j++) tma_load_4d(a + j * Cfg::A_BOX, &tdz, full + s, mb * 128 + j * AB, q0, p0, b0);
#pragma unroll
        for (int j = 0; j < Cfg::NBOX; j++) {
          const int cc = nb * BN + j * BB;
          if (MODE == A_S1) {
            tma_load_4d(b + j * Cfg::B_BOX, &tx, full + s, cc, q0 + c - d.pad, p0 + r - d.pad, b0);
          } else {
            const int dr = r - d.pad, dc = c - d.pad;
            tma_load_5d(b + j * Cfg::B_BOX, &tx, full + s, (dc & 1) * d.C + cc, q0 + (dc >> 1), dr & 1,
                        p0 + (dr >> 1), b0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32_mn(128, BN);
      uint32_t it = 0;
      bool ok = true;
      for (int t = t0; t < t1; t++, it++) {
        const int s = it % STAGES;
        if (!mbar_wait(full + s, (it / STAGES) & 1, d.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a = smem_u32(base + s * Cfg::STAGE_BYTES), b = a + Cfg::MBOX * Cfg::A_BOX;
#pragma unroll
        for (int k = 0; k < 8; k++)  // 16 pixels (reduction rows) per MMA
          umma_f16(tmem, smem_desc_mnmajor(a + k * 16 * AB * 2, AB * 2, Cfg::A_BOX),
                   smem_desc_mnmajor(b + k * 16 * BB * 2, BB * 2, Cfg::B_BOX), idesc, (it | k) != 0);
        umma_commit(empty + s);
      }
      if (ok && t1 > t0) umma_commit(accf);
    }
  } else {
    // ---------------------------------------------------------------- read-out: fp32 block → atomics
    const int quad = warp & 3;
    const int k = mb * 128 + quad * 32 + lane;  // this lane's output channel
    const bool ok = t1 > t0 && mbar_wait(accf, 0, d.err);
    tc_fence_after();
    if (ok) {
      const uint32_t dt = tmem + ((uint32_t)(quad * 32) << 16);
      float* row = acc + (((long long)k * d.R + r) * d.S + c) * d.C + nb * BN;
#pragma unroll 1
      for (int j = 0; j < BN; j += 16) {
        __syncwarp();
        float v[16];
        tmem_ld16(dt + j, v);
        if (k < d.K) {
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            if (nb * BN + j + i + 4 <= d.C)
              atomicAdd(reinterpret_cast<float4*>(row + j + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------------------
// Small-C input conv (R·S·C ≤ 32: the RGB stem, 3×3×3).  Replaces the reference's wgrad_rgb_s2
// (src/misc.cu:193-273, a WMMA kernel because cuDNN cannot use tensor cores at C = 3).
//   D[j][k] = Σ_pixels patch[pixel][j] · dz[pixel][k],   j = (r·S + s)·C + c,   dW[k][r][s][c] = D[j][k]
// A = the im2col patch tile (M = patch column j, reduction = 128 output pixels), written by the producer
// warps straight into the MN-major 64-byte-swizzled layout (a row of 32 patch columns per pixel); B = the
// dz tile, 128 consecutive output pixels × K channels, one contiguous TMA box (MN-major: channels
// contiguous).  M = 128 of which only the R·S·C ≤ 32 rows the patch fills are read back: the descriptor's
// other three 32-row blocks point into the following shared memory and their products are discarded.
// Warps 0–7: two groups of patch producers taking alternate tiles (one output pixel per thread); warp 8:
// dz TMA; warp 9: TMEM owner + MMA issuer.  Warp 0 reads the 32×K fp32 block out and adds it into the
// zeroed workspace.  HBM traffic: dz once, x ≈ (st·(Q−1)+S)/(st·Q)·(R/st) times (L1/L2 serve the overlap).
template <int K>
struct StemWgCfg {
  static constexpr int A_BYTES = 128 * 64;     // 128 pixels × 32 patch columns (fp16)
  static constexpr int B_BYTES = 128 * K * 2;  // 128 pixels × K dz channels
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = 4;
  static constexpr int SLACK = 3 * A_BYTES;    // the three discarded M blocks of the last stage's A
  static constexpr int THREADS = 320;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE + SLACK + 256;
  static_assert(STAGES % 2 == 0, "the two producer groups own alternate stages");
};

template <int K>
__global__ void __launch_bounds__(StemWgCfg<K>::THREADS, 1)
    k_conv_wgrad_stem(const __grid_constant__ CUtensorMap tdz, const __half* __restrict__ x, const ConvDev d,
                      float* __restrict__ acc, int tiles_per_cta) {
  using Cfg = StemWgCfg<K>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_joff[32], s_jr[32], s_js[32];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + STAGES * Cfg::STAGE + Cfg::SLACK);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accf + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int RSC = d.R * d.S * d.C;
  const long long tiles = (d.M + 127) / 128;
  const long long t0 = (long long)blockIdx.x * tiles_per_cta;
  const long long t1 = t0 + tiles_per_cta < tiles ? t0 + tiles_per_cta : tiles;
  const int n_it = t1 > t0 ? int(t1 - t0) : 0;

  if (threadIdx.x < 32) {
    const int j = threadIdx.x;
    if (j < RSC) {
      const int rr = j / (d.S * d.C), ss = (j / d.C) % d.S, cc = j % d.C;
      s_joff[j] = (rr * d.W + ss) * d.C + cc;
      s_jr[j] = rr;
      s_js[j] = ss;
    } else {
      s_joff[j] = 0;
      s_jr[j] = -1;  // zero column
      s_js[j] = 0;
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full + s, 128 + 1);  // the producer group's 128 threads + the dz TMA's expect_tx arrival
      mbar_init(empty + s, 1);
    }
    mbar_init(accf, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tdz);
  }
  if (warp == 9) {
    tmem_alloc(tslot, K);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp < 8) {
    // ---------------------------------------------------------------- patch producers
    const int grp = warp >> 2, row = threadIdx.x & 127;
    const int PQ = d.P * d.Q;
    for (int it = grp; it < n_it; it += 2) {
      const int s = it % STAGES;
      if (it >= STAGES && !mbar_wait(empty + s, ((it / STAGES) - 1) & 1, d.err)) break;
      const long long pix = (t0 + it) * 128 + row;
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; i++) pk[i] = 0u;
      if (pix < d.M) {
        const int n = int(pix / PQ), rem = int(pix - (long long)n * PQ), p = rem / d.Q, q = rem - p * d.Q;
        const int y0 = p * d.stride - d.pad, x0 = q * d.stride - d.pad;
        const long long b0 = ((long long)(n * d.H + y0) * d.W + x0) * d.C;  // index of patch (0, 0, 0); may be < 0
        const unsigned short* xs = reinterpret_cast<const unsigned short*>(x);
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const int jr = s_jr[j], js = s_js[j];
          unsigned v = 0u;
          if (jr >= 0 && (unsigned)(y0 + jr) < (unsigned)d.H && (unsigned)(x0 + js) < (unsigned)d.W)
            v = __ldg(xs + b0 + s_joff[j]);
          pk[j >> 1] |= v << ((j & 1) * 16);
        }
      }
      uint8_t* a = base + s * Cfg::STAGE + row * 64;
      const int sw = (row >> 1) & 3;
#pragma unroll
      for (int c = 0; c < 4; c++)
        *reinterpret_cast<uint4*>(a + ((c ^ sw) << 4)) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_proxy_async_smem();
      mbar_arrive(full + s);
    }
    if (warp == 0) {
      // ---------------------------------------------------------------- read-out: lane j = patch column j
      const bool ok = n_it > 0 && mbar_wait(accf, 0, d.err);
      tc_fence_after();
      if (ok) {
#pragma unroll 1
        for (int k0 = 0; k0 < K; k0 += 16) {
          __syncwarp();
          float v[16];
          tmem_ld16(tmem + k0, v);
          if (lane < RSC) {
#pragma unroll
            for (int i = 0; i < 16; i++) atomicAdd(acc + (long long)(k0 + i) * RSC + lane, v[i]);
          }
        }
      }
    }
  } else if (warp == 8) {
    // ---------------------------------------------------------------- dz TMA
    if (lane == 0) {
      for (int it = 0; it < n_it; it++) {
        const int s = it % STAGES;
        if (it >= STAGES && !mbar_wait(empty + s, ((it / STAGES) - 1) & 1, d.err)) break;
        mbar_arrive_expect_tx(full + s, Cfg::B_BYTES);
        tma_load_2d(base + s * Cfg::STAGE + Cfg::A_BYTES, &tdz, full + s, 0, int((t0 + it) * 128));
      }
    }
  } else {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32_mn(128, K);
      bool ok = true;
      for (int it = 0; it < n_it; it++) {
        const int s = it % STAGES;
        if (!mbar_wait(full + s, (it / STAGES) & 1, d.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a = smem_u32(base + s * Cfg::STAGE), b = a + Cfg::A_BYTES;
#pragma unroll
        for (int k = 0; k < 8; k++)  // 16 pixels per MMA
          umma_f16(tmem, smem_desc_mnmajor(a + k * 16 * 64, 64, Cfg::A_BYTES),
                   smem_desc_mnmajor(b + k * 16 * K * 2, K * 2, Cfg::B_BYTES), idesc, (it | k) != 0);
        umma_commit(empty + s);
      }
      if (ok && n_it > 0) umma_commit(accf);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, K);
  }
}

// ------------------------------------------------------------------------------------------------------
// Window form for 3×3 / pad-1 convs with 32 or 64 input channels (the narrow C2f bottlenecks, the narrow
// head branches and the first stride-2 convs).  Per-tap CTAs reload a tile's dz and its shifted x box
// nine times and, with K = 32 output channels, fill a quarter of the M = 128 accumulator.  Here the nine
// taps of a 128-pixel tile come from a few boxes, both GEMM operands MN-major:
//  * row taps stacked in M: the x window (the tile's rows plus the row halo, 64-byte rows of 32 channels)
//    has its pixel rows in the tile's (row, image, column) order, so row tap r starts r·ni·tw rows further
//    on — a constant distance, which is the descriptor's M-block stride: the four 32-row M blocks of one
//    M = 128 MMA are the row taps 0, 1, 2 and a discarded block;
//  * column taps stacked in N: with the reduction re-indexed by the column shift (pixel q' = q + s − 1),
//    tap s pairs the UNSHIFTED x window with dz shifted by 1 − s columns,
//      dW[k][r][s][c] = Σ_{n,p,q'} x[n][p + r − 1][q'][c] · dz[n][p][q' + 1 − s][k],
//    every (q, s) term counted once over the tiles of q', with the TMA zero fill outside dz; the three
//    shifted dz boxes sit one box apart, the descriptor's N-block stride, so one MMA has N = 3·NB.
// Stride 2 (parity view of x: the two row parities of a row pair side by side, output row i of row tap r
// at window row 16·i + 8·(r + 1)): column tap 1 reads the even columns (window of parity 0, dz unshifted);
// taps 2 and 0 read the odd columns (window of parity 1) with dz unshifted and shifted by one column,
// so per 32-channel block one MMA of N = NB and one of N = 2·NB.
// One CTA takes a run of tiles and accumulates in TMEM (3·NB columns per channel block) for the whole run;
// at the end the warps on TMEM quadrants 0–2 (= row taps) add the accumulators into the fp32 KRSC
// workspace with coalesced atomics (lane = input channel).  Rings: dz stages and x window slots, each
// released by its own MMA commit.  Warp 0: TMA producer; warp 1: TMEM owner + MMA issuer.  No multicast;
// every wait is bounded.
__device__ __forceinline__ uint64_t smem_desc_mn_sw64(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (saddr & 0x3FFFFu) >> 4;
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;  // LBO: next 32-element M block (here: the next row tap)
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;  // SBO: next 8 reduction rows
  d |= uint64_t(1) << 46;
  d |= uint64_t(4) << 61;                     // 64-byte swizzle
  return d;
}

template <int CB, int NB, bool S2>
struct WgWinCfg {
  static constexpr int DZ_ROWB = NB * 2;             // one dz box per column shift: 64- or 128-byte rows
  static constexpr int DZ_BOX = 128 * DZ_ROWB;
  static constexpr int NDZ = S2 ? 2 : 3;             // dz boxes per tile (column shifts)
  static constexpr int DZ_BYTES = NDZ * DZ_BOX;
  static constexpr int DSTAGES = DZ_BYTES <= 32 * 1024 ? 4 : 2;
  static constexpr int NWIN = CB * (S2 ? 2 : 1);     // x windows per tile
  // window rows read, the discarded fourth M block included: stride 1 128 + 3·ni·tw (ni·tw ≤ 16);
  // stride 2 32·7 + 24 + 3·8 + 8 = 280
  static constexpr int WIN_ROWS = S2 ? 280 : 128 + 3 * 16;
  static constexpr int WIN_BYTES = (WIN_ROWS * 64 + 1023) & ~1023;
  static constexpr int WST_RAW = (210 * 1024 - DSTAGES * DZ_BYTES) / WIN_BYTES;
  static constexpr int WSTAGES = WST_RAW > 4 * NWIN ? 4 * NWIN : WST_RAW;
  static constexpr int ACC_COLS = 3 * CB * NB;
  static constexpr int TMEM_COLS = ACC_COLS <= 32 ? 32 : ACC_COLS <= 64 ? 64 : ACC_COLS <= 128 ? 128
                                 : ACC_COLS <= 256 ? 256 : 512;
  static constexpr int THREADS = 192;
  static constexpr int BAR_BYTES = ((2 * DSTAGES + 2 * WSTAGES + 1) * 8 + 4 + 15) & ~15;  // barriers + TMEM slot
  static constexpr int SMEM_BYTES = 1024 + DSTAGES * DZ_BYTES + WSTAGES * WIN_BYTES + BAR_BYTES;
  static_assert(NB == 32 || NB == 64, "dz block: one 32- or 64-channel box per column shift");
  static_assert(ACC_COLS <= 512, "accumulators must fit in TMEM");
  static_assert(WSTAGES >= 2, "window ring too small");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
  static_assert((228 * 1024 / (SMEM_BYTES + 1024)) * TMEM_COLS <= 512, "co-resident CTAs must fit in TMEM");
};

template <int CB, int NB, bool S2>
__global__ void __launch_bounds__(192, 1)
    k_conv_wgrad_win(const __grid_constant__ CUtensorMap tdz, const __grid_constant__ CUtensorMap tx, const ConvDev d,
                     float* __restrict__ acc, int nblk, int tiles_per_split, int win_bytes) {
  using Cfg = WgWinCfg<CB, NB, S2>;
  constexpr int DST = Cfg::DSTAGES, WST = Cfg::WSTAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* dzb = base;
  uint8_t* wnb = base + DST * Cfg::DZ_BYTES;
  uint64_t* dfull = reinterpret_cast<uint64_t*>(wnb + WST * Cfg::WIN_BYTES);
  uint64_t* dempty = dfull + DST;
  uint64_t* wfull = dempty + DST;
  uint64_t* wempty = wfull + WST;
  uint64_t* accf = wempty + WST;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accf + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = blockIdx.x % nblk, split = blockIdx.x / nblk;
  const int t0 = split * tiles_per_split, t1 = min(d.tiles_m, t0 + tiles_per_split);

  if (threadIdx.x == 0) {
    for (int s = 0; s < DST; s++) {
      mbar_init(dfull + s, 1);
      mbar_init(dempty + s, 1);
    }
    for (int s = 0; s < WST; s++) {
      mbar_init(wfull + s, 1);
      mbar_init(wempty + s, 1);
    }
    mbar_init(accf, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tdz);
    tma_prefetch_desc(&tx);
  }
  if (warp == 1) {
    tmem_alloc(tslot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t wit = 0;
      bool ok = true;
      for (int t = t0, it = 0; t < t1 && ok; t++, it++) {
        const int tq = t % d.tiles_q, rest = t / d.tiles_q;
        const int tp = rest % d.tiles_p, tn = rest / d.tiles_p;
        const int q0 = tq * d.tw, p0 = tp * d.th, n0 = tn * d.tn;
        const int ds = it % DST;
        if (it >= DST && !mbar_wait(dempty + ds, ((it / DST) - 1) & 1, d.err)) break;
        mbar_arrive_expect_tx(dfull + ds, Cfg::DZ_BYTES);
        // dz boxes: stride 1 shifted by 1 − s for s = 0, 1, 2; stride 2 unshifted and shifted by one column
#pragma unroll
        for (int j = 0; j < Cfg::NDZ; j++)
          tma_load_4d(dzb + ds * Cfg::DZ_BYTES + j * Cfg::DZ_BOX, &tdz, dfull + ds, nb * NB, S2 ? q0 + j : q0 + 1 - j,
                      n0, p0);
        for (int w = 0; w < Cfg::NWIN; w++, wit++) {
          const int ws = wit % WST;
          if (wit >= WST && !mbar_wait(wempty + ws, ((wit / WST) - 1) & 1, d.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(wfull + ws, win_bytes);
          uint8_t* dst = wnb + ws * Cfg::WIN_BYTES;
          if (!S2) {
            tma_load_4d(dst, &tx, wfull + ws, w * 32, q0, n0, p0 - 1);
          } else {  // w = 2·cb + column parity
            tma_load_5d(dst, &tx, wfull + ws, (w & 1) * d.C + (w >> 1) * 32, q0, 0, p0 - 1, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t a_lbo = S2 ? 8 * 64 : (uint32_t)(d.tn * d.tw * 64);  // row-tap distance in the window
      const uint32_t a_sbo = S2 ? 16 * 64 : 8 * 64;                        // next 8 tile pixels
      uint32_t wit = 0;
      bool ok = true;
      for (int t = t0, it = 0; t < t1 && ok; t++, it++) {
        const int ds = it % DST;
        if (!mbar_wait(dfull + ds, (it / DST) & 1, d.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t bz = smem_u32(dzb + ds * Cfg::DZ_BYTES);
        for (int w = 0; w < Cfg::NWIN; w++, wit++) {
          const int ws = wit % WST;
          if (!mbar_wait(wfull + ws, (wit / WST) & 1, d.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(wnb + ws * Cfg::WIN_BYTES);
          // accumulator slots per channel block: stride 1 (s = 0, 1, 2); stride 2 (s = 1 | s = 2, s = 0)
          const int cb = S2 ? (w >> 1) : w;
          const int slot = S2 ? (w & 1) : 0;
          const uint32_t dcol = tmem + (uint32_t)((cb * 3 + slot) * NB);
          const uint32_t idesc = S2 ? ((w & 1) ? idesc_f16_f32_mn(128, 2 * NB) : idesc_f16_f32_mn(128, NB))
                                    : idesc_f16_f32_mn(128, 3 * NB);
#pragma unroll
          for (int kk = 0; kk < 8; kk++) {  // 16 tile pixels (reduction rows) per MMA
            const uint32_t arow = S2 ? (uint32_t)(32 * kk + 8) : (uint32_t)(16 * kk);
            umma_f16(dcol, smem_desc_mn_sw64(a + arow * 64, a_lbo, a_sbo),
                     smem_desc_mnmajor(bz + kk * 16 * Cfg::DZ_ROWB, Cfg::DZ_ROWB, Cfg::DZ_BOX), idesc,
                     (it | kk) != 0);
          }
          umma_commit(wempty + ws);
        }
        if (ok) umma_commit(dempty + ds);
      }
      if (ok && t1 > t0) umma_commit(accf);
    }
  } else {
    // ---------------------------------------------------------------- read-out: quadrant = row tap
    const int r = warp & 3;  // warps 2–5 → TMEM lane quadrants 2, 3, 0, 1; quadrant 3 (warp 3) is discarded
    const bool ok = t1 > t0 && mbar_wait(accf, 0, d.err);
    tc_fence_after();
    if (ok && r < 3) {
      const uint32_t lrow = tmem + ((uint32_t)(r * 32) << 16);
      const long long kstride = 9LL * d.C;
#pragma unroll 1
      for (int cb = 0; cb < CB; cb++)
#pragma unroll 1
        for (int slot = 0; slot < 3; slot++) {
          const int s = S2 ? (slot + 1) % 3 : slot;
          float* dst = acc + ((long long)nb * NB * 9 + r * 3 + s) * d.C + cb * 32 + lane;
#pragma unroll 1
          for (int n0 = 0; n0 < NB; n0 += 16) {
            __syncwarp();
            float v[16];
            tmem_ld16(lrow + (uint32_t)((cb * 3 + slot) * NB + n0), v);
#pragma unroll
            for (int i = 0; i < 16; i++) atomicAdd(dst + (n0 + i) * kstride, v[i]);
          }
        }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// dw (fp16) = acc (fp32) + beta · dw, or dw32 (fp32) = acc + beta · dw32
__global__ void k_wgrad_finish(const float* __restrict__ acc, __half* __restrict__ dw, float* __restrict__ dw32,
                               long long n, float beta) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    float v = acc[i];
    if (dw32) {
      dw32[i] = beta != 0.f ? v + beta * dw32[i] : v;
    } else {
      if (beta != 0.f) v += beta * __half2float(dw[i]);
      dw[i] = __float2half_rn(v);
    }
  }
}

template <int AB, int BB, int BN, int MODE>
static cudaError_t wgrad_launch_one(const WgradLaunch& L, cudaStream_t st) {
  using Cfg = WgCfg<AB, BB, BN>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_conv_wgrad<AB, BB, BN, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  k_conv_wgrad<AB, BB, BN, MODE><<<L.grid, Cfg::THREADS, Cfg::SMEM_BYTES, st>>>(L.tdz, L.tx, L.d, L.acc, L.nsplit,
                                                                              L.tiles_per_split);
  return cudaGetLastError();
}

template <int AB, int BB, int BN>
static cudaError_t wgrad_launch_mode(const WgradLaunch& L, cudaStream_t st) {
  if (L.mode == A_S1) return wgrad_launch_one<AB, BB, BN, A_S1>(L, st);
  if (L.mode == A_S2) return wgrad_launch_one<AB, BB, BN, A_S2>(L, st);
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------------------------------------------
// 1×1 convs with one output channel (the class heads, 128 → 1): both gradients are outer products / channel
// sums, HBM-bound, with no GEMM to give the tensor cores.
//   dgrad: dx[pixel][c] = dy[pixel]·w[c] (+ beta·dx)      wgrad: dw[c] = Σ_pixel dy[pixel]·x[pixel][c]
__global__ void __launch_bounds__(256) k_dgrad_k1(const __half* __restrict__ dy, const __half* __restrict__ w,
                                                  __half* __restrict__ dx, long long npix, int C, float beta) {
  const int V = C / 8;
  const long long n = npix * V;
  for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += (long long)gridDim.x * 256) {
    const long long pix = i / V;
    const int c = int(i - pix * V) * 8;
    const float g = __half2float(dy[pix]);
    float wv[8], o[8];
    ld8h(w + c, wv);
    if (beta != 0.f) ld8h(dx + pix * C + c, o);
#pragma unroll
    for (int k = 0; k < 8; k++) o[k] = beta != 0.f ? fmaf(g, wv[k], beta * o[k]) : g * wv[k];
    st8h(dx + pix * C + c, o);
  }
}
__global__ void __launch_bounds__(256) k_wgrad_k1(const __half* __restrict__ x, const __half* __restrict__ dy,
                                                  float* __restrict__ acc, long long npix, int C, long long rows) {
  extern __shared__ float k1_red[];  // [256 / V][C]
  const int V = C / 8, RL = 256 / V;
  const int rl = threadIdx.x / V, c = (threadIdx.x - rl * V) * 8;
  const long long r0 = blockIdx.x * rows, r1 = r0 + rows < npix ? r0 + rows : npix;
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (rl < RL) {
    for (long long r = r0 + rl; r < r1; r += RL) {
      float xv[8];
      ld8h(x + r * C + c, xv);
      const float g = __half2float(dy[r]);
#pragma unroll
      for (int k = 0; k < 8; k++) a[k] = fmaf(g, xv[k], a[k]);
    }
#pragma unroll
    for (int k = 0; k < 8; k++) k1_red[rl * C + c + k] = a[k];
  }
  __syncthreads();
  for (int ch = threadIdx.x; ch < C; ch += 256) {
    float t = 0.f;
    for (int q = 0; q < RL; q++) t += k1_red[q * C + ch];
    atomicAdd(acc + ch, t);
  }
}

template <int K>
static cudaError_t wgrad_stem_launch(const WgradLaunch& L, cudaStream_t st) {
  using Cfg = StemWgCfg<K>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_conv_wgrad_stem<K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  k_conv_wgrad_stem<K><<<L.grid, Cfg::THREADS, Cfg::SMEM_BYTES, st>>>(L.tdz, L.xp, L.d, L.acc, L.tiles_per_split);
  return cudaGetLastError();
}

template <int CB, int NB, bool S2>
static cudaError_t wgrad_win_launch(const WgradLaunch& L, cudaStream_t st) {
  using Cfg = WgWinCfg<CB, NB, S2>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_conv_wgrad_win<CB, NB, S2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  k_conv_wgrad_win<CB, NB, S2><<<L.grid, Cfg::THREADS, Cfg::SMEM_BYTES, st>>>(L.tdz, L.tx, L.d, L.acc, L.nsplit ? L.grid / L.nsplit : 1,
                                                                             L.tiles_per_split, L.win_bytes);
  return cudaGetLastError();
}

template <bool S2>
static cudaError_t wgrad_win_dispatch(const WgradLaunch& L, cudaStream_t st) {
  if (L.CB == 1) {
    if (L.NB == 32) return wgrad_win_launch<1, 32, S2>(L, st);
    if (L.NB == 64) return wgrad_win_launch<1, 64, S2>(L, st);
  } else if (L.CB == 2) {
    if (L.NB == 32) return wgrad_win_launch<2, 32, S2>(L, st);
    if (L.NB == 64) return wgrad_win_launch<2, 64, S2>(L, st);
  }
  return cudaErrorInvalidValue;
}

bool wgrad_win_supported(int CB, int NB) { return (CB == 1 || CB == 2) && (NB == 32 || NB == 64); }

cudaError_t launch_conv_wgrad(const WgradLaunch& L, cudaStream_t st) {
  cudaError_t e = L.direct ? cudaSuccess : cudaMemsetAsync(L.acc, 0, (size_t)L.n_out * 4, st);
  if (e != cudaSuccess) return e;
  const int AB = L.AB, BB = L.BB, BN = L.BN;
  if (L.win) {
    e = L.mode == A_S2 ? wgrad_win_dispatch<true>(L, st) : wgrad_win_dispatch<false>(L, st);
  } else if (L.mode == A_STEM) {
    if (L.d.K == 32) e = wgrad_stem_launch<32>(L, st);
    else if (L.d.K == 64) e = wgrad_stem_launch<64>(L, st);
    else return cudaErrorInvalidValue;
  } else if (AB == 64 && BB == 64) {
    switch (BN) {
      case 64: e = wgrad_launch_mode<64, 64, 64>(L, st); break;
      case 128: e = wgrad_launch_mode<64, 64, 128>(L, st); break;
      case 256: e = wgrad_launch_mode<64, 64, 256>(L, st); break;
      default: return cudaErrorInvalidValue;
    }
  } else if (AB == 64 && BB == 32 && BN == 32) {
    e = wgrad_launch_mode<64, 32, 32>(L, st);
  } else if (AB == 32 && BB == 64) {
    switch (BN) {
      case 64: e = wgrad_launch_mode<32, 64, 64>(L, st); break;
      case 128: e = wgrad_launch_mode<32, 64, 128>(L, st); break;
      case 256: e = wgrad_launch_mode<32, 64, 256>(L, st); break;
      default: return cudaErrorInvalidValue;
    }
  } else if (AB == 32 && BB == 32 && BN == 32) {
    e = wgrad_launch_mode<32, 32, 32>(L, st);
  } else {
    return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess || L.direct) return e;
  int grid = (int)((L.n_out + 255) / 256);
  if (grid > 4096) grid = 4096;
  k_wgrad_finish<<<grid, 256, 0, st>>>(L.acc, L.dw, L.dw32, L.n_out, L.beta);
  return cudaGetLastError();
}

}  // namespace osam

namespace osam {

cudaError_t launch_dgrad_k1(const __half* dy, const __half* w, __half* dx, long long npix, int C, float beta,
                            cudaStream_t st) {
  const long long n = npix * (C / 8);
  long long grid = (n + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  k_dgrad_k1<<<(unsigned)grid, 256, 0, st>>>(dy, w, dx, npix, C, beta);
  return cudaGetLastError();
}

cudaError_t launch_wgrad_k1(const __half* x, const __half* dy, float* acc, __half* dw, float* dw32, long long npix,
                            int C, float beta, bool direct, cudaStream_t st) {
  if (direct) acc = dw32;
  cudaError_t e = direct ? cudaSuccess : cudaMemsetAsync(acc, 0, (size_t)C * sizeof(float), st);
  if (e != cudaSuccess) return e;
  const int RL = 256 / (C / 8);
  long long rows = (npix + 148 * 4 - 1) / (148 * 4);
  if (rows < 4LL * RL) rows = 4LL * RL;
  const long long grid = (npix + rows - 1) / rows;
  k_wgrad_k1<<<(unsigned)grid, 256, (size_t)RL * C * sizeof(float), st>>>(x, dy, acc, npix, C, rows);
  if ((e = cudaGetLastError()) != cudaSuccess || direct) return e;
  k_wgrad_finish<<<(C + 255) / 256, 256, 0, st>>>(acc, dw, dw32, C, beta);
  return cudaGetLastError();
}

}  // namespace osam
