// Convolution with a tiny reduction (R·S·C ≤ 32, e.g. the 3×3/s2 RGB stem, C = 3) on the tensor cores.
//
// The reference runs this layer through cuDNN, which cannot use tensor cores at C = 3 (its own note,
// src/misc.cu:194-196, measures 4.7 TFLOP/s for the wgrad of this layer).  Here a CTA owns a th × tw
// block of output pixels of one image (128 pixels):
//   1. the block's input window ((th-1)·s+R rows × (tw-1)·s+S columns × C) is read with coalesced
//      loads into shared memory (zero outside the image = the conv padding);
//   2. each thread builds its pixel's im2col row (R·S·C taps zero-padded to 32 fp16 = one 64-byte row)
//      from shared memory, straight into the 64-byte-swizzled K-major layout the UMMA reads;
//   3. one elected thread issues two M=128 × N=BN × K=16 tcgen05 MMAs into TMEM;
//   4. the four warps run the fused epilogue and store whole pixel rows through a per-warp stage.
// The layer is HBM-bound (6 B in, 64 B out per output pixel); eight CTAs per SM overlap one CTA's loads
// with another's epilogue.
#include "epilogue.cuh"

namespace osam {

constexpr int kStemStage = 4 * 32 * 64;  // epilogue stage, 4 warps

// FR/FS/FC/FSTR > 0: geometry fixed at compile time (the 3×3/s2/C=3 stem) so the im2col row stays in
// registers; 0 = runtime geometry.
template <int BN, int FR, int FS, int FC, int FSTR>
__global__ void __launch_bounds__(128) k_conv_stem(const __half* __restrict__ x, const __half* __restrict__ w,
                                                   const ConvDev d) {
  const int R = FR ? FR : d.R, S = FS ? FS : d.S, C = FC ? FC : d.C, STR = FSTR ? FSTR : d.stride;
  constexpr int TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : 128;
  __shared__ __align__(1024) uint8_t sA[128 * 64];
  __shared__ __align__(1024) uint8_t sB[BN * 64];
  __shared__ __align__(16) uint8_t s_stage[kStemStage];
  __shared__ uint64_t bar;
  __shared__ uint32_t tslot;
  __shared__ __align__(16) float s_sc[BN];
  __shared__ __align__(16) float s_sh[BN];
  extern __shared__ __half win[];  // input window, rows × cols × C
  const int tid = threadIdx.x, warp = tid >> 5;
  const int RSC = R * S * C;
  const int WR = (d.th - 1) * STR + R, WC = (d.tw - 1) * STR + S, WCC = WC * C;

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
  load_epilogue_consts(d.ep, d.gemm_n, 0, BN, tid, 128, s_sc, s_sh);
  fence_proxy_async_smem();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  constexpr uint32_t idesc = idesc_f16_f32(128, BN);
  const int ntiles = d.tiles_m;
  uint8_t* stage = s_stage + warp * (32 * 64);
  uint32_t phase = 0;

  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int tq = tile % d.tiles_q, rest = tile / d.tiles_q;
    const int tp = rest % d.tiles_p, n = rest / d.tiles_p;
    const int q0 = tq * d.tw, p0 = tp * d.th;
    const int ih0 = p0 * STR - d.pad, iw0 = q0 * STR - d.pad;
    // 1. input window (coalesced along each row: consecutive threads → consecutive halves)
    const __half* img = x + (long long)n * d.H * d.W * C;
    for (int r = 0; r < WR; r++) {
      const int ih = ih0 + r;
      const bool row_in = ih >= 0 && ih < d.H;
      const __half* src = img + ((long long)ih * d.W + iw0) * C;
      for (int e = tid; e < WCC; e += 128) {
        const int iw = iw0 + e / C;
        __half v = __float2half(0.f);
        if (row_in && iw >= 0 && iw < d.W) v = src[e];
        win[r * WCC + e] = v;
      }
    }
    __syncthreads();
    // 2. this thread's im2col row
    const int i = tid / d.tw, j = tid - (tid / d.tw) * d.tw;
    const int p = p0 + i, q = q0 + j;
    const bool valid = p < d.P && q < d.Q;
    __align__(16) __half row[32];
#pragma unroll
    for (int k = 0; k < 32; k++) row[k] = __float2half(0.f);
    if (FR) {
#pragma unroll
      for (int r = 0; r < FR; r++)
#pragma unroll
        for (int s = 0; s < FS; s++)
#pragma unroll
          for (int c = 0; c < FC; c++) row[(r * FS + s) * FC + c] = win[((i * STR + r) * WC + (j * STR + s)) * FC + c];
    } else {
      for (int r = 0; r < R; r++)
        for (int s = 0; s < S; s++) {
          const __half* src = win + ((i * STR + r) * WC + (j * STR + s)) * C;
          const int k0 = (r * S + s) * C;
          for (int c = 0; c < C; c++) row[k0 + c] = src[c];
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
    // 3. MMA
    if (tid == 0) {
      const uint32_t a = smem_u32(sA), b = smem_u32(sB);
      umma_f16(tmem, smem_desc_kmajor(a, 64), smem_desc_kmajor(b, 64), idesc, 0);
      umma_f16(tmem, smem_desc_kmajor(a + 32, 64), smem_desc_kmajor(b + 32, 64), idesc, 1);
      umma_commit(&bar);
    }
    const bool ok = mbar_wait(&bar, phase, d.err);
    phase ^= 1;
    if (!__syncthreads_and(ok)) break;
    tc_fence_after();
    // 4. epilogue
    const uint32_t dt = tmem + ((uint32_t)(warp * 32) << 16);
    if (d.ep.coop) {
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        __syncwarp();
        uint32_t r0[16];
        tmem_ld16_nowait(dt + c, r0);
        tmem_wait_ld();
        float v[16];
#pragma unroll
        for (int t = 0; t < 16; t++) v[t] = __uint_as_float(r0[t]);
        epilogue_warp<16>(d.ep, d.K, d.P, d.Q, v, c, s_sc, s_sh, valid, n, p, q, stage);
      }
    } else {
      const long long pix = ((long long)n * d.P + p) * d.Q + q;
#pragma unroll 1
      for (int jc = 0; jc < BN / 16; jc++) {
        __syncwarp();
        float v[16];
        tmem_ld16(dt + jc * 16, v);
        if (!valid) continue;
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int col = jc * 16 + h * 8;
          if (col >= d.gemm_n) break;
          const int cnt = d.gemm_n - col < 8 ? d.gemm_n - col : 8;
          float y[8];
#pragma unroll
          for (int t = 0; t < 8; t++) y[t] = v[h * 8 + t];
          epilogue8(d.ep, d.K, d.P, d.Q, y, cnt, col, col, s_sc, s_sh, pix, n, p, q);
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // TMEM and the window are reused by the next tile
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

size_t stem_window_bytes(const ConvDev& d) {
  const int WR = (d.th - 1) * d.stride + d.R, WC = (d.tw - 1) * d.stride + d.S;
  return (size_t)WR * WC * d.C * sizeof(__half);
}

cudaError_t launch_conv_stem(const __half* x, const __half* w, const ConvDev& d, int BN, cudaStream_t st) {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const long long cap = (long long)sms * 8;
  const int grid = (int)(d.tiles_m < cap ? d.tiles_m : cap);
  const size_t smem = stem_window_bytes(d);
  const bool rgb = d.R == 3 && d.S == 3 && d.C == 3 && d.stride == 2;
  if (rgb && BN == 32) {
    k_conv_stem<32, 3, 3, 3, 2><<<grid, 128, smem, st>>>(x, w, d);
    return cudaGetLastError();
  }
  switch (BN) {
    case 16: k_conv_stem<16, 0, 0, 0, 0><<<grid, 128, smem, st>>>(x, w, d); break;
    case 32: k_conv_stem<32, 0, 0, 0, 0><<<grid, 128, smem, st>>>(x, w, d); break;
    case 64: k_conv_stem<64, 0, 0, 0, 0><<<grid, 128, smem, st>>>(x, w, d); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace osam

// ------------------------------------------------------------------------------------------------
// Pipelined RGB stem (3×3, stride 2, pad 1, C = 3, K = 32): tiles of 2 output rows × 64 columns of one
// image, persistent over the tile list, warp-specialised like the main conv kernel:
//   warp 0       TMA: the tile's input window (5 rows × 387 fp16, i.e. 129 pixels × 3 channels) as two
//                208-element boxes of the (W·C, H, N) view into a 6-slot ring; the out-of-range zero fill
//                of the tensor engine supplies every conv pad (top/bottom rows, left/right columns);
//   warps 2, 3   im2col: each thread builds two 64-byte swizzled K-major rows of the A tile (4-slot ring)
//                from three aligned 20-byte runs of the window per row, one per kernel row;
//   warp 1       TMEM owner + MMA issuer: two K=16 UMMAs per tile into one of two accumulators;
//   warps 4..11  epilogue: two warps per TMEM lane quadrant, 16 of the 32 channels each — folded BN +
//                SiLU, fp16, and one TMA tensor store of the warp's 32 pixels × 16 channels.
// The layer moves 6 B in and 64 B out per output pixel, and the BN + SiLU of 32 channels per pixel is
// the largest instruction stream in it: eight epilogue warps per CTA (sixteen per SM) keep enough
// independent work in flight to hide the exponential's and the reciprocal's latency (with four the
// epilogue set the pace: 0.236 ms per 64 images, 0.127 ms with the math left out).
// K layout of a row: kernel row r occupies k = 10r … 10r+9.  For output column q the nine taps of row r
// (input columns 2q−1 … 2q+1, three channels each) are the nine consecutive halves that start at element
// 6q − 3 of the input row; the run of TEN halves that starts one element earlier (at 6q − 4, always even)
// is 4-byte aligned in the window, so it is read as five 32-bit words.  Its first half belongs to the
// previous pixel and meets a zero weight (k = 10r), as do k = 30, 31.  The weights (32 × 27, laid out
// this way) stay in shared memory for the whole kernel.
namespace osam {

constexpr int kS2Win = 6, kS2A = 4;
constexpr int kS2Box = 208;                  // fp16 elements per window box row (416 B)
constexpr int kS2Box1 = 200;                 // the second box starts 200 elements in (overlapping the first by 8,
                                             // so no ten-element run straddles the two)
constexpr int kS2BoxBytes = 2176;            // one box of 5 rows (2080 B), padded to 128 B
constexpr int kS2WinBytes = 2 * kS2BoxBytes;  // two boxes per window
constexpr int kS2EpiWarps = 8, kS2Im2colWarps = 2;
constexpr int kS2Threads = 32 * (2 + kS2Im2colWarps + kS2EpiWarps);
constexpr int kS2StageBytes = 32 * 32;       // per epilogue warp: 32 pixels × 16 channels, unswizzled
constexpr int kS2Smem =
    1024 + kS2A * 8192 + 2048 + kS2EpiWarps * kS2StageBytes + kS2Win * kS2WinBytes + 2 * 32 * 4 + 512;

// The epilogue of 16 accumulator columns of one pixel row per lane — folded BN (+ SiLU), bias or the plain
// value, as the generic TMA-store epilogue does — then the warp's 32 rows × 16 channels leave through one
// tensor store per destination view (four for a 2×-upsampled destination).
__device__ __forceinline__ void stem_epilogue16(const EpiDev& e, const StoreMaps& maps, float* v, int col,
                                                const float* s_sc, const float* s_sh, int bq, int bp, int bn,
                                                uint8_t* stage) {
  const int lane = threadIdx.x & 31;
  if (e.round_z) {
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __half2float(__float2half_rn(v[i]));
  }
  if (e.kind == OSAM_EPI_BN_ACT) {  // folded BN (+ SiLU)
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      const float4 sc = *reinterpret_cast<const float4*>(s_sc + col + i);
      const float4 sh = *reinterpret_cast<const float4*>(s_sh + col + i);
      if (e.act) {
        bn_silu4(sc, sh, v + i, v + i);
      } else {
        v[i] = fmaf(sc.x, v[i], sh.x);
        v[i + 1] = fmaf(sc.y, v[i + 1], sh.y);
        v[i + 2] = fmaf(sc.z, v[i + 2], sh.z);
        v[i + 3] = fmaf(sc.w, v[i + 3], sh.w);
      }
    }
  } else if (e.kind == OSAM_EPI_BIAS) {
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] += s_sh[col + i];
  }
  if (lane == 0) bulk_wait_group_read0();  // the previous tile's store has read the stage
  __syncwarp();
  uint4* row = reinterpret_cast<uint4*>(stage + lane * 32);
  row[0] = pack8h(v);
  row[1] = pack8h(v + 8);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
#pragma unroll
    for (int t = 0; t < OSAM_MAX_DEST; t++) {
      if (t >= e.ndest) break;
      const DestDev& ds = e.dest[t];
      if (col < ds.c0 || col >= ds.c1) continue;
      const int kk = ds.choff + col - ds.c0;
      const int views = ds.up == 1 ? 1 : 4;
      for (int vw = 0; vw < views; vw++) tma_store_4d(&maps.m[4 * t + vw], stage, kk, bq, bp, bn);
    }
    bulk_commit_group();
  }
}

__global__ void __launch_bounds__(kS2Threads, 2)
    k_conv_stem_rgb(const __grid_constant__ CUtensorMap tw, const __grid_constant__ StoreMaps sm,
                    const __half* __restrict__ w, const ConvDev d) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;                         // kS2A × 8 KiB, 1024-aligned
  uint8_t* sB = sA + kS2A * 8192;             // 32 × 64 B
  uint8_t* s_stage = sB + 2048;               // kS2EpiWarps × 1 KiB
  uint8_t* s_win = s_stage + kS2EpiWarps * kS2StageBytes;  // kS2Win windows
  float* s_sc = reinterpret_cast<float*>(s_win + kS2Win * kS2WinBytes);
  float* s_sh = s_sc + 32;
  uint64_t* wfull = reinterpret_cast<uint64_t*>(s_sh + 32);
  uint64_t* wempty = wfull + kS2Win;
  uint64_t* afull = wempty + kS2Win;
  uint64_t* aempty = afull + kS2A;
  uint64_t* accf = aempty + kS2A;
  uint64_t* acce = accf + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acce + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = d.tiles_m;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kS2Win; i++) {
      mbar_init(wfull + i, 1);
      mbar_init(wempty + i, kS2Im2colWarps);
    }
    for (int i = 0; i < kS2A; i++) {
      mbar_init(afull + i, kS2Im2colWarps);
      mbar_init(aempty + i, 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(accf + i, 1);
      mbar_init(acce + i, kS2EpiWarps);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tw);
  }
  if (warp == 1) {
    tmem_alloc(tslot, 64);
    tmem_relinquish();
  }
  // weights: row k = the 27 taps of output channel k (KRSC) at k = 10r + 1 + 3s + c, 64-byte swizzle
  for (int i = threadIdx.x; i < 32 * 4; i += blockDim.x) {
    const int r = i >> 2, ch = i & 3;
    __align__(16) __half v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const int kk = ch * 8 + e, kr = kk / 10, t = kk - kr * 10;
      v[e] = (r < d.K && kr < 3 && t > 0) ? w[r * 27 + kr * 9 + (t - 1)] : __float2half(0.f);
    }
    *reinterpret_cast<uint4*>(sB + r * 64 + ((ch ^ ((r >> 1) & 3)) << 4)) = *reinterpret_cast<const uint4*>(v);
  }
  if (threadIdx.x < 32) load_epilogue_consts(d.ep, d.gemm_n, 0, 32, threadIdx.x, 32, s_sc, s_sh);
  fence_proxy_async_smem();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  // the next conv (launched with programmatic dependent launch; it waits for this grid before it reads)
  // may be scheduled as soon as this grid's CTAs retire, instead of after the launch gap
  grid_dep_launch();

  if (warp == 0) {
    // ---------------------------------------------------------------- window producer
    if (lane == 0) {
      int lt = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, lt++) {
        const int s = lt % kS2Win;
        if (lt >= kS2Win && !mbar_wait(wempty + s, ((lt / kS2Win) - 1) & 1, d.err)) break;
        const int rest = d.f_tq.quo(t), tq = d.f_tq.rem(t, rest), n = d.f_tp.quo(rest), tp = d.f_tp.rem(rest, n);
        const int x0 = (2 * tq * 64 - 1) * 3;          // first element of the window row in the W·C row
        const int xa = x0 >= 0 ? (x0 & ~7) : -((-x0 + 7) & ~7);  // aligned down to 8 elements (16 B)
        const int ih0 = 2 * tp * 2 - 1;
        mbar_arrive_expect_tx(wfull + s, 2 * 5 * kS2Box * 2);
        uint8_t* dst = s_win + s * kS2WinBytes;
        tma_load_3d(dst, &tw, wfull + s, xa, ih0, n);
        tma_load_3d(dst + kS2BoxBytes, &tw, wfull + s, xa + kS2Box1, ih0, n);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, 32);
      int lt = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, lt++) {
        const int s = lt % kS2A;
        const uint32_t buf = lt & 1;
        if (lt >= 2 && !mbar_wait(acce + buf, ((lt >> 1) - 1) & 1, d.err)) break;
        if (!mbar_wait(afull + s, (lt / kS2A) & 1, d.err)) break;
        tc_fence_after();
        const uint32_t a = smem_u32(sA + s * 8192), b = smem_u32(sB);
        umma_f16(tmem + buf * 32, smem_desc_kmajor(a, 64), smem_desc_kmajor(b, 64), idesc, 0);
        umma_f16(tmem + buf * 32, smem_desc_kmajor(a + 32, 64), smem_desc_kmajor(b + 32, 64), idesc, 1);
        umma_commit(aempty + s);
        umma_commit(accf + buf);
      }
    }
  } else if (warp < 2 + kS2Im2colWarps) {
    // ---------------------------------------------------------------- im2col (two A rows per thread)
    const int tid = threadIdx.x - 64;  // 0..63: rows tid (output row 0 of the tile) and tid + 64 (row 1)
    // the ten-half run of kernel row r starts at window element 6j + 4 (the window starts 4 elements before
    // the run of the tile's first column: xa = 6·q0 − 8 rounded as the producer rounds it); a run ending
    // past element 208 is read from the second box, which starts at element 200
    const int e0 = 6 * tid + 4;
    const int run_off = e0 + 10 <= kS2Box ? e0 * 2 : kS2BoxBytes + (e0 - kS2Box1) * 2;  // bytes into a window row
    int lt = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, lt++) {
      const int ws = lt % kS2Win, as = lt % kS2A;
      if (!mbar_wait(wfull + ws, (lt / kS2Win) & 1, d.err)) break;
      if (lt >= kS2A && !mbar_wait(aempty + as, ((lt / kS2A) - 1) & 1, d.err)) break;
      const uint8_t* win = s_win + ws * kS2WinBytes + run_off;
#pragma unroll
      for (int i = 0; i < 2; i++) {
        const int arow = i * 64 + tid;
        uint32_t row[16];
#pragma unroll
        for (int r = 0; r < 3; r++) {
          const uint32_t* src = reinterpret_cast<const uint32_t*>(win + (2 * i + r) * (kS2Box * 2));
#pragma unroll
          for (int u = 0; u < 5; u++) row[5 * r + u] = src[u];
        }
        row[15] = 0u;
        uint8_t* dst = sA + as * 8192 + arow * 64;
#pragma unroll
        for (int ch = 0; ch < 4; ch++)
          *reinterpret_cast<uint4*>(dst + ((ch ^ ((arow >> 1) & 3)) << 4)) =
              make_uint4(row[4 * ch], row[4 * ch + 1], row[4 * ch + 2], row[4 * ch + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(afull + as);
        mbar_arrive(wempty + ws);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 4..11)
    const int ew = warp - 2 - kS2Im2colWarps;  // 0..7
    const int quad = warp & 3;                 // TMEM lane quadrant this warp may access
    const int col = (ew >> 2) * 16;            // its 16 of the 32 channels
    uint8_t* stage = s_stage + ew * kS2StageBytes;
    int lt = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, lt++) {
      const int rest = d.f_tq.quo(t), tq = d.f_tq.rem(t, rest), n = d.f_tp.quo(rest), tp = d.f_tp.rem(rest, n);
      const int bq = tq * 64 + ((quad * 32) & 63), bp = tp * 2 + (quad >> 1);
      const uint32_t buf = lt & 1;
      const bool ok = mbar_wait(accf + buf, (lt >> 1) & 1, d.err);
      tc_fence_after();
      if (!ok) break;
      uint32_t r0[16];
      tmem_ld16_nowait(tmem + buf * 32 + col + ((uint32_t)(quad * 32) << 16), r0);
      tmem_wait_ld();
      float v[16];
#pragma unroll
      for (int k = 0; k < 16; k++) v[k] = __uint_as_float(r0[k]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce + buf);  // accumulator registers are loaded: TMEM may be reused
      stem_epilogue16(d.ep, sm, v, col, s_sc, s_sh, bq, bp, n, stage);
    }
    if (lane == 0) bulk_wait_group0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

cudaError_t launch_conv_stem_rgb(const ConvLaunch& L, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_conv_stem_rgb, cudaFuncAttributeMaxDynamicSharedMemorySize, kS2Smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int grid = L.d.tiles_m < 2 * sms ? L.d.tiles_m : 2 * sms;  // two CTAs per SM
  k_conv_stem_rgb<<<grid, kS2Threads, kS2Smem, st>>>(L.ta, L.sm, L.w, L.d);
  return cudaGetLastError();
}

}  // namespace osam
