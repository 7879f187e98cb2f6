// Fused conv epilogue shared by the conv kernels: the per-output-channel math that the reference runs as
// separate HBM passes after cuDNN (bn_eval_scale + bn_forward_apply, src/bn.cu:204-238, :277-284;
// add_bias, src/misc.cu:116-134) and its multi-destination store (Dest/DestList, src/bn.cuh:10-21).
#pragma once
#include "conv_internal.h"
#include "sm100.cuh"

namespace osam {

// SiLU with the fast exponential and division the reference's fast-math build also uses
// (CMakeLists.txt:11 --use_fast_math, src/bn.cu:35).
__device__ __forceinline__ float silu_f(float y) { return __fdividef(y, 1.f + __expf(-y)); }

// Store `cnt` (≤ 8) consecutive output channels starting at `k` of one output pixel to every destination
// whose channel range holds them.  `pix` indexes the P×Q output grid; (n, p, q) locate it for the 2×
// upsampled destinations.
__device__ __forceinline__ void store_dests(const EpiDev& e, long long pix, int n, int p, int q, int P, int Q, int k,
                                            const float* y, int cnt) {
#pragma unroll 1
  for (int t = 0; t < e.ndest; t++) {
    const DestDev& ds = e.dest[t];
    if (k + cnt <= ds.c0 || k >= ds.c1) continue;
    const bool full = cnt == 8 && ds.vec && k >= ds.c0 && k + 8 <= ds.c1;
    if (ds.up == 1) {
      __half* o = ds.p + pix * ds.ctot + ds.choff - ds.c0;
      if (full) {
        st8h(o + k, y);
      } else {
        for (int i = 0; i < cnt; i++)
          if (k + i >= ds.c0 && k + i < ds.c1) o[k + i] = __float2half_rn(y[i]);
      }
    } else {
      const long long Q2 = 2LL * Q, base = ((long long)n * 2 * P + 2 * p) * Q2 + 2 * q;
      const long long px4[4] = {base, base + 1, base + Q2, base + Q2 + 1};
#pragma unroll
      for (int u = 0; u < 4; u++) {
        __half* o = ds.p + px4[u] * ds.ctot + ds.choff - ds.c0;
        if (full) {
          st8h(o + k, y);
        } else {
          for (int i = 0; i < cnt; i++)
            if (k + i >= ds.c0 && k + i < ds.c1) o[k + i] = __float2half_rn(y[i]);
        }
      }
    }
  }
}

// Epilogue of 8 accumulator columns [col, col+8) (local columns [li, li+8) of the CTA's tile) of the
// output pixel `pix` = (n, p, q) on the P×Q grid.  `cnt` columns are real (the rest are GEMM padding).
// s_sc/s_sh hold the per-column scale and shift (or bias).
__device__ __forceinline__ void epilogue8(const EpiDev& e, int K, int P, int Q, float (&y)[8], int cnt, int col,
                                          int li, const float* s_sc, const float* s_sh,
                                          long long pix, int n, int p, int q) {
  if (e.round_z) {
#pragma unroll
    for (int i = 0; i < 8; i++) y[i] = __half2float(__float2half_rn(y[i]));
  }
  long long opix = pix;
  int op = p, oq = q, k = col, OP = P, OQ = Q;
  if (e.shuffle) {  // transposed conv: column block (dy·2+dx) → output pixel (2p+dy, 2q+dx)
    const int blk = col / e.kout;
    k = col - blk * e.kout;
    op = 2 * p + (blk >> 1);
    oq = 2 * q + (blk & 1);
    OP = 2 * P;
    OQ = 2 * Q;
    opix = ((long long)n * OP + op) * OQ + oq;
  }
  if (e.kind == OSAM_EPI_BN_ACT) {
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float t = s_sc[li + i] * y[i] + s_sh[li + i];
      y[i] = e.act ? silu_f(t) : t;
    }
    if (e.res) {
      const __half* rp = e.res + pix * K + k;
      if (cnt == 8 && (K & 7) == 0) {
        float r8[8];
        ld8h(rp, r8);
#pragma unroll
        for (int i = 0; i < 8; i++) y[i] += r8[i];
      } else {
        for (int i = 0; i < cnt; i++) y[i] += __half2float(rp[i]);
      }
    }
  } else if (e.kind == OSAM_EPI_BIAS) {
#pragma unroll
    for (int i = 0; i < 8; i++) y[i] += s_sh[li + i];
  } else if (e.beta != 0.f) {
    const DestDev& ds = e.dest[0];
    const __half* old = ds.p + opix * ds.ctot + ds.choff + k - ds.c0;
    for (int i = 0; i < cnt; i++) y[i] += e.beta * __half2float(old[i]);
  }
  store_dests(e, opix, n, op, oq, OP, OQ, k, y, cnt);
}

// ------------------------------------------------------------------ warp-cooperative (coalesced) epilogue
//
// One warp owns 32 accumulator rows (= 32 output pixels, lane i ↔ row i).  A pass handles W = 16 or 32
// columns: each lane computes its row, writes it as fp16 16-byte chunks into a per-warp shared-memory
// stage (32 rows × 64 B, chunk index XOR-swizzled by row so both the row-wise writes and the
// column-wise reads are bank-conflict free), then the warp re-reads the stage so that consecutive
// lanes hold consecutive chunks of the same pixel and stores them: one warp instruction writes
// 32/(W/8) whole pixel rows instead of 32 scattered 16-byte pieces.  The residual is brought in the
// same way in reverse.  Requires EpiDev::coop (every destination 8-channel aligned, full tiles).

__device__ __forceinline__ uint32_t stage_off(int r, int c) { return r * 64 + ((c ^ ((r >> 1) & 3)) << 4); }

__device__ __forceinline__ uint4 pack8h(const float* y) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(y[2 * i], y[2 * i + 1]);
  return u;
}
__device__ __forceinline__ void unpack8h(uint4 u, float* o) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    float2 f = __half22float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}

// v: this lane's W accumulator values of GEMM columns [col, col+W); (valid, n, p, q): this lane's output
// pixel on the P×Q GEMM grid.  s_sc/s_sh are indexed by GEMM column.
template <int W>
__device__ __forceinline__ void epilogue_warp(const EpiDev& e, int K, int P, int Q, const float* v, int col,
                                              const float* s_sc, const float* s_sh, bool valid,
                                              int n, int p, int q, uint8_t* stage) {
  constexpr int CPR = W / 8;     // 16-byte chunks per row
  constexpr int RPI = 32 / CPR;  // rows per cooperative instruction
  const int lane = threadIdx.x & 31;
  const int my_n = valid ? n : -1;
  const int my_pq = (p << 16) | (q & 0xffff);
  int k0 = col, dy = 0, dx = 0, OP = P, OQ = Q;
  if (e.shuffle) {  // transposed conv: the pass lies in one (dy, dx) block (kout % 32 == 0)
    const int blk = col / e.kout;
    k0 = col - blk * e.kout;
    dy = blk >> 1;
    dx = blk & 1;
    OP = 2 * P;
    OQ = 2 * Q;
  }
  float y[W];
#pragma unroll
  for (int i = 0; i < W; i++) {
    float z = v[i];
    if (e.round_z) z = __half2float(__float2half_rn(z));
    if (e.kind == OSAM_EPI_BN_ACT) {
      const float t = s_sc[col + i] * z + s_sh[col + i];
      z = e.act ? silu_f(t) : t;
    } else if (e.kind == OSAM_EPI_BIAS) {
      z += s_sh[col + i];
    }
    y[i] = z;
  }
  if (e.kind == OSAM_EPI_BN_ACT && e.res) {
#pragma unroll
    for (int it = 0; it < CPR; it++) {
      const int rr = it * RPI + lane / CPR, ch = lane % CPR;
      const int rn = __shfl_sync(0xffffffffu, my_n, rr);
      const int rpq = __shfl_sync(0xffffffffu, my_pq, rr);
      uint4 val = make_uint4(0, 0, 0, 0);
      if (rn >= 0) {
        const long long rpix = ((long long)rn * P + (rpq >> 16)) * Q + (rpq & 0xffff);
        val = *reinterpret_cast<const uint4*>(e.res + rpix * K + col + ch * 8);
      }
      *reinterpret_cast<uint4*>(stage + stage_off(rr, ch)) = val;
    }
    __syncwarp();
#pragma unroll
    for (int ch = 0; ch < CPR; ch++) {
      float r8[8];
      unpack8h(*reinterpret_cast<const uint4*>(stage + stage_off(lane, ch)), r8);
#pragma unroll
      for (int i = 0; i < 8; i++) y[ch * 8 + i] += r8[i];
    }
    __syncwarp();
  }
#pragma unroll
  for (int ch = 0; ch < CPR; ch++) *reinterpret_cast<uint4*>(stage + stage_off(lane, ch)) = pack8h(y + ch * 8);
  __syncwarp();
#pragma unroll
  for (int it = 0; it < CPR; it++) {
    const int rr = it * RPI + lane / CPR, ch = lane % CPR;
    const int rn = __shfl_sync(0xffffffffu, my_n, rr);
    const int rpq = __shfl_sync(0xffffffffu, my_pq, rr);
    const uint4 val = *reinterpret_cast<const uint4*>(stage + stage_off(rr, ch));
    if (rn < 0) continue;
    int op = rpq >> 16, oq = rpq & 0xffff;
    if (e.shuffle) {
      op = 2 * op + dy;
      oq = 2 * oq + dx;
    }
    const int k = k0 + ch * 8;
#pragma unroll 1
    for (int t = 0; t < e.ndest; t++) {
      const DestDev& ds = e.dest[t];
      if (k < ds.c0 || k >= ds.c1) continue;
      __half* b = ds.p + ds.choff - ds.c0 + k;
      if (ds.up == 1) {
        *reinterpret_cast<uint4*>(b + (((long long)rn * OP + op) * OQ + oq) * ds.ctot) = val;
      } else {
        const long long Q2 = 2LL * OQ, px = ((long long)rn * 2 * OP + 2 * op) * Q2 + 2 * oq;
        *reinterpret_cast<uint4*>(b + px * ds.ctot) = val;
        *reinterpret_cast<uint4*>(b + (px + 1) * ds.ctot) = val;
        *reinterpret_cast<uint4*>(b + (px + Q2) * ds.ctot) = val;
        *reinterpret_cast<uint4*>(b + (px + Q2 + 1) * ds.ctot) = val;
      }
    }
  }
  __syncwarp();
}

// Per-column epilogue constants of the tile starting at GEMM column n0 (BN columns) into shared memory:
// s_sc = BN scale (1 otherwise), s_sh = BN shift or the bias (0 otherwise).
__device__ __forceinline__ void load_epilogue_consts(const EpiDev& e, int gemm_n, int n0, int BN, int tid,
                                                     int nthreads, float* s_sc, float* s_sh) {
  for (int i = tid; i < BN; i += nthreads) {
    const int col = n0 + i;
    const bool ok = col < gemm_n;
    const int kc = e.shuffle ? col % e.kout : col;
    const bool bn = e.kind == OSAM_EPI_BN_ACT, bias = e.kind == OSAM_EPI_BIAS;
    s_sc[i] = (ok && bn && e.scale) ? e.scale[kc] : 1.f;
    s_sh[i] = ok ? ((bn && e.shift) ? e.shift[kc] : ((bias && e.bias) ? e.bias[kc] : 0.f)) : 0.f;
  }
}

}  // namespace osam
