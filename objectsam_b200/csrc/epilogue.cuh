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
// s_sc/s_sh/s_bi hold the tile's per-column scale, shift and bias.
__device__ __forceinline__ void epilogue8(const EpiDev& e, int K, int P, int Q, float (&y)[8], int cnt, int col,
                                          int li, const float* s_sc, const float* s_sh, const float* s_bi,
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
    for (int i = 0; i < 8; i++) y[i] += s_bi[li + i];
  } else if (e.beta != 0.f) {
    const DestDev& ds = e.dest[0];
    const __half* old = ds.p + opix * ds.ctot + ds.choff + k - ds.c0;
    for (int i = 0; i < cnt; i++) y[i] += e.beta * __half2float(old[i]);
  }
  store_dests(e, opix, n, op, oq, OP, OQ, k, y, cnt);
}

// Per-column epilogue constants of the tile starting at GEMM column n0 (BN columns) into shared memory.
__device__ __forceinline__ void load_epilogue_consts(const EpiDev& e, int gemm_n, int n0, int BN, int tid,
                                                     int nthreads, float* s_sc, float* s_sh, float* s_bi) {
  for (int i = tid; i < BN; i += nthreads) {
    const int col = n0 + i;
    const bool ok = col < gemm_n;
    const int kc = e.shuffle ? col % e.kout : col;
    s_sc[i] = (ok && e.scale) ? e.scale[kc] : 1.f;
    s_sh[i] = (ok && e.shift) ? e.shift[kc] : 0.f;
    s_bi[i] = (ok && e.bias) ? e.bias[kc] : 0.f;
  }
}

}  // namespace osam
