// Fused conv epilogue shared by the conv kernels: the per-output-channel math that the reference runs as
// separate HBM passes after cuDNN (bn_eval_scale + bn_forward_apply, src/bn.cu:204-238, :277-284;
// add_bias, src/misc.cu:116-134) and its multi-destination store (Dest/DestList, src/bn.cuh:10-21).
#pragma once
#include "conv_internal.h"
#include "sm100.cuh"

namespace osam {

// 1/d for d ≥ 1 on the FMA pipe: the exponent-flip initial estimate (magic-constant method; with this
// constant its relative error is at most 5.1 %, measured over every fp32 mantissa) refined by two
// Newton–Raphson steps r ← r·(2 − d·r), which square the error each time: ≤ 6.5e-6, 75× below half an
// fp16 ulp (the epilogue's results are stored in fp16).  Keeps the quarter-rate MUFU unit free for the
// exponential.
__device__ __forceinline__ float rcp_nr(float d) {
  float r = __int_as_float(0x7EF311C3 - __float_as_int(d));
  r = r * fmaf(-d, r, 2.f);
  r = r * fmaf(-d, r, 2.f);
  return r;
}
// SiLU y·σ(y) = y / (1 + e^{−y}): one MUFU exponential (the reference's fast-math build uses __expf too,
// CMakeLists.txt:11, src/bn.cu:35) and the FMA-pipe reciprocal above.  y is clamped at −80 so 1 + e^{−y}
// stays finite; silu(−80) ≈ −1e-33 rounds to −0 in fp16 either way.
__device__ __forceinline__ float silu_f(float y) {
  const float e = __expf(-fmaxf(y, -80.f));
  return y * rcp_nr(1.f + e);
}

// ---- packed pairs: sm_100's f32x2 FMA-pipe instructions take one issue slot for two fp32 values
__device__ __forceinline__ uint64_t f2bits(float2 a) {
  uint64_t u;
  asm("mov.b64 %0, {%1, %2};" : "=l"(u) : "f"(a.x), "f"(a.y));
  return u;
}
__device__ __forceinline__ float2 f2from(uint64_t u) {
  float2 a;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a.x), "=f"(a.y) : "l"(u));
  return a;
}
__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2bits(a)), "l"(f2bits(b)), "l"(f2bits(c)));
  return f2from(d);
}
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2bits(a)), "l"(f2bits(b)));
  return f2from(d);
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// SiLU of two values, t·σ(t) with σ(t) = 1 / (1 + 2^(−t·log₂e)), on packed pairs: the exponent argument
// is clamped at 115.4 (t ≥ −80, as silu_f), nd = −(1 + e) comes from one FMA, and 1/(1 + e) is the
// exponent-flip estimate (rcp_nr's constant, the sign bit folded in: 0xFEF311C3 − bits(nd) =
// 0x7EF311C3 − bits(−nd)) refined by the same two Newton–Raphson steps r ← r·(2 + nd·r).
__device__ __forceinline__ float2 silu2(float2 t) {
  constexpr float kNegLog2e = -1.4426950408889634f;
  const float2 a = f2mul(t, make_float2(kNegLog2e, kNegLog2e));
  const float2 e = make_float2(ex2_approx(fminf(a.x, 115.4f)), ex2_approx(fminf(a.y, 115.4f)));
  const float2 nd = f2fma(e, make_float2(-1.f, -1.f), make_float2(-1.f, -1.f));
  float2 r = make_float2(__uint_as_float(0xFEF311C3u - __float_as_uint(nd.x)),
                         __uint_as_float(0xFEF311C3u - __float_as_uint(nd.y)));
  const float2 two = make_float2(2.f, 2.f);
  r = f2mul(r, f2fma(nd, r, two));
  r = f2mul(r, f2fma(nd, r, two));
  return f2mul(t, r);
}

// BN + SiLU of four consecutive columns: y = silu(sc·v + sh).
__device__ __forceinline__ void bn_silu4(const float4 sc, const float4 sh, const float* v, float* y) {
  const float2 t0 = f2fma(make_float2(sc.x, sc.y), make_float2(v[0], v[1]), make_float2(sh.x, sh.y));
  const float2 t1 = f2fma(make_float2(sc.z, sc.w), make_float2(v[2], v[3]), make_float2(sh.z, sh.w));
  const float2 y0 = silu2(t0), y1 = silu2(t1);
  y[0] = y0.x;
  y[1] = y0.y;
  y[2] = y1.x;
  y[3] = y1.y;
}

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
  if (e.shuffle || e.par) {  // column block (dy·2+dx), or the fixed parity class → pixel (2p+dy, 2q+dx)
    const int blk = e.par ? e.par - 1 : col / e.kout;
    k = e.par ? col : col - blk * e.kout;
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

// v: this lane's W accumulator values of GEMM columns [col, col+W) (col % 16 == 0); (valid, n, p, q):
// this lane's output pixel on the P×Q GEMM grid.  s_sc/s_sh are indexed by GEMM column.
// The math runs as branch-free unrolled loops (the kind/act/round flags are hoisted), and the stores
// use one shuffled 32-bit pixel index per row, so independent elements overlap in the pipelines.
template <int W>
__device__ __forceinline__ void epilogue_warp(const EpiDev& e, int K, int P, int Q, float* v, int col,
                                              const float* s_sc, const float* s_sh, bool valid, int n, int p,
                                              int q, uint8_t* stage) {
  constexpr int CPR = W / 8;     // 16-byte chunks per row
  constexpr int RPI = 32 / CPR;  // rows per cooperative instruction
  const int lane = threadIdx.x & 31;
  int k0 = col, OP = P, OQ = Q, op = p, oq = q;
  if (e.shuffle || e.par) {  // transposed conv: the pass lies in one (dy, dx) block (kout % 32 == 0)
    const int blk = e.par ? e.par - 1 : col / e.kout;
    k0 = e.par ? col : col - blk * e.kout;
    OP = 2 * P;
    OQ = 2 * Q;
    op = 2 * p + (blk >> 1);
    oq = 2 * q + (blk & 1);
  }
  // this lane's output pixel (−1: outside the output) and its 2×-upsampled base pixel
  const int my_o = valid ? (n * OP + op) * OQ + oq : -1;
  const int my_u = (n * 2 * OP + 2 * op) * (2 * OQ) + 2 * oq;
  const int my_r = (n * P + p) * Q + q;  // residual pixel (GEMM grid)

  // ---- math (hoisted flags, branch-free loops)
  if (e.round_z) {
#pragma unroll
    for (int i = 0; i < W; i++) v[i] = __half2float(__float2half_rn(v[i]));
  }
  float y[W];
  if (e.kind == OSAM_EPI_BN_ACT) {
    float sc[W], sh[W];
#pragma unroll
    for (int i = 0; i < W; i += 4) {
      *reinterpret_cast<float4*>(sc + i) = *reinterpret_cast<const float4*>(s_sc + col + i);
      *reinterpret_cast<float4*>(sh + i) = *reinterpret_cast<const float4*>(s_sh + col + i);
    }
    if (e.act) {
#pragma unroll
      for (int i = 0; i < W; i += 4)
        bn_silu4(make_float4(sc[i], sc[i + 1], sc[i + 2], sc[i + 3]), make_float4(sh[i], sh[i + 1], sh[i + 2], sh[i + 3]),
                 v + i, y + i);
    } else {
#pragma unroll
      for (int i = 0; i < W; i++) y[i] = fmaf(sc[i], v[i], sh[i]);
    }
  } else if (e.kind == OSAM_EPI_BIAS) {
#pragma unroll
    for (int i = 0; i < W; i += 4) {
      const float4 b = *reinterpret_cast<const float4*>(s_sh + col + i);
      y[i] = v[i] + b.x;
      y[i + 1] = v[i + 1] + b.y;
      y[i + 2] = v[i + 2] + b.z;
      y[i + 3] = v[i + 3] + b.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < W; i++) y[i] = v[i];
    // beta ≠ 0 (one plain destination): y += beta·(its current values), the rows read coalesced into the
    // stage and each lane taking its own, the same way as the residual below
    if (e.beta != 0.f) {
      const DestDev& ds = e.dest[0];
      const __half* ob = ds.p + (ds.choff - ds.c0);
#pragma unroll
      for (int it = 0; it < CPR; it++) {
        const int rr = it * RPI + lane / CPR, ch = lane % CPR, k = k0 + ch * 8;
        const int ro = __shfl_sync(0xffffffffu, my_o, rr);
        uint4 val = make_uint4(0, 0, 0, 0);
        if (ro >= 0 && k >= ds.c0 && k < ds.c1) val = *reinterpret_cast<const uint4*>(ob + (long long)ro * ds.ctot + k);
        *reinterpret_cast<uint4*>(stage + stage_off(rr, ch)) = val;
      }
      __syncwarp();
#pragma unroll
      for (int ch = 0; ch < CPR; ch++) {
        float o8[8];
        unpack8h(*reinterpret_cast<const uint4*>(stage + stage_off(lane, ch)), o8);
#pragma unroll
        for (int i = 0; i < 8; i++) y[ch * 8 + i] += e.beta * o8[i];
      }
      __syncwarp();
    }
  }

  // ---- residual: coalesced rows into the stage, then each lane reads its own row
  if (e.kind == OSAM_EPI_BN_ACT && e.res) {
    const int my_rv = valid ? my_r : -1;
#pragma unroll
    for (int it = 0; it < CPR; it++) {
      const int rr = it * RPI + lane / CPR, ch = lane % CPR;
      const int rpix = __shfl_sync(0xffffffffu, my_rv, rr);
      uint4 val = make_uint4(0, 0, 0, 0);
      if (rpix >= 0) val = *reinterpret_cast<const uint4*>(e.res + (long long)rpix * K + col + ch * 8);
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

  // ---- fp16 rows into the stage, then whole pixel rows out
#pragma unroll
  for (int ch = 0; ch < CPR; ch++) *reinterpret_cast<uint4*>(stage + stage_off(lane, ch)) = pack8h(y + ch * 8);
  __syncwarp();
  const int nd = e.ndest;
#pragma unroll
  for (int it = 0; it < CPR; it++) {
    const int rr = it * RPI + lane / CPR, ch = lane % CPR;
    const int ro = __shfl_sync(0xffffffffu, my_o, rr);
    const int ru = __shfl_sync(0xffffffffu, my_u, rr);
    const uint4 val = *reinterpret_cast<const uint4*>(stage + stage_off(rr, ch));
    if (ro < 0) continue;
    const int k = k0 + ch * 8;
#pragma unroll
    for (int t = 0; t < OSAM_MAX_DEST; t++) {
      if (t >= nd) break;
      const DestDev& ds = e.dest[t];
      if (k < ds.c0 || k >= ds.c1) continue;
      __half* b = ds.p + (ds.choff - ds.c0 + k);
      if (ds.up == 1) {
        *reinterpret_cast<uint4*>(b + (long long)ro * ds.ctot) = val;
      } else {
        const long long c = ds.ctot, q2 = 2LL * OQ;
        __half* u = b + (long long)ru * c;
        *reinterpret_cast<uint4*>(u) = val;
        *reinterpret_cast<uint4*>(u + c) = val;
        *reinterpret_cast<uint4*>(u + q2 * c) = val;
        *reinterpret_cast<uint4*>(u + (q2 + 1) * c) = val;
      }
    }
  }
  __syncwarp();
}

// TMA-store variant (EpiDev::tstore): the warp's 32 rows form a box (wtn images × wth rows × wtw cols)
// whose origin on the GEMM grid is (bq, bp, bn).  After the math, the rows go into the per-warp stage in
// the 64-byte TMA swizzle and one lane issues a tensor store per destination (four for 2× upsampled
// destinations and for the transposed conv's pixel shuffle, one per (dy, dx) view).  The tensor engine
// clips rows outside the output, so partial tiles need no masking.  W = 32 (64-byte stage rows).
// `rsm` (optional): this pass's residual rows already in shared memory (32 rows × 64 B, stage_off layout),
// read instead of the global residual.  `rreg` (optional): this pass's residual rows already in registers,
// loaded by residual_rows (below) before the accumulator was ready.
__device__ __forceinline__ void epilogue_warp_tma(const EpiDev& e, const StoreMaps& maps, int K, int P, int Q,
                                                  float* v, int col, const float* s_sc, const float* s_sh,
                                                  bool valid, int n, int p, int q, int bq, int bp, int bn,
                                                  uint8_t* stage, const uint8_t* rsm = nullptr,
                                                  const uint4* rreg = nullptr) {
  constexpr int W = 32, CPR = 4, RPI = 8;
  const int lane = threadIdx.x & 31;
  if (e.round_z) {
#pragma unroll
    for (int i = 0; i < W; i++) v[i] = __half2float(__float2half_rn(v[i]));
  }
  float* y = v;  // in place: keeps the live register set small
  if (e.kind == OSAM_EPI_BN_ACT) {
    if (e.act) {
#pragma unroll
      for (int i = 0; i < W; i += 4) {
        const float4 sc = *reinterpret_cast<const float4*>(s_sc + col + i);
        const float4 sh = *reinterpret_cast<const float4*>(s_sh + col + i);
        bn_silu4(sc, sh, v + i, y + i);
      }
    } else {
#pragma unroll
      for (int i = 0; i < W; i += 4) {
        const float4 sc = *reinterpret_cast<const float4*>(s_sc + col + i);
        const float4 sh = *reinterpret_cast<const float4*>(s_sh + col + i);
        y[i] = fmaf(sc.x, v[i], sh.x);
        y[i + 1] = fmaf(sc.y, v[i + 1], sh.y);
        y[i + 2] = fmaf(sc.z, v[i + 2], sh.z);
        y[i + 3] = fmaf(sc.w, v[i + 3], sh.w);
      }
    }
  } else if (e.kind == OSAM_EPI_BIAS) {
#pragma unroll
    for (int i = 0; i < W; i += 4) {
      const float4 b = *reinterpret_cast<const float4*>(s_sh + col + i);
      y[i] += b.x;
      y[i + 1] += b.y;
      y[i + 2] += b.z;
      y[i + 3] += b.w;
    }
  }
  // the stage is free once the previous pass's tensor store has read it
  if (lane == 0) bulk_wait_group_read0();
  __syncwarp();
  if (e.kind == OSAM_EPI_BN_ACT && e.res && rsm) {
#pragma unroll
    for (int ch = 0; ch < CPR; ch++) {
      float r8[8];
      unpack8h(*reinterpret_cast<const uint4*>(rsm + stage_off(lane, ch)), r8);
#pragma unroll
      for (int i = 0; i < 8; i++) y[ch * 8 + i] += r8[i];
    }
  } else if (e.kind == OSAM_EPI_BN_ACT && e.res) {
    const int my_rv = valid ? (n * P + p) * Q + q : -1;
#pragma unroll
    for (int it = 0; it < CPR; it++) {
      const int rr = it * RPI + lane / CPR, ch = lane % CPR;
      uint4 val = make_uint4(0, 0, 0, 0);
      if (rreg) {
        val = rreg[it];
      } else {
        const int rpix = __shfl_sync(0xffffffffu, my_rv, rr);
        if (rpix >= 0) val = *reinterpret_cast<const uint4*>(e.res + (long long)rpix * K + col + ch * 8);
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
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (e.shuffle || e.par) {
      const int blk = e.par ? e.par - 1 : col / e.kout;
      tma_store_4d(&maps.m[blk], stage, e.par ? col : col - blk * e.kout, bq, bp, bn);
    } else {
#pragma unroll
      for (int t = 0; t < OSAM_MAX_DEST; t++) {
        if (t >= e.ndest) break;
        const DestDev& ds = e.dest[t];
        if (col < ds.c0 || col >= ds.c1) continue;
        const int kk = ds.choff + col - ds.c0;
        if (ds.up == 1) {
          tma_store_4d(&maps.m[4 * t], stage, kk, bq, bp, bn);
        } else {
#pragma unroll
          for (int vw = 0; vw < 4; vw++) tma_store_4d(&maps.m[4 * t + vw], stage, kk, bq, bp, bn);
        }
      }
    }
    bulk_commit_group();
  }
}

// The residual of a warp's 32 rows × 32 channels from column `col` on, in the coalesced order
// epilogue_warp_tma stages it (lane l holds row 8·it + l/4, channels 8·(l%4)…+7 in rv[it]); `my_pix` is
// this lane's own row's pixel, −1 outside the output.  Issued before the accumulator is ready, so the
// loads overlap the MMAs instead of stalling the epilogue.
__device__ __forceinline__ void residual_rows(const EpiDev& e, long long my_pix, int K, int col, uint4 (&rv)[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int it = 0; it < 4; it++) {
    const long long rpix = __shfl_sync(0xffffffffu, my_pix, it * 8 + lane / 4);
    rv[it] = rpix >= 0 ? *reinterpret_cast<const uint4*>(e.res + rpix * K + col + (lane % 4) * 8) : make_uint4(0, 0, 0, 0);
  }
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
