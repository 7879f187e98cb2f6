// Training-mode BatchNorm + SiLU as standalone HBM passes, and the bias passes of the head convs.
//
// Replaces the reference's src/bn.cu (bn_forward_stats :311-322, bn_forward_apply :324-327,
// bn_backward :329-344, bn_eval_scale :306-309) and src/misc.cu (chan_sum :168-172, add_bias :174-177).
// The inference path never runs these: there BN is folded into the conv epilogue.  Training needs the
// batch statistics of z before it can normalise z, and the backward needs two reductions over the whole
// batch, so these stay separate passes over HBM.
//
// Layout: z, residuals, gradients are NHWC fp16 viewed as [M = N·H·W rows][C channels]; one thread owns
// 8 channels (one 16-byte vector) of a row, V = C/8 consecutive threads cover a row, so a warp reads
// 32·16 contiguous bytes.  Per-channel statistics are per-thread fp32 sums over the thread's rows, fp32
// sums over the CTA's row lanes in shared memory, then fp64 atomics into a per-call workspace; the CTA
// that arrives last turns the fp64 sums into the outputs and zeroes the workspace again for the next
// call.  Every CTA owns one contiguous chunk of rows, and each pass that re-reads a chunk right after a
// reduction over it (forward apply after statistics, backward apply after the gradient sums) walks the
// chunk from its end: the rows a CTA read last are the ones the 126 MB L2 still holds.
#include "conv_internal.h"
#include "epilogue.cuh"
#include "sm100.cuh"

namespace osam {
namespace {

constexpr int kBnT = 256;            // threads per CTA
constexpr int kBnMaxC = kBnT * 8;    // one 8-channel vector per thread per row at least
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// σ(y) = 1 / (1 + 2^(−y·log2 e)) on the MUFU unit; y is clamped at −80 so 1 + e^{−y} stays finite.
__device__ __forceinline__ float sigmoid_fast(float y) {
  return rcp_approx(1.f + ex2_approx(-kLog2e * fmaxf(y, -80.f)));
}

// Row r = n·H·W + h·W + w of an H×W map lands, in the 2H×2W map that its nearest 2× upsample fills, on
// the 2×2 block whose top-left pixel is 2·(2·(n·H + h)·W + w); with nh = r / W that is 4·nh·W + 2·(r − nh·W).
__device__ __forceinline__ long long up2_corner(long long r, int W) {
  const long long nh = r / W;
  return 4 * nh * W + 2 * (r - nh * W);
}

// A destination the forward wrote to, read back as a gradient source.  `g` is offset so that channel c
// of the producing conv sits at g[pixel·ctot + c] (g = buffer + choff − c0); it holds channels
// [c_lo, c_hi) of the producer, 2×2-upsampled when up = 2.
struct GradSrc {
  const __half* g;
  int ctot, c_lo, c_hi, up;
};

// dA for channels c..c+7 of row r: the sum over every gradient source that holds those channels; an
// upsampled source contributes the four pixels of its 2×2 block.
__device__ __forceinline__ void dest_grad_sum8(const GradSrc* srcs, int n, long long r, int c, int W,
                                               float (&dA)[8]) {
#pragma unroll
  for (int i = 0; i < 8; i++) dA[i] = 0.f;
  long long corner = -1;
#pragma unroll
  for (int k = 0; k < OSAM_MAX_DEST; k++) {
    if (k >= n) break;
    const GradSrc sk = srcs[k];
    if (c < sk.c_lo || c >= sk.c_hi) continue;
    const __half* base = sk.g + c;
    const long long pitch = sk.ctot;
    float t[8];
    if (sk.up == 1) {
      ld8h(base + r * pitch, t);
#pragma unroll
      for (int i = 0; i < 8; i++) dA[i] += t[i];
      continue;
    }
    if (corner < 0) corner = up2_corner(r, W);
#pragma unroll
    for (int dy = 0; dy < 2; dy++)
#pragma unroll
      for (int dx = 0; dx < 2; dx++) {
        ld8h(base + (corner + dy * 2LL * W + dx) * pitch, t);
#pragma unroll
        for (int i = 0; i < 8; i++) dA[i] += t[i];
      }
  }
}

__device__ __forceinline__ void ld8f(const float* p, float (&o)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
  o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
// Per-channel parameters may sit anywhere in a parameter arena: 4-byte alignment only.
__device__ __forceinline__ void ld8f_any(const float* p, float (&o)[8]) {
#pragma unroll
  for (int i = 0; i < 8; i++) o[i] = p[i];
}

enum RedMode : int { RED_STATS = 0, RED_BWD = 1, RED_SUM = 2 };

// Programmatic dependent launch: the BN passes are launched with the programmatic-serialization attribute,
// so their CTAs are scheduled while the previous kernel of the stream drains; every thread waits for that
// kernel (and so for all earlier work) before its first global access, then lets the next kernel of the
// stream be scheduled in turn (it waits for this one the same way before touching memory).
__device__ __forceinline__ void bn_pdl_entry() {
  grid_dep_wait();
  grid_dep_launch();
}

// The rows a pass walks: z as [M][C] (W = the map's width, for upsampled destinations); each CTA owns
// `chunk` consecutive rows and processes `lanes` of them side by side (kBnT / (C/8) threads per row).
struct Rows {
  const __half* z;
  long long M, chunk;
  int W, C, lanes;
};
// Cross-CTA reduction state: fp64 sums [2C] and an arrival count, zero between calls.
// `copies` interleaved copies of the sums, [copies][2C] (CTA b adds into copy b % copies), so that fewer
// CTAs' atomics meet at one address; the finalising CTA adds the copies in a fixed order.
struct Accum {
  double* acc;
  unsigned* arrivals;
  int copies;
};
// RED_STATS: batch statistics in, the normalisation and the running statistics out.
struct StatsIO {
  const float* gamma;
  const float* beta;
  float momentum, eps;
  float* run_mean;
  float* run_var;
  float* mean;
  float* istd;
  float* scale;
  float* shift;
};
// RED_BWD: what the forward used, where the gradients come from, where the sums go.
struct BwdIO {
  const float* mean;
  const float* istd;
  const float* scale;
  const float* shift;
  GradSrc src[OSAM_MAX_DEST];
  int nsrc, silu, accum;
  float* gmean;  // [2C] Σg/M, Σg·x̂/M for the apply pass
  float* d_gamma;
  float* d_beta;
};
// RED_SUM: per-channel sums (=|+=) into out.
struct SumIO {
  float* out;
  int accum;
};
struct RedArgs {
  Rows rows;
  Accum red;
  StatsIO st;
  BwdIO bw;
  SumIO sum;
};

// Per-channel reductions over the rows of z (reference k_reduce<0|1>, src/bn.cu:112-202, and
// chan_sum, src/misc.cu:103-113, :168-172):
//   RED_STATS: Σ(z−K), Σ(z−K)² with K = running mean (shifted sums: no cancellation when |mean| ≫ std)
//   RED_BWD:   Σg, Σg·x̂ with g = dA·silu'(y), y = scale·z + shift, x̂ = (z − mean)·istd
//   RED_SUM:   Σz
// SIMPLE (RED_BWD): one destination, not upsampled, all channels — dA is one 16-byte load per row, kept raw.
// The thread's per-channel constants: RED_STATS k0 = K; RED_BWD k0 = scale, k1 = shift, k2 = istd,
// k3 = −mean·istd (x̂ = z·k2 + k3).
template <int MODE>
__device__ __forceinline__ void red_consts(const RedArgs& P, int c, float (&k0)[8], float (&k1)[8], float (&k2)[8],
                                           float (&k3)[8]) {
  if (MODE == RED_STATS) ld8f_any(P.st.run_mean + c, k0);
  if (MODE == RED_BWD) {
    float mu[8];
    ld8f_any(P.bw.scale + c, k0);
    ld8f_any(P.bw.shift + c, k1);
    ld8f_any(P.bw.istd + c, k2);
    ld8f_any(P.bw.mean + c, mu);
#pragma unroll
    for (int i = 0; i < 8; i++) k3[i] = -mu[i] * k2[i];
  }
}

// The thread's partial sums (a, b) over rows r0 + rl, r0 + rl + RL, … of its CTA's chunk [r0, r1).
template <int MODE, int U, bool SIMPLE>
__device__ __forceinline__ void red_rows(const RedArgs& P, long long r0, long long r1, int rl, int c,
                                         const float (&k0)[8], const float (&k1)[8], const float (&k2)[8],
                                         const float (&k3)[8], float (&a)[8], float (&b)[8]) {
  const Rows R = P.rows;
  const int C = R.C, RL = R.lanes;
#pragma unroll
  for (int i = 0; i < 8; i++) a[i] = b[i] = 0.f;
  for (long long r = r0 + rl; r < r1; r += (long long)U * RL) {
    uint4 zr[U], gr[SIMPLE ? U : 1];
    float dA[SIMPLE ? 1 : U][8];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const long long rr = r + (long long)u * RL;
      if (rr < r1) {
        zr[u] = *reinterpret_cast<const uint4*>(R.z + rr * C + c);
        if (SIMPLE) gr[u] = *reinterpret_cast<const uint4*>(P.bw.src[0].g + rr * P.bw.src[0].ctot + c);
      }
    }
    if (MODE == RED_BWD && !SIMPLE) {
#pragma unroll
      for (int u = 0; u < U; u++) {
        const long long rr = r + (long long)u * RL;
        if (rr < r1) dest_grad_sum8(P.bw.src, P.bw.nsrc, rr, c, R.W, dA[SIMPLE ? 0 : u]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (r + (long long)u * RL >= r1) break;
      float v[8];
      unpack8h(zr[u], v);
      if (SIMPLE) unpack8h(gr[u], dA[0]);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        if (MODE == RED_STATS) {
          const float d = v[i] - k0[i];
          a[i] += d;
          b[i] = fmaf(d, d, b[i]);
        } else if (MODE == RED_BWD) {
          float g = dA[SIMPLE ? 0 : u][i];
          if (P.bw.silu) {
            const float y = fmaf(k0[i], v[i], k1[i]), s = sigmoid_fast(y);
            g *= s * fmaf(y, 1.f - s, 1.f);
          }
          a[i] += g;
          b[i] = fmaf(g, fmaf(v[i], k2[i], k3[i]), b[i]);
        } else {
          a[i] += v[i];
        }
      }
    }
  }
}

// The CTA's sums of (a, b) per channel (shared memory, [row lanes][C]) added into the fp64 accumulators.
template <int MODE>
__device__ __forceinline__ void red_flush(const RedArgs& P, float2* bn_red, int rl, int c, bool active,
                                          const float (&a)[8], const float (&b)[8]) {
  const int C = P.rows.C, RL = P.rows.lanes;
  if (active) {
#pragma unroll
    for (int i = 0; i < 8; i++) bn_red[rl * C + c + i] = make_float2(a[i], b[i]);
  }
  __syncthreads();
  double* acc = P.red.acc + (size_t)(blockIdx.x % P.red.copies) * (MODE == RED_SUM ? C : 2 * C);
  for (int ch = threadIdx.x; ch < C; ch += kBnT) {
    float sa = 0.f, sb = 0.f;
    for (int k = 0; k < RL; k++) {
      const float2 t = bn_red[k * C + ch];
      sa += t.x;
      sb += t.y;
    }
    atomicAdd(&acc[ch], double(sa));
    if (MODE != RED_SUM) atomicAdd(&acc[C + ch], double(sb));
  }
}

// Batch statistics of one channel from its shifted sums: mean = K + E[z−K]; biased variance
// E[(z−K)²] − E[z−K]² (clamped at 0) for normalising; the running variance takes the unbiased M/(M−1)
// form (reference src/bn.cu:176-191).
struct ChanStats {
  float mean, istd, var, scale, shift;
};
__device__ __forceinline__ ChanStats stats_from_sums(double sx, double sy, double Md, float K, float gamma,
                                                     float beta, float eps) {
  ChanStats s;
  const float dm = float(sx / Md);
  float var = float(sy / Md - double(dm) * double(dm));
  var = var < 0.f ? 0.f : var;
  s.var = var;
  s.mean = K + dm;
  s.istd = rsqrtf(var + eps);
  s.scale = gamma * s.istd;
  s.shift = beta - s.mean * s.scale;
  return s;
}
__device__ __forceinline__ void stats_store(const StatsIO& S, int ch, float K, const ChanStats& s, double Md) {
  S.mean[ch] = s.mean;
  S.istd[ch] = s.istd;
  S.scale[ch] = s.scale;
  S.shift[ch] = s.shift;
  if (S.momentum > 0.f) {
    S.run_mean[ch] = (1.f - S.momentum) * K + S.momentum * s.mean;
    S.run_var[ch] = (1.f - S.momentum) * S.run_var[ch] + S.momentum * float(double(s.var) * Md / (Md - 1.0));
  }
}

template <int MODE, int U, bool SIMPLE = false>
__global__ void __launch_bounds__(kBnT, MODE == RED_BWD ? 2 : 3) k_bn_reduce(const RedArgs P) {
  extern __shared__ float2 bn_red[];  // [rowlanes][C]
  __shared__ unsigned s_last;
  bn_pdl_entry();
  const Rows R = P.rows;
  const int C = R.C, V = C >> 3, RL = R.lanes;
  const int rl = threadIdx.x / V, c = (threadIdx.x - rl * V) * 8;
  const bool active = rl < RL;
  const long long r0 = (long long)blockIdx.x * R.chunk;
  const long long r1 = r0 + R.chunk < R.M ? r0 + R.chunk : R.M;
  float a[8], b[8];
  if (active) {
    float k0[8], k1[8], k2[8], k3[8];
    red_consts<MODE>(P, c, k0, k1, k2, k3);
    red_rows<MODE, U, SIMPLE>(P, r0, r1, rl, c, k0, k1, k2, k3, a, b);
  }
  red_flush<MODE>(P, bn_red, rl, c, active, a, b);
  // The last CTA to arrive finalises (threadfence reduction: every CTA's atomics are visible before its
  // arrival on the counter).
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(P.red.arrivals, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const double Md = double(R.M);
  const int stride = MODE == RED_SUM ? C : 2 * C;
  for (int ch = threadIdx.x; ch < C; ch += kBnT) {
    double sx = 0.0, sy = 0.0;
    for (int g = 0; g < P.red.copies; g++) {
      double* acc = P.red.acc + (size_t)g * stride;
      sx += __ldcg(&acc[ch]);
      acc[ch] = 0.0;
      if (MODE != RED_SUM) {
        sy += __ldcg(&acc[C + ch]);
        acc[C + ch] = 0.0;
      }
    }
    if (MODE == RED_STATS) {
      const StatsIO S = P.st;
      const float K = S.run_mean[ch];
      stats_store(S, ch, K, stats_from_sums(sx, sy, Md, K, S.gamma[ch], S.beta[ch], S.eps), Md);
    } else if (MODE == RED_BWD) {
      const BwdIO G = P.bw;
      G.gmean[ch] = float(sx / Md);
      G.gmean[C + ch] = float(sy / Md);
      G.d_beta[ch] = G.accum ? G.d_beta[ch] + float(sx) : float(sx);
      G.d_gamma[ch] = G.accum ? G.d_gamma[ch] + float(sy) : float(sy);
    } else {
      P.sum.out[ch] = P.sum.accum ? P.sum.out[ch] + float(sx) : float(sx);
    }
  }
  if (threadIdx.x == 0) *P.red.arrivals = 0u;
}

struct ApplyArgs {
  Rows rows;
  const float* scale;
  const float* shift;
  const __half* res;  // [M][C] added after the activation, or null
  DestDev dest[OSAM_MAX_DEST];
  int ndest, silu;
};

// a = act(scale·z + shift) (+ res) → every destination, for the thread's rows of [r0, r1), walked from
// the chunk's end (reference k_apply, src/bn.cu:204-238).
template <int U>
__device__ __forceinline__ void apply_rows(const ApplyArgs& P, long long r0, long long r1, int rl, int c,
                                           const float (&sc)[8], const float (&sh)[8]) {
  const Rows R = P.rows;
  const int C = R.C, RL = R.lanes;
  for (long long r = r1 - 1 - rl; r >= r0; r -= (long long)U * RL) {
    uint4 zr[U], rr4[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const long long rr = r - (long long)u * RL;
      if (rr >= r0) {
        zr[u] = *reinterpret_cast<const uint4*>(R.z + rr * C + c);
        if (P.res) rr4[u] = *reinterpret_cast<const uint4*>(P.res + rr * C + c);
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const long long rr = r - (long long)u * RL;
      if (rr < r0) break;
      float o[8], rv[8];
      unpack8h(zr[u], o);
      if (P.res) unpack8h(rr4[u], rv);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const float y = fmaf(sc[i], o[i], sh[i]);
        o[i] = P.silu ? y * sigmoid_fast(y) : y;
        if (P.res) o[i] += rv[i];
      }
#pragma unroll 1
      for (int k = 0; k < OSAM_MAX_DEST; k++) {
        if (k >= P.ndest) break;
        const DestDev& d = P.dest[k];
        if (c < d.c0 || c >= d.c1) continue;
        const int cc = d.choff + c - d.c0;
        if (d.up == 1) {
          st8h(d.p + rr * d.ctot + cc, o);
        } else {
          const long long q = up2_corner(rr, R.W);
#pragma unroll
          for (int dy = 0; dy < 2; dy++)
#pragma unroll
            for (int dx = 0; dx < 2; dx++) st8h(d.p + (q + dy * 2LL * R.W + dx) * d.ctot + cc, o);
        }
      }
    }
  }
}

template <int U>
__global__ void __launch_bounds__(kBnT, 3) k_bn_apply(const ApplyArgs P) {
  bn_pdl_entry();
  const Rows R = P.rows;
  const int V = R.C >> 3;
  const int rl = threadIdx.x / V, c = (threadIdx.x - rl * V) * 8;
  if (rl >= R.lanes) return;
  const long long r0 = (long long)blockIdx.x * R.chunk;
  const long long r1 = r0 + R.chunk < R.M ? r0 + R.chunk : R.M;
  float sc[8], sh[8];
  ld8f_any(P.scale + c, sc);
  ld8f_any(P.shift + c, sh);
  apply_rows<U>(P, r0, r1, rl, c, sc, sh);
}

struct BwdArgs {
  Rows rows;
  const float* mean;
  const float* istd;
  const float* scale;
  const float* shift;
  const float* gmean;  // [2C] from the reduction pass
  GradSrc src[OSAM_MAX_DEST];
  int nsrc, silu;
  __half* dz;
  __half* res_grad;
  int res_accum;
};

// dz = scale·g + ka·z + kb with ka = −scale·istd·m2, kb = scale·(istd·m2·mean − m1), m1 = Σg/M, m2 = Σg·x̂/M.
__device__ __forceinline__ void bwd_consts(const BwdArgs& P, int c, const float (&m1)[8], const float (&m2)[8],
                                           float (&sc)[8], float (&sh)[8], float (&ka)[8], float (&kb)[8]) {
  float mu[8], is[8];
  ld8f_any(P.scale + c, sc);
  ld8f_any(P.shift + c, sh);
  ld8f_any(P.mean + c, mu);
  ld8f_any(P.istd + c, is);
#pragma unroll
  for (int i = 0; i < 8; i++) {
    ka[i] = -sc[i] * is[i] * m2[i];
    kb[i] = sc[i] * (is[i] * m2[i] * mu[i] - m1[i]);
  }
}

// dz = scale·(g − mean(g) − x̂·mean(g·x̂)); res_grad (=|+=) dA, for the thread's rows of [r0, r1) walked
// from the chunk's end (reference k_bwd_apply, src/bn.cu:240-270).
template <int U, bool SIMPLE>
__device__ __forceinline__ void bwd_apply_rows(const BwdArgs& P, long long r0, long long r1, int rl, int c,
                                               const float (&sc)[8], const float (&sh)[8], const float (&ka)[8],
                                               const float (&kb)[8]) {
  const Rows R = P.rows;
  const int C = R.C, RL = R.lanes;
  for (long long r = r1 - 1 - rl; r >= r0; r -= (long long)U * RL) {
    uint4 zr[U], gr[SIMPLE ? U : 1];
    float dAf[SIMPLE ? 1 : U][8];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const long long rr = r - (long long)u * RL;
      if (rr >= r0) {
        zr[u] = *reinterpret_cast<const uint4*>(R.z + rr * C + c);
        if (SIMPLE)
          gr[u] = *reinterpret_cast<const uint4*>(P.src[0].g + rr * P.src[0].ctot + c);
        else
          dest_grad_sum8(P.src, P.nsrc, rr, c, R.W, dAf[SIMPLE ? 0 : u]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const long long rr = r - (long long)u * RL;
      if (rr < r0) break;
      const long long off = rr * C + c;
      float (&dA)[8] = dAf[SIMPLE ? 0 : u];
      if (SIMPLE) unpack8h(gr[u], dA);
      if (P.res_grad) {
        float t[8];
        if (P.res_accum) {
          ld8h(P.res_grad + off, t);
#pragma unroll
          for (int i = 0; i < 8; i++) t[i] += dA[i];
        } else {
#pragma unroll
          for (int i = 0; i < 8; i++) t[i] = dA[i];
        }
        st8h(P.res_grad + off, t);
      }
      float v[8];
      unpack8h(zr[u], v);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        float g = dA[i];
        if (P.silu) {
          const float y = fmaf(sc[i], v[i], sh[i]), s = sigmoid_fast(y);
          g *= s * fmaf(y, 1.f - s, 1.f);
        }
        v[i] = fmaf(sc[i], g, fmaf(ka[i], v[i], kb[i]));
      }
      st8h(P.dz + off, v);
    }
  }
}

template <int U, bool SIMPLE = false>
__global__ void __launch_bounds__(kBnT, 2) k_bn_bwd_apply(const BwdArgs P) {
  bn_pdl_entry();
  const Rows R = P.rows;
  const int C = R.C, V = C >> 3;
  const int rl = threadIdx.x / V, c = (threadIdx.x - rl * V) * 8;
  if (rl >= R.lanes) return;
  const long long r0 = (long long)blockIdx.x * R.chunk;
  const long long r1 = r0 + R.chunk < R.M ? r0 + R.chunk : R.M;
  float m1[8], m2[8], sc[8], sh[8], ka[8], kb[8];
  ld8f(P.gmean + c, m1);
  ld8f(P.gmean + C + c, m2);
  bwd_consts(P, c, m1, m2, sc, sh, ka, kb);
  bwd_apply_rows<U, SIMPLE>(P, r0, r1, rl, c, sc, sh, ka, kb);
}

// Σ over rows of x for channel counts that are not a multiple of 8 (the 1-channel class head): every
// element goes to shared-memory channel sums, then to the fp64 accumulators; last CTA finalises.
__global__ void __launch_bounds__(kBnT) k_chan_sum_any(const __half* __restrict__ x, long long n, int C,
                                                        long long per_cta, float* out, int accum, double* acc,
                                                        unsigned* counter) {
  extern __shared__ float s_sum[];  // [C]
  __shared__ unsigned s_last;
  for (int ch = threadIdx.x; ch < C; ch += kBnT) s_sum[ch] = 0.f;
  __syncthreads();
  const long long e0 = (long long)blockIdx.x * per_cta;
  const long long e1 = e0 + per_cta < n ? e0 + per_cta : n;
  float run = 0.f;
  int run_ch = -1;
  for (long long e = e0 + threadIdx.x; e < e1; e += kBnT) {
    const int ch = int(e % C);
    const float v = __half2float(x[e]);
    if (ch == run_ch) {
      run += v;
    } else {
      if (run_ch >= 0) atomicAdd(&s_sum[run_ch], run);
      run_ch = ch;
      run = v;
    }
  }
  if (run_ch >= 0) atomicAdd(&s_sum[run_ch], run);
  __syncthreads();
  for (int ch = threadIdx.x; ch < C; ch += kBnT) atomicAdd(&acc[ch], double(s_sum[ch]));
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int ch = threadIdx.x; ch < C; ch += kBnT) {
    const double s = __ldcg(&acc[ch]);
    acc[ch] = 0.0;
    out[ch] = accum ? out[ch] + float(s) : float(s);
  }
  if (threadIdx.x == 0) *counter = 0u;
}

// y += bias per channel, fp32 add then one fp16 rounding (reference k_add_bias8 / k_add_bias,
// src/misc.cu:116-134).
__global__ void __launch_bounds__(kBnT) k_add_bias8(__half* __restrict__ y, long long nvec, int C,
                                                     const float* __restrict__ bias) {
  const int V = C >> 3;
  for (long long i = (long long)blockIdx.x * kBnT + threadIdx.x; i < nvec; i += (long long)gridDim.x * kBnT) {
    const int c = int(i % V) * 8;
    float v[8], b[8];
    ld8h(y + i * 8, v);
    ld8f_any(bias + c, b);
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] += b[k];
    st8h(y + i * 8, v);
  }
}
__global__ void __launch_bounds__(kBnT) k_add_bias1(__half* __restrict__ y, long long n, int C,
                                                     const float* __restrict__ bias) {
  for (long long i = (long long)blockIdx.x * kBnT + threadIdx.x; i < n; i += (long long)gridDim.x * kBnT)
    y[i] = __float2half(__half2float(y[i]) + bias[i % C]);
}

// Eval-mode fold: scale = γ/√(var+eps), shift = β − μ·scale (reference k_eval_scale, src/bn.cu:277-284).
__global__ void k_bn_eval_scale(int C, const float* g, const float* b, const float* rm, const float* rv, float eps,
                                float* scale, float* shift) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const float sc = g[c] * rsqrtf(rv[c] + eps);
  scale[c] = sc;
  shift[c] = b[c] - rm[c] * sc;
}

// ------------------------------------------------------------------ host side
constexpr int kUStats = 4, kUBwd = 2, kUApply = 4, kUBwdApply = 2, kUBwdSimple = 4;

int g_sms_cache[64] = {};
int g_occ_cache[64][3] = {};

template <class K>
int occupancy(K kernel, size_t smem) {
  int occ = 0;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kBnT, smem) == cudaSuccess && occ > 0 ? occ : 1;
}

// CTAs that are resident at once for a pass pair — mode 0: statistics (or channel sums) and the forward
// apply; mode 1: the backward sums and the backward apply; mode 2: the same for a single plain destination —
// so that both kernels of a pair run as one wave over the same row chunks.
int resident_ctas(int mode) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148 * 2;
  if (!g_sms_cache[dev]) {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    g_sms_cache[dev] = sms > 0 ? sms : 148;
  }
  if (!g_occ_cache[dev][mode]) {
    const size_t smem = size_t(kBnT) * 8 * sizeof(float2);
    int a, b;
    if (mode == 0) {
      a = occupancy(k_bn_reduce<RED_STATS, kUStats>, smem);
      b = occupancy(k_bn_apply<kUApply>, 0);
    } else if (mode == 1) {
      a = occupancy(k_bn_reduce<RED_BWD, kUBwd>, smem);
      b = occupancy(k_bn_bwd_apply<kUBwdApply>, 0);
    } else {
      a = occupancy(k_bn_reduce<RED_BWD, kUBwdSimple, true>, smem);
      b = occupancy(k_bn_bwd_apply<kUBwdSimple, true>, 0);
    }
    g_occ_cache[dev][mode] = a < b ? a : b;
  }
  return g_sms_cache[dev] * g_occ_cache[dev][mode];
}

struct Chunking {
  int rowlanes, nblk;
  long long rows;
};
// One contiguous chunk of rows per CTA, at most one resident wave, at least two row iterations per thread.
Chunking chunking(long long M, int C, int mode) {
  Chunking k;
  k.rowlanes = kBnT / (C / 8);
  const long long target = resident_ctas(mode);
  long long rows = (M + target - 1) / target;
  const long long min_rows = 2LL * k.rowlanes;
  if (rows < min_rows) rows = min_rows;
  k.rows = rows;
  k.nblk = int((M + rows - 1) / rows);
  return k;
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int bad(int code, const char* what) {
  set_last_error("%s", what);
  return code;
}

struct BnWs {
  double* acc;
  unsigned* counter;
  float* sums;
};
// BN workspace: kBnCopies × [2C] fp64 sums, the arrival counter (16 bytes), the backward's [2C] fp32 means.
constexpr int kBnCopies = 8;
size_t bn_ws_bytes(int C) { return ((size_t(C) * (16 * kBnCopies + 8) + 16) + 255) / 256 * 256; }
BnWs bn_ws(void* ws, int C) {
  char* p = static_cast<char*>(ws);
  BnWs w;
  w.acc = reinterpret_cast<double*>(p);
  w.counter = reinterpret_cast<unsigned*>(p + size_t(C) * 16 * kBnCopies);
  w.sums = reinterpret_cast<float*>(p + size_t(C) * 16 * kBnCopies + 16);
  return w;
}

int check_shape(const void* z, int N, int H, int W, int C) {
  if (!z || N < 1 || H < 1 || W < 1) return bad(OSAM_ERR_INVALID, "bn: empty tensor");
  if (C < 8 || C % 8 || C > kBnMaxC) return bad(OSAM_ERR_INVALID, "bn: channels must be a multiple of 8 in [8, 2048]");
  if (!al16(z)) return bad(OSAM_ERR_INVALID, "bn: tensor not 16-byte aligned");
  if ((long long)N * H * W >= (1LL << 40)) return bad(OSAM_ERR_INVALID, "bn: tensor too large");
  return OSAM_OK;
}

// Launch with the programmatic-serialization attribute (the kernels call bn_pdl_entry first).
template <typename... KArgs, typename... Args>
void pdl_launch(void (*kernel)(KArgs...), int grid, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kBnT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, args...);
}

int launched(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("%s launch: %s", what, cudaGetErrorString(e));
    return OSAM_ERR_CUDA;
  }
  return OSAM_OK;
}

}  // namespace
}  // namespace osam

using namespace osam;

extern "C" {

size_t osam_bn_workspace_size(int C) { return C > 0 ? bn_ws_bytes(C) : 0; }

int osam_bn_eval_scale(int C, const float* gamma, const float* beta, const float* run_mean, const float* run_var,
                       float eps, float* scale, float* shift, osam_stream_t stream) {
  if (C < 1 || !gamma || !beta || !run_mean || !run_var || !scale || !shift)
    return bad(OSAM_ERR_INVALID, "bn_eval_scale arguments");
  k_bn_eval_scale<<<(C + 127) / 128, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(C, gamma, beta, run_mean,
                                                                                        run_var, eps, scale, shift);
  return launched("osam_bn_eval_scale");
}

int osam_bn_forward_stats(const void* z, int N, int H, int W, int C, const float* gamma, const float* beta,
                          float* run_mean, float* run_var, float momentum, float eps, float* mean, float* istd,
                          float* scale, float* shift, void* ws, size_t ws_bytes, osam_stream_t stream) {
  int rc = check_shape(z, N, H, W, C);
  if (rc) return rc;
  if (!gamma || !beta || !run_mean || !run_var || !mean || !istd || !scale || !shift)
    return bad(OSAM_ERR_INVALID, "bn_forward_stats: null parameter");
  const long long M = (long long)N * H * W;
  if (M < 2) return bad(OSAM_ERR_INVALID, "bn_forward_stats: batch statistics need at least 2 values per channel");
  if (!ws || ws_bytes < bn_ws_bytes(C) || !al16(ws)) return bad(OSAM_ERR_INVALID, "bn_forward_stats: workspace");
  const Chunking k = chunking(M, C, 0);
  const BnWs w = bn_ws(ws, C);
  RedArgs P{};
  P.rows = Rows{static_cast<const __half*>(z), M, k.rows, W, C, k.rowlanes};
  P.red = Accum{w.acc, w.counter, kBnCopies};
  P.st = StatsIO{gamma, beta, momentum, eps, run_mean, run_var, mean, istd, scale, shift};
  const size_t smem = size_t(k.rowlanes) * C * sizeof(float2);
  pdl_launch(k_bn_reduce<RED_STATS, kUStats>, k.nblk, smem, reinterpret_cast<cudaStream_t>(stream), P);
  return launched("osam_bn_forward_stats");
}

int osam_bn_forward_apply(const void* z, int N, int H, int W, int C, const float* scale, const float* shift,
                          const void* res, const osam_dest* dests, int n_dest, int act, osam_stream_t stream) {
  int rc = check_shape(z, N, H, W, C);
  if (rc) return rc;
  if (!scale || !shift) return bad(OSAM_ERR_INVALID, "bn_forward_apply: null scale/shift");
  if (n_dest < 1 || n_dest > OSAM_MAX_DEST || !dests) return bad(OSAM_ERR_INVALID, "bn_forward_apply: 1..4 dests");
  if (res && !al16(res)) return bad(OSAM_ERR_INVALID, "bn_forward_apply: residual not 16-byte aligned");
  const long long M = (long long)N * H * W;
  const Chunking k = chunking(M, C, 0);
  ApplyArgs P{};
  P.rows = Rows{static_cast<const __half*>(z), M, k.rows, W, C, k.rowlanes};
  P.scale = scale;
  P.shift = shift;
  P.res = static_cast<const __half*>(res);
  P.ndest = n_dest;
  P.silu = act ? 1 : 0;
  for (int i = 0; i < n_dest; i++) {
    const osam_dest& d = dests[i];
    const int c1 = d.c1 > 0 ? d.c1 : C;
    if (!d.p || !al16(d.p) || d.c0 < 0 || d.c0 % 8 || c1 % 8 || c1 > C || d.c0 >= c1 || d.choff < 0 ||
        d.choff % 8 || d.ctot % 8 || d.choff + (c1 - d.c0) > d.ctot || (d.up != 1 && d.up != 2))
      return bad(OSAM_ERR_INVALID, "bn_forward_apply: destination (16-byte aligned, channels multiple of 8)");
    P.dest[i] = DestDev{static_cast<__half*>(d.p), d.ctot, d.choff, d.c0, c1, d.up, 1};
  }
  pdl_launch(k_bn_apply<kUApply>, k.nblk, 0, reinterpret_cast<cudaStream_t>(stream), P);
  return launched("osam_bn_forward_apply");
}

int osam_bn_forward_train(const void* z, int N, int H, int W, int C, const float* gamma, const float* beta,
                          float* run_mean, float* run_var, float momentum, float eps, float* mean, float* istd,
                          float* scale, float* shift, const void* res, const osam_dest* dests, int n_dest, int act,
                          void* ws, size_t ws_bytes, osam_stream_t stream) {
  if (n_dest < 1 || n_dest > OSAM_MAX_DEST || !dests) return bad(OSAM_ERR_INVALID, "bn_forward_train: 1..4 dests");
  const int rc = osam_bn_forward_stats(z, N, H, W, C, gamma, beta, run_mean, run_var, momentum, eps, mean, istd, scale,
                                       shift, ws, ws_bytes, stream);
  return rc ? rc : osam_bn_forward_apply(z, N, H, W, C, scale, shift, res, dests, n_dest, act, stream);
}

int osam_bn_backward(const void* z, int N, int H, int W, int C, const float* mean, const float* istd,
                     const float* scale, const float* shift, const osam_dest* grad_dests, int n_dest, int act,
                     void* dz, float* gw_gamma, float* gw_beta, int accum, void* res_grad, int res_accum, void* ws,
                     size_t ws_bytes, osam_stream_t stream) {
  int rc = check_shape(z, N, H, W, C);
  if (rc) return rc;
  if (!mean || !istd || !scale || !shift || !gw_gamma || !gw_beta)
    return bad(OSAM_ERR_INVALID, "bn_backward: null parameter");
  if (!dz || !al16(dz)) return bad(OSAM_ERR_INVALID, "bn_backward: dz missing or not 16-byte aligned");
  if (res_grad && !al16(res_grad)) return bad(OSAM_ERR_INVALID, "bn_backward: res_grad not 16-byte aligned");
  if (n_dest < 1 || n_dest > OSAM_MAX_DEST || !grad_dests) return bad(OSAM_ERR_INVALID, "bn_backward: 1..4 dests");
  if (!ws || ws_bytes < bn_ws_bytes(C) || !al16(ws)) return bad(OSAM_ERR_INVALID, "bn_backward: workspace");
  const long long M = (long long)N * H * W;
  const bool simple = n_dest == 1 && grad_dests[0].up == 1 && grad_dests[0].c0 == 0 &&
                      (grad_dests[0].c1 == 0 || grad_dests[0].c1 == C);
  const Chunking k = chunking(M, C, simple ? 2 : 1);
  const BnWs w = bn_ws(ws, C);
  RedArgs P{};
  BwdArgs B{};
  for (int i = 0; i < n_dest; i++) {
    const osam_dest& d = grad_dests[i];
    const int c1 = d.c1 > 0 ? d.c1 : C;
    if (!d.p || !al16(d.p) || d.c0 < 0 || d.c0 % 8 || c1 % 8 || c1 > C || d.c0 >= c1 || d.choff < 0 ||
        d.choff % 8 || d.ctot % 8 || d.choff + (c1 - d.c0) > d.ctot || (d.up != 1 && d.up != 2))
      return bad(OSAM_ERR_INVALID, "bn_backward: gradient destination (16-byte aligned, channels multiple of 8)");
    P.bw.src[i] = B.src[i] = GradSrc{static_cast<const __half*>(d.p) + d.choff - d.c0, d.ctot, d.c0, c1, d.up};
  }
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  P.rows = B.rows = Rows{static_cast<const __half*>(z), M, k.rows, W, C, k.rowlanes};
  P.red = Accum{w.acc, w.counter, kBnCopies};
  P.bw.nsrc = B.nsrc = n_dest;
  P.bw.silu = B.silu = act ? 1 : 0;
  P.bw.mean = B.mean = mean;
  P.bw.istd = B.istd = istd;
  P.bw.scale = B.scale = scale;
  P.bw.shift = B.shift = shift;
  P.bw.gmean = w.sums;
  B.gmean = w.sums;
  P.bw.d_gamma = gw_gamma;
  P.bw.d_beta = gw_beta;
  P.bw.accum = accum ? 1 : 0;
  B.dz = static_cast<__half*>(dz);
  B.res_grad = static_cast<__half*>(res_grad);
  B.res_accum = res_accum ? 1 : 0;
  const size_t smem = size_t(k.rowlanes) * C * sizeof(float2);
  if (simple) {
    pdl_launch(k_bn_reduce<RED_BWD, kUBwdSimple, true>, k.nblk, smem, st, P);
    if ((rc = launched("osam_bn_backward (sums)"))) return rc;
    pdl_launch(k_bn_bwd_apply<kUBwdSimple, true>, k.nblk, 0, st, B);
    return launched("osam_bn_backward (apply)");
  }
  pdl_launch(k_bn_reduce<RED_BWD, kUBwd>, k.nblk, smem, st, P);
  if ((rc = launched("osam_bn_backward (sums)"))) return rc;
  pdl_launch(k_bn_bwd_apply<kUBwdApply>, k.nblk, 0, st, B);
  return launched("osam_bn_backward (apply)");
}

size_t osam_chan_sum_workspace_size(int C) { return C > 0 ? ((size_t(C) * 8 + 16) + 255) / 256 * 256 : 0; }

int osam_chan_sum(const void* x, int64_t M, int C, float* out, int accum, void* ws, size_t ws_bytes,
                  osam_stream_t stream) {
  if (!x || M < 1 || C < 1 || C > kBnMaxC || !out) return bad(OSAM_ERR_INVALID, "chan_sum arguments");
  if (!ws || ws_bytes < osam_chan_sum_workspace_size(C) || !al16(ws))
    return bad(OSAM_ERR_INVALID, "chan_sum: workspace");
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  double* acc = static_cast<double*>(ws);
  unsigned* counter = reinterpret_cast<unsigned*>(static_cast<char*>(ws) + size_t(C) * 8);
  if (C % 8 == 0 && al16(x)) {
    const Chunking k = chunking(M, C, 0);
    RedArgs P{};
    P.rows = Rows{static_cast<const __half*>(x), M, k.rows, 1, C, k.rowlanes};
    P.red = Accum{acc, counter, 1};
    P.sum = SumIO{out, accum ? 1 : 0};
    const size_t smem = size_t(k.rowlanes) * C * sizeof(float2);
    pdl_launch(k_bn_reduce<RED_SUM, kUStats>, k.nblk, smem, st, P);
  } else {
    const long long n = (long long)M * C;
    long long per = (n + resident_ctas(0) - 1) / resident_ctas(0);
    if (per < 8LL * kBnT) per = 8LL * kBnT;
    const int nblk = int((n + per - 1) / per);
    k_chan_sum_any<<<nblk, kBnT, size_t(C) * sizeof(float), st>>>(static_cast<const __half*>(x), n, C, per, out,
                                                                   accum ? 1 : 0, acc, counter);
  }
  return launched("osam_chan_sum");
}

int osam_add_bias(void* y, int64_t M, int C, const float* bias, osam_stream_t stream) {
  if (!y || M < 1 || C < 1 || !bias) return bad(OSAM_ERR_INVALID, "add_bias arguments");
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const long long n = (long long)M * C;
  const int grid = resident_ctas(0);
  if (C % 8 == 0 && al16(y)) {
    const long long nv = n / 8;
    const int g = int(nv / kBnT + 1 < grid ? nv / kBnT + 1 : grid);
    k_add_bias8<<<g, kBnT, 0, st>>>(static_cast<__half*>(y), nv, C, bias);
  } else {
    const int g = int(n / kBnT + 1 < grid ? n / kBnT + 1 : grid);
    k_add_bias1<<<g, kBnT, 0, st>>>(static_cast<__half*>(y), n, C, bias);
  }
  return launched("osam_add_bias");
}

}  // extern "C"
