// Training mask loss of the segment head: the coefficient × prototype contraction, per-pixel BCE against
// the ground-truth mask bits inside the cropped box, and the gradients of proto and of the positive
// anchors' mask coefficients.  Replaces the reference's mask part of SegLoss::run (src/loss.cu:393-543:
// k_mask_tile + k_mask_coef, launched at :613-619).
//
// For image b, positive i (anchor a_i with assigned ground truth j_i), proto pixel p inside i's crop:
//   z = coef_i · proto_p,  y = bit p of gt mask j_i,  loss += bce(z, y)·inv_i,  g = (σ(z) − y)·inv_i·gk
//   dproto_p += g·coef_i,   dcoef_i += g·proto_p
// with inv_i = 1/(Hp·Wp·area_i) (area of the box normalised to the image) and gk = box_gain·B/max(fg,1)·scale.
//
// On the tensor cores, one CTA per 16×8-pixel proto tile (128 pixels), positives overlapping the tile in
// batches of ≤ 96, three tcgen05 GEMMs per batch:
//   MMA1  Zᵀ[pixel][pos]   = Proto[pixel][32] · Coef[pos][32]ᵀ          (both K-major, 64-byte swizzle)
//   (epilogue warps: G'[pixel][pos] = σ(z) − y inside the crop, 0 outside → fp16, 128-byte swizzle; loss)
//   MMA2  dProto[pixel][32] += G'[pixel][pos] · CoefS[pos][32]          (A K-major, B MN-major)
//   MMA3  dCoef[pos][32]     = G'ᵀ[pos][pixel] · Proto[pixel][32]        (A and B MN-major: the same
//                                                                         shared-memory tiles read the other way)
// G' = σ(z) − y lies in (−1, 1), so fp16 keeps its precision; the per-positive scale s_i = inv_i·gk, which
// spans many decades, never enters an fp16 operand except as CoefS_i = coef_i·s_i·2^−E_b with E_b the
// exponent of the image's largest s_i (so CoefS ≤ |coef|), and 2^E_b is applied to dProto in fp32.
// dCoef blocks are scaled by s_i in fp32 and added into an fp32 workspace row per positive; a last pass
// writes them to the coef-gradient heads in fp16 and zeroes the rows again.
// Warps 0–3: overlap scan, operand gather, epilogues (thread = TMEM lane); warp 4: TMEM owner + MMA issuer.
// Every wait is bounded (sm100.cuh).
#include "conv_internal.h"
#include "sm100.cuh"

namespace osam {
namespace {

constexpr int kMlPos = 96;          // positives per batch (MMA1 N)
constexpr int kMlWorkers = 128;     // warps 0-3
constexpr int kMlThreads = kMlWorkers + 32;
constexpr int kMlListCap = kMlPos + kMlWorkers;
constexpr int kMlTmemCols = 128;    // Zᵀ in [0, 96) (dCoef reuses [0, 32)), dProto in [96, 128)
constexpr int kMlDProtoCol = 96;
constexpr int kMlTileW = 16, kMlTileH = 8;
// shared memory (dynamic, 1024-aligned): proto 8 KB | coef 8 KB | coefS 8 KB | G' 2 × 16 KB
constexpr int kMlProto = 0, kMlCoef = 8192, kMlCoefS = 16384, kMlG = 24576, kMlGBlock = 16384;
constexpr int kMlSmem = 1024 + kMlG + 2 * kMlGBlock;
constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;

struct MlMeta {  // one positive: crop box on the proto grid, 1/(Hp·Wp·area), gt index, coef head row
  float x1, y1, x2, y2, inv;
  int j, l, row;
};

struct MlArgs {
  const __half* coef[3];
  int lvl_h[3], lvl_w[3], off[4];
  const __half* proto;
  __half* dproto;
  __half* dcoef[3];
  int B, A, G, Hp, Wp, imgsz;
  const int* npos;
  const int* pos;
  const int* agt;
  const float4* gtb;
  const uint32_t* gmask;
  const float* fg;
  const float* scale;
  float box_gain;
  float* loss;
  MlMeta* meta;        // [B][A]
  int* smax;           // [B] float bits of max_i s_i
  float* acc;          // [B][A][32] dCoef rows (zero outside a call)
  int* err;
};

__device__ __forceinline__ float ml_gk(const MlArgs& P) {
  return P.box_gain * float(P.B) / fmaxf(*P.fg, 1.f) * *P.scale;
}

// Per positive: crop (reference crop_of, src/loss.cu:409-415), inv, head row; per image: max s_i.
__global__ void k_ml_meta(const MlArgs P) {
  const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= (long long)P.B * P.A) return;
  const int b = int(q / P.A), i = int(q - (long long)b * P.A);
  if (i >= P.npos[b]) return;
  const int a = P.pos[(long long)b * P.A + i];
  const int j = P.agt[(long long)b * P.A + a];
  const float4 tg = P.gtb[(long long)b * P.G + j];
  const float s = float(P.imgsz);
  const float nx1 = tg.x / s, ny1 = tg.y / s, nx2 = tg.z / s, ny2 = tg.w / s;
  const float area = (nx2 - nx1) * (ny2 - ny1);
  MlMeta m;
  m.x1 = nx1 * P.Wp;
  m.x2 = nx2 * P.Wp;
  m.y1 = ny1 * P.Hp;
  m.y2 = ny2 * P.Hp;
  m.inv = 1.f / (float(P.Hp) * float(P.Wp) * area);
  m.j = j;
  // level by range (ternaries: no dynamic indexing into the parameter block)
  const int l = a < P.off[1] ? 0 : (a < P.off[2] ? 1 : 2);
  const int lo = l == 0 ? 0 : (l == 1 ? P.off[1] : P.off[2]);
  const int lw = l == 0 ? P.lvl_w[0] : (l == 1 ? P.lvl_w[1] : P.lvl_w[2]);
  const int lh = l == 0 ? P.lvl_h[0] : (l == 1 ? P.lvl_h[1] : P.lvl_h[2]);
  const int r = a - lo, h = r / lw, w = r - h * lw;
  m.l = l;
  m.row = (b * lh + h) * lw + w;
  P.meta[q] = m;
  const float sv = m.inv * ml_gk(P);
  if (sv > 0.f) atomicMax(&P.smax[b], __float_as_int(sv));
}

__device__ __forceinline__ uint32_t sw64(int row, int chunk) { return row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4); }
__device__ __forceinline__ uint32_t sw128(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

__device__ __forceinline__ uint64_t desc_mn(uint32_t saddr, int row_bytes, uint32_t block_bytes) {
  uint64_t d = (saddr & 0x3FFFFu) >> 4;
  d |= uint64_t((block_bytes >> 4) & 0x3FFFu) << 16;       // LBO: next 64 (32) M/N elements
  d |= uint64_t(((8 * row_bytes) >> 4) & 0x3FFFu) << 32;   // SBO: next 8 reduction rows
  d |= uint64_t(1) << 46;
  d |= uint64_t(row_bytes == 128 ? 2 : 4) << 61;
  return d;
}
// kind::f16, fp32 D; a_mn / b_mn select MN-major A / B.
__host__ __device__ constexpr uint32_t ml_idesc(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) | (uint32_t(N >> 3) << 17) |
         (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ float ml_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float ml_lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float ml_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kMlThreads, 3) k_ml_tile(const MlArgs P) {
  extern __shared__ uint8_t ml_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ml_raw) + 1023) & ~uintptr_t(1023));
  __shared__ MlMeta s_pend[kMlListCap];
  __shared__ int s_pidx[kMlListCap];
  __shared__ int s_wcnt[4];
  __shared__ int s_nb;
  __shared__ uint32_t s_tmem;
  __shared__ __align__(8) uint64_t bar_in, bar_z, bar_g, bar_c;
  __shared__ float s_loss[4];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int tiles_x = P.Wp / kMlTileW;
  const int b = blockIdx.y, px0 = (blockIdx.x % tiles_x) * kMlTileW, py0 = (blockIdx.x / tiles_x) * kMlTileH;
  const int np = P.npos[b];

  if (tid == 0) {
    mbar_init(&bar_in, kMlWorkers);
    mbar_init(&bar_z, 1);
    mbar_init(&bar_g, kMlWorkers);
    mbar_init(&bar_c, 1);
    fence_barrier_init();
  }
  if (warp == 4) {
    tmem_alloc(&s_tmem, kMlTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const uint32_t sbase = smem_u32(sm);

  if (warp == 4) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      for (uint32_t batch = 0;; batch++) {
        if (!mbar_wait(&bar_in, batch & 1, P.err)) break;
        tc_fence_after();
        const int nb = s_nb;
        if (nb == 0) break;
        const int nb16 = (nb + 15) & ~15;
        const uint32_t i1 = ml_idesc(128, nb16, 0, 0);
#pragma unroll
        for (int k = 0; k < 2; k++)  // K = 32 channels
          umma_f16(tmem, smem_desc_kmajor(sbase + kMlProto + 32 * k, 64), smem_desc_kmajor(sbase + kMlCoef + 32 * k, 64),
                   i1, k);
        umma_commit(&bar_z);
        if (!mbar_wait(&bar_g, batch & 1, P.err)) break;
        tc_fence_after();
        constexpr uint32_t i2 = ml_idesc(128, 32, 0, 1), i3 = ml_idesc(128, 32, 1, 1);
        for (int s = 0; s < nb16 / 16; s++)  // K = positives, 16 per MMA
          umma_f16(tmem + kMlDProtoCol,
                   smem_desc_kmajor(sbase + kMlG + (s >> 2) * kMlGBlock + (s & 3) * 32, 128),
                   desc_mn(sbase + kMlCoefS + s * 16 * 64, 64, 8192), i2, (batch | s) != 0);
#pragma unroll
        for (int s = 0; s < 8; s++)  // K = 128 pixels, 16 per MMA
          umma_f16(tmem, desc_mn(sbase + kMlG + s * 16 * 128, 128, kMlGBlock), desc_mn(sbase + kMlProto + s * 16 * 64, 64, 8192),
                   i3, s);
        umma_commit(&bar_c);
      }
    }
  } else {
    // ------------------------------------------------------------------ workers (thread = TMEM lane)
    const int m = tid;  // pixel row of Zᵀ / dProto; positive row of dCoef
    const int mpx = px0 + (m & 15), mpy = py0 + (m >> 4);
    const float fpx = float(mpx), fpy = float(mpy);
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    // proto tile → shared memory (64-byte swizzled rows)
    {
      const uint4* src = reinterpret_cast<const uint4*>(P.proto + (((long long)b * P.Hp + mpy) * P.Wp + mpx) * 32);
#pragma unroll
      for (int c = 0; c < 4; c++) *reinterpret_cast<uint4*>(sm + kMlProto + sw64(m, c)) = src[c];
    }
    const float gk = ml_gk(P);
    int e_b = 0;
    if (np > 0) frexpf(__int_as_float(P.smax[b]), &e_b);  // s_i·2^−e_b < 1
    const int words = P.Hp * P.Wp / 32;
    float lsum = 0.f;
    int pend = 0, cand = 0;
    uint32_t batch = 0;
    bool ok = true;
    while (ok) {
      // ---- overlap scan: append positives whose crop meets the tile, in positive order
      while (pend < kMlPos && cand < np) {
        const int i = cand + m;
        bool hit = false;
        MlMeta mm;
        if (i < np) {
          mm = P.meta[(long long)b * P.A + i];
          hit = px0 + kMlTileW - 1 >= mm.x1 && px0 < mm.x2 && py0 + kMlTileH - 1 >= mm.y1 && py0 < mm.y2;
        }
        const unsigned bal = __ballot_sync(~0u, hit);
        if (lane == 0) s_wcnt[warp] = __popc(bal);
        named_bar_sync(1, kMlWorkers);
        int slot = pend + __popc(bal & ((1u << lane) - 1u)), tot = 0;
#pragma unroll
        for (int w = 0; w < 4; w++) {
          if (w < warp) slot += s_wcnt[w];
          tot += s_wcnt[w];
        }
        if (hit) {
          s_pend[slot] = mm;
          s_pidx[slot] = i;
        }
        named_bar_sync(1, kMlWorkers);
        pend += tot;
        cand += kMlWorkers;
      }
      const int nb = pend < kMlPos ? pend : kMlPos;
      const int nb16 = (nb + 15) & ~15;
      if (tid == 0) s_nb = nb;
      // ---- gather coef rows (K-major B of MMA1) and the scaled rows (MN-major B of MMA2)
      for (int it = m; it < nb16 * 4; it += kMlWorkers) {
        const int e = it >> 2, c = it & 3;
        uint4 u = make_uint4(0, 0, 0, 0), us = u;
        if (e < nb) {
          const MlMeta& mm = s_pend[e];
          const __half* cb = mm.l == 0 ? P.coef[0] : (mm.l == 1 ? P.coef[1] : P.coef[2]);
          u = reinterpret_cast<const uint4*>(cb + (long long)mm.row * 32)[c];
          const float ms = ldexpf(mm.inv * gk, -e_b);
          const __half2* h = reinterpret_cast<const __half2*>(&u);
          __half2* hs = reinterpret_cast<__half2*>(&us);
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const float2 f = __half22float2(h[q]);
            hs[q] = __floats2half2_rn(f.x * ms, f.y * ms);
          }
        }
        *reinterpret_cast<uint4*>(sm + kMlCoef + sw64(e, c)) = u;
        *reinterpret_cast<uint4*>(sm + kMlCoefS + sw64(e, c)) = us;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bar_in);
      if (nb == 0) break;
      // ---- Zᵀ → G' (σ(z) − y inside the crop) and the loss
      if (!mbar_wait(&bar_z, batch & 1, P.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int c0 = 0; c0 < nb16; c0 += 16) {
        float z[16];
        __syncwarp();
        tmem_ld16(lane_base + c0, z);
#pragma unroll
        for (int h = 0; h < 2; h++) {
          float g[8];
#pragma unroll
          for (int q = 0; q < 8; q++) {
            const int e = c0 + 8 * h + q;
            g[q] = 0.f;
            if (e < nb) {
              const MlMeta& mm = s_pend[e];
              if (fpx >= mm.x1 && fpx < mm.x2 && fpy >= mm.y1 && fpy < mm.y2) {
                const int pi = mpy * P.Wp + mpx;
                const float y = (P.gmask[((long long)b * P.G + mm.j) * words + (pi >> 5)] >> (pi & 31)) & 1u ? 1.f : 0.f;
                const float zz = z[8 * h + q];
                const float ex = ml_ex2(-kLog2e * fabsf(zz)), d = 1.f + ex, r = ml_rcp(d);
                const float sg = zz >= 0.f ? r : ex * r;
                g[q] = sg - y;
                lsum += (fmaxf(zz, 0.f) - zz * y + ml_lg2(d) * kLn2) * mm.inv;
              }
            }
          }
          const int e0 = c0 + 8 * h;
          uint4 u;
          __half2* hh = reinterpret_cast<__half2*>(&u);
#pragma unroll
          for (int q = 0; q < 4; q++) hh[q] = __floats2half2_rn(g[2 * q], g[2 * q + 1]);
          *reinterpret_cast<uint4*>(sm + kMlG + (e0 >> 6) * kMlGBlock + sw128(m, (e0 & 63) >> 3)) = u;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bar_g);
      // ---- dCoef block: scale by s_i, add into the positive's fp32 row
      if (!mbar_wait(&bar_c, batch & 1, P.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < 32; c0 += 16) {
        float v[16];
        __syncwarp();
        tmem_ld16(lane_base + c0, v);
        if (m < nb) {
          const float s = s_pend[m].inv * gk;
          float* row = P.acc + ((long long)b * P.A + s_pidx[m]) * 32 + c0;
#pragma unroll
          for (int q = 0; q < 16; q += 4)
            atomicAdd(reinterpret_cast<float4*>(row + q), make_float4(v[q] * s, v[q + 1] * s, v[q + 2] * s, v[q + 3] * s));
        }
      }
      tc_fence_before();
      // ---- drop the batch from the pending list
      named_bar_sync(1, kMlWorkers);
      for (int e = m; e < pend - nb; e += kMlWorkers) {
        s_pend[e] = s_pend[nb + e];
        s_pidx[e] = s_pidx[nb + e];
      }
      named_bar_sync(1, kMlWorkers);
      pend -= nb;
      batch++;
    }
    // ---- dProto: 2^e_b · accumulator → fp16 (zero where no positive reaches the pixel)
    {
      float v[32];
#pragma unroll
      for (int q = 0; q < 32; q++) v[q] = 0.f;
      if (ok && batch > 0) {
        __syncwarp();
        tmem_ld16(lane_base + kMlDProtoCol, *reinterpret_cast<float(*)[16]>(&v[0]));
        __syncwarp();
        tmem_ld16(lane_base + kMlDProtoCol + 16, *reinterpret_cast<float(*)[16]>(&v[16]));
#pragma unroll
        for (int q = 0; q < 32; q++) v[q] = ldexpf(v[q], e_b);
      }
      uint4* dst = reinterpret_cast<uint4*>(P.dproto + (((long long)b * P.Hp + mpy) * P.Wp + mpx) * 32);
#pragma unroll
      for (int c = 0; c < 4; c++) {
        uint4 u;
        __half2* hh = reinterpret_cast<__half2*>(&u);
#pragma unroll
        for (int q = 0; q < 4; q++) hh[q] = __floats2half2_rn(v[8 * c + 2 * q], v[8 * c + 2 * q + 1]);
        dst[c] = u;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lsum += __shfl_down_sync(~0u, lsum, o);
    if (lane == 0) s_loss[warp] = lsum;
    named_bar_sync(1, kMlWorkers);
    if (tid == 0) {
      const float t = (s_loss[0] + s_loss[1]) + (s_loss[2] + s_loss[3]);
      if (t != 0.f) atomicAdd(P.loss, t);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, kMlTmemCols);
  }
}

// dCoef rows → the coef-gradient heads (fp16) at the positive anchors; the rows, the positives' records and
// the per-image maximum are zeroed again for the next call.
__global__ void k_ml_finish(const MlArgs P) {
  const long long bi = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // (b, i)
  if (bi >= (long long)P.B * P.A) return;
  const int b = int(bi / P.A), i = int(bi - (long long)b * P.A);
  if (i == 0) P.smax[b] = 0;
  if (i >= P.npos[b]) return;
  const MlMeta m = P.meta[bi];
  P.meta[bi] = MlMeta{0.f, 0.f, 0.f, 0.f, 0.f, 0, 0, 0};
  float4* src = reinterpret_cast<float4*>(P.acc + bi * 32);
  __half* db = m.l == 0 ? P.dcoef[0] : (m.l == 1 ? P.dcoef[1] : P.dcoef[2]);
  uint4* dst = reinterpret_cast<uint4*>(db + (long long)m.row * 32);
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const float4 a0 = src[2 * c], a1 = src[2 * c + 1];
    src[2 * c] = make_float4(0.f, 0.f, 0.f, 0.f);
    src[2 * c + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
    uint4 u;
    __half2* hh = reinterpret_cast<__half2*>(&u);
    hh[0] = __floats2half2_rn(a0.x, a0.y);
    hh[1] = __floats2half2_rn(a0.z, a0.w);
    hh[2] = __floats2half2_rn(a1.x, a1.y);
    hh[3] = __floats2half2_rn(a1.z, a1.w);
    dst[c] = u;
  }
}

size_t ml_ws_bytes(int B, int A) {
  const size_t acc = (size_t)B * A * 32 * sizeof(float);
  const size_t meta = (size_t)B * A * sizeof(MlMeta);
  return ((acc + meta + (size_t)B * sizeof(int)) + 255) / 256 * 256;
}

int ml_fail(int code, const char* what) {
  set_last_error("%s", what);
  return code;
}

}  // namespace
}  // namespace osam

using namespace osam;

extern "C" {

size_t osam_mask_loss_workspace_size(int batch, int anchors) {
  return batch > 0 && anchors > 0 ? ml_ws_bytes(batch, anchors) : 0;
}

int osam_mask_loss(const void* const* coef, const int* level_hw, const void* proto, int batch, int proto_h, int proto_w,
                   int imgsz, int max_gt, const int* npos, const int* pos, const int* agt, const float* gt_box,
                   const uint32_t* gt_mask, const float* fg, const float* scale, float box_gain, void* dproto,
                   void* const* dcoef, float* loss_sum, void* ws, size_t ws_bytes, osam_stream_t stream) {
  if (!coef || !level_hw || !proto || !npos || !pos || !agt || !gt_box || !gt_mask || !fg || !scale || !dproto ||
      !dcoef || !loss_sum)
    return ml_fail(OSAM_ERR_INVALID, "mask_loss: null argument");
  if (batch < 1 || imgsz < 1 || max_gt < 1 || proto_w % kMlTileW || proto_h % kMlTileH || proto_w < kMlTileW ||
      proto_h < kMlTileH || (proto_h * proto_w) % 32)
    return ml_fail(OSAM_ERR_INVALID, "mask_loss: proto grid must be a multiple of 16 wide and 8 high");
  MlArgs P{};
  P.off[0] = 0;
  for (int l = 0; l < 3; l++) {
    P.coef[l] = static_cast<const __half*>(coef[l]);
    P.dcoef[l] = static_cast<__half*>(dcoef[l]);
    P.lvl_h[l] = level_hw[2 * l];
    P.lvl_w[l] = level_hw[2 * l + 1];
    if (!P.coef[l] || !P.dcoef[l] || P.lvl_h[l] < 1 || P.lvl_w[l] < 1 ||
        ((reinterpret_cast<uintptr_t>(P.coef[l]) | reinterpret_cast<uintptr_t>(P.dcoef[l])) & 15))
      return ml_fail(OSAM_ERR_INVALID, "mask_loss: coef heads (16-byte aligned NHWC, 32 channels)");
    P.off[l + 1] = P.off[l] + P.lvl_h[l] * P.lvl_w[l];
  }
  if (((reinterpret_cast<uintptr_t>(proto) | reinterpret_cast<uintptr_t>(dproto) |
        reinterpret_cast<uintptr_t>(gt_box)) & 15))
    return ml_fail(OSAM_ERR_INVALID, "mask_loss: proto / dproto / gt boxes must be 16-byte aligned");
  P.proto = static_cast<const __half*>(proto);
  P.dproto = static_cast<__half*>(dproto);
  P.B = batch;
  P.A = P.off[3];
  P.G = max_gt;
  P.Hp = proto_h;
  P.Wp = proto_w;
  P.imgsz = imgsz;
  P.npos = npos;
  P.pos = pos;
  P.agt = agt;
  P.gtb = reinterpret_cast<const float4*>(gt_box);
  P.gmask = gt_mask;
  P.fg = fg;
  P.scale = scale;
  P.box_gain = box_gain;
  P.loss = loss_sum;
  const size_t need = ml_ws_bytes(batch, P.A);
  if (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255))
    return ml_fail(OSAM_ERR_INVALID, "mask_loss: workspace (osam_mask_loss_workspace_size, 256-byte aligned)");
  char* w = static_cast<char*>(ws);
  P.acc = reinterpret_cast<float*>(w);
  P.meta = reinterpret_cast<MlMeta*>(w + (size_t)batch * P.A * 32 * sizeof(float));
  P.smax = reinterpret_cast<int*>(w + (size_t)batch * P.A * (32 * sizeof(float) + sizeof(MlMeta)));
  P.err = device_error_word();
  if (!P.err) return ml_fail(OSAM_ERR_CUDA, "mask_loss: no device error word");
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(k_ml_tile, cudaFuncAttributeMaxDynamicSharedMemorySize, kMlSmem) != cudaSuccess)
      return ml_fail(OSAM_ERR_CUDA, "mask_loss: shared-memory opt-in");
    attr = true;
  }
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const long long nba = (long long)batch * P.A;
  k_ml_meta<<<(unsigned)((nba + 255) / 256), 256, 0, st>>>(P);
  k_ml_tile<<<dim3((proto_w / kMlTileW) * (proto_h / kMlTileH), batch), kMlThreads, kMlSmem, st>>>(P);
  k_ml_finish<<<(unsigned)((nba + 255) / 256), 256, 0, st>>>(P);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("osam_mask_loss launch: %s", cudaGetErrorString(e));
    return OSAM_ERR_CUDA;
  }
  return OSAM_OK;
}

}  // extern "C"
