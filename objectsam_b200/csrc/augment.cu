// GPU augmentation of one training batch: the model input and the targets of the segmentation loss.
//
// Replaces the reference's augment() (src/augment.cuh:19, kernels src/augment.cu): per output image, a
// 2S × 2S mosaic canvas of up to four source tiles (fill value 114 outside them), an affine map canvas →
// output (out = s·u + t; the output pixel samples the canvas at M⁻¹·(x, y), bilinear, pixel centres on
// integer coordinates), OpenCV's u8 HSV round trip with per-image gains, a left-right flip, and fp16 in
// 0..1; the targets (each instance's box clipped to its tile, mapped, clipped to the image, flipped and
// filtered: w, h > 2 px, kept area > 10 %, aspect < 100), their mask bits on the Hp × Wp loss grid
// (each cell centre followed back to the instance's bitmap) and the ignore-region bits.
//
// The float steps of every pixel, box and cell are the reference's, in its order, and this file is
// compiled under the same fast-math arithmetic as the reference's build (build.py), so that rounding
// agrees bit for bit (tests/test_augment_gpu.py checks it against the reference's own kernels).
//
// Layout of the work (B200: HBM-bound byte work, no tensor cores):
//   k_aug_image    one thread per output pixel (the canvas gathers are latency-bound: all the threads the SM
//                  holds are needed): the image's sample record and its tiles' source records are staged in
//                  shared memory once per block, and the block's 256 pixels (1536 B of fp16) are staged there
//                  too and leave as 16-byte stores;
//   k_aug_targets  one block per image: an ordered compaction of its instances (warp ballots + a block
//                  scan), writing boxes, instance indices and n_gt; slots past n_gt are zeroed;
//   k_aug_gtmask   one block per (image, target slot), one lane per cell and one warp per 32-cell word (the
//                  word is a ballot: no per-thread chain of dependent bitmap loads): every word of every
//                  slot is written once (zeros outside the target's window and in empty slots), so the
//                  bitmaps need no separate clearing pass;
//   k_aug_ignore   blocks of 64 words per image: each gathers its image's ignore instances and their cell
//                  windows into shared memory, and each warp ORs the instances' ballots into its 8 words in
//                  registers (no atomics), written once.
#include "conv_internal.h"

#include <cuda_fp16.h>
#include <stdint.h>

namespace osam {
namespace {

constexpr int kAugThreads = 256;
constexpr int kFill = 114;  // canvas value outside every tile (the mosaic fill and the affine border)

// Exact small-integer ↔ float conversions on the FP32 / integer pipes instead of the conversion unit, which
// the image kernel's ~38 conversions per pixel would otherwise queue on.  For |x| < 2²², the float whose bits
// are 0x4B400000 + x is 1.5·2²³ + x, so subtracting 1.5·2²³ leaves x exactly; and for |v| < 2²², v + 1.5·2²³
// lies in [2²³, 2²⁴), where the float spacing is 1, so the rounded sum holds v rounded to the nearest integer
// (ties to even) in its low bits, as __float2int_rn gives.  The explicitly rounded intrinsics keep the
// compiler from fusing the magic add into a preceding multiply.
constexpr float kMagic = 12582912.f;  // 1.5·2²³, bits 0x4B400000
__device__ __forceinline__ float small_i2f(int x) { return __fsub_rn(__int_as_float(0x4B400000 + x), kMagic); }
__device__ __forceinline__ int small_f2i_rn(float v) {
  return fabsf(v) < 4194304.f ? __float_as_int(__fadd_rn(v, kMagic)) - 0x4B400000 : __float2int_rn(v);
}

// The sample record and its tiles' source records, staged per block.
struct AugShared {
  osam_aug_sample sm;
  osam_aug_src src[4];
};

__device__ __forceinline__ void stage_sample(AugShared& sh, const osam_aug_batch& bt, int i) {
  if (threadIdx.x == 0) {
    sh.sm = bt.smp[i];
    for (int t = 0; t < 4; t++)
      if (sh.sm.src[t] >= 0) sh.src[t] = bt.src[sh.sm.src[t]];
  }
  __syncthreads();
}

// Canvas pixel (px, py): the first tile (0..3, present) whose rectangle holds it, read from its source;
// kFill outside the canvas or every tile.
__device__ __forceinline__ void canvas_rgb(const AugShared& sh, const uint8_t* __restrict__ img, int S, int px,
                                           int py, float c[3]) {
  c[0] = c[1] = c[2] = (float)kFill;
  if (px < 0 || py < 0 || px >= 2 * S || py >= 2 * S) return;
#pragma unroll
  for (int t = 0; t < 4; t++) {
    if (sh.sm.src[t] < 0) continue;
    const int* r = sh.sm.ta[t];
    if (px < r[0] || px >= r[2] || py < r[1] || py >= r[3]) continue;
    const int xs = px - r[0] + sh.sm.tb[t][0], ys = py - r[1] + sh.sm.tb[t][1];
    const uint8_t* p = img + sh.src[t].img_off + ((int64_t)ys * sh.src[t].iw + xs) * 3;
    c[0] = small_i2f(p[0]);
    c[1] = small_i2f(p[1]);
    c[2] = small_i2f(p[2]);
    return;
  }
}

// The four canvas pixels of a bilinear quad (cx, cy) … (cx + 1, cy + 1), as canvas_rgb gives them.  The
// first present tile whose rectangle touches the quad decides: when it holds all four corners (and the quad
// is on the canvas) they are read from it together — no earlier tile touches the quad, so it is every
// corner's first holder; when no tile touches the quad all four are the fill value; otherwise (a tile or
// canvas edge through the quad) corner by corner.
__device__ __forceinline__ void canvas_quad(const AugShared& sh, const uint8_t* __restrict__ img, int S, int cx,
                                            int cy, float p00[3], float p10[3], float p01[3], float p11[3]) {
  int first = -1;
#pragma unroll
  for (int t = 0; t < 4; t++) {
    if (sh.sm.src[t] < 0) continue;
    const int* r = sh.sm.ta[t];
    if (r[0] <= cx + 1 && r[2] > cx && r[1] <= cy + 1 && r[3] > cy) {
      first = t;
      break;
    }
  }
  if (first < 0) {
#pragma unroll
    for (int c = 0; c < 3; c++) p00[c] = p10[c] = p01[c] = p11[c] = (float)kFill;
    return;
  }
  const int* r = sh.sm.ta[first];
  if (cx >= r[0] && cx + 1 < r[2] && cy >= r[1] && cy + 1 < r[3] && cx >= 0 && cy >= 0 && cx + 1 < 2 * S &&
      cy + 1 < 2 * S) {
    const osam_aug_src& si = sh.src[first];
    const uint8_t* q = img + si.img_off + ((int64_t)(cy - r[1] + sh.sm.tb[first][1]) * si.iw +
                                           (cx - r[0] + sh.sm.tb[first][0])) * 3;
    const uint8_t* q1 = q + (int64_t)si.iw * 3;
#pragma unroll
    for (int c = 0; c < 3; c++) {
      p00[c] = small_i2f(q[c]);
      p10[c] = small_i2f(q[3 + c]);
      p01[c] = small_i2f(q1[c]);
      p11[c] = small_i2f(q1[3 + c]);
    }
    return;
  }
  canvas_rgb(sh, img, S, cx, cy, p00);
  canvas_rgb(sh, img, S, cx + 1, cy, p10);
  canvas_rgb(sh, img, S, cx, cy + 1, p01);
  canvas_rgb(sh, img, S, cx + 1, cy + 1, p11);
}

__device__ __forceinline__ int clamp_u8(float v) { return min(255, max(0, small_f2i_rn(v))); }

// u8 RGB → u8 HSV with H in 0..179 (OpenCV's convention): V = max, S = 255·(max − min)/max, H from the
// sector of the largest channel, halved.
__device__ __forceinline__ void to_hsv(int r, int g, int b, int& h, int& s, int& v) {
  const int hi = max(r, max(g, b)), lo = min(r, min(g, b)), span = hi - lo;
  v = hi;
  const float fspan = small_i2f(span);
  s = hi ? small_f2i_rn(255.f * fspan / small_i2f(hi)) : 0;
  float deg = 0.f;
  if (span) {
    if (hi == r)
      deg = 60.f * small_i2f(g - b) / fspan;
    else if (hi == g)
      deg = 120.f + 60.f * small_i2f(b - r) / fspan;
    else
      deg = 240.f + 60.f * small_i2f(r - g) / fspan;
    if (deg < 0) deg += 360.f;
  }
  h = small_f2i_rn(deg * 0.5f);
  if (h >= 180) h -= 180;
}

// u8 HSV (H 0..179) → u8 RGB: sector i = ⌊H/60°⌋, fraction f, and the three intermediate levels.
__device__ __forceinline__ void from_hsv(int h, int s, int v, int& r, int& g, int& b) {
  const float hs = small_i2f(h) * 2.f / 60.f, sat = small_i2f(s) / 255.f, val = small_i2f(v);
  const int sector = int(floorf(hs)) % 6;
  const float f = hs - floorf(hs);
  const float p = val * (1 - sat), q = val * (1 - sat * f), t = val * (1 - sat * (1 - f));
  float R = val, G = p, B = q;  // sector 5
  if (sector == 0) { R = val; G = t; B = p; }
  else if (sector == 1) { R = q; G = val; B = p; }
  else if (sector == 2) { R = p; G = val; B = t; }
  else if (sector == 3) { R = p; G = q; B = val; }
  else if (sector == 4) { R = t; G = p; B = val; }
  r = clamp_u8(R);
  g = clamp_u8(G);
  b = clamp_u8(B);
}

// fmodf(x, 180) for the hue: for 0 ≤ x < 360 it is x or x − 180, and that difference is exact (Sterbenz:
// 180 ≤ x < 360), so the single subtraction equals the exactly-defined fmod; elsewhere fmodf itself.
__device__ __forceinline__ float hue_mod180(float x) {
  if (x >= 0.f && x < 360.f) return x >= 180.f ? x - 180.f : x;
  return fmodf(x, 180.f);
}

__global__ void __launch_bounds__(kAugThreads) k_aug_image(const osam_aug_batch bt, int S, __half* __restrict__ out) {
  __shared__ AugShared sh;
  __shared__ __align__(16) __half stage[kAugThreads * 3];  // the block's pixels, written out as 16-byte rows
  const int i = blockIdx.y;
  stage_sample(sh, bt, i);
  const int64_t npix = (int64_t)S * S, p0 = (int64_t)blockIdx.x * kAugThreads;
  const int64_t pix = p0 + threadIdx.x;
  const osam_aug_sample& sm = sh.sm;
  if (pix < npix) {
    const int y = (int)pix / S, x = (int)pix - y * S;  // S ≤ 16384: S² fits 31 bits
    const int xs = sm.flip ? S - 1 - x : x;
    // output → canvas: (x, y) = s·(u, v) + t, sampled bilinearly around (u, v)
    const float u = (xs - sm.tx) / sm.s, v = (y - sm.ty) / sm.s;
    const int cx = int(floorf(u)), cy = int(floorf(v));
    const float fx = u - cx, fy = v - cy;
    float p00[3], p10[3], p01[3], p11[3];
    canvas_quad(sh, bt.img, S, cx, cy, p00, p10, p01, p11);
    int rgb[3];
#pragma unroll
    for (int c = 0; c < 3; c++)
      rgb[c] = clamp_u8((p00[c] * (1 - fx) + p10[c] * fx) * (1 - fy) + (p01[c] * (1 - fx) + p11[c] * fx) * fy);
    // HSV gains as a lookup of the u8 levels: hue (H·g₀) mod 180, saturation and value clipped to 0..255
    int h, s, vv;
    to_hsv(rgb[0], rgb[1], rgb[2], h, s, vv);
    h = int(hue_mod180(small_i2f(h) * sm.hsv[0]));
    s = int(fminf(fmaxf(small_i2f(s) * sm.hsv[1], 0.f), 255.f));
    vv = int(fminf(fmaxf(small_i2f(vv) * sm.hsv[2], 0.f), 255.f));
    from_hsv(h, s, vv, rgb[0], rgb[1], rgb[2]);
#pragma unroll
    for (int c = 0; c < 3; c++) stage[3 * threadIdx.x + c] = __float2half(small_i2f(rgb[c]) / 255.f);
  }
  __syncthreads();
  // the block's pixels are contiguous in the output: 6 bytes each, 16-byte rows (S² is a multiple of 64,
  // so every block's byte count is a multiple of 16 and its start is 16-byte aligned)
  const int nb = (int)((npix - p0 < kAugThreads ? npix - p0 : kAugThreads) * 6 / 16);
  uint4* dst = reinterpret_cast<uint4*>(out + ((int64_t)i * npix + p0) * 3);
  const uint4* src = reinterpret_cast<const uint4*>(stage);
  for (int q = threadIdx.x; q < nb; q += kAugThreads) dst[q] = src[q];
}

// Exclusive rank of `flag` among the block's threads in thread order, and the block's total.
__device__ __forceinline__ int block_rank_of(bool flag, int* warp_tot, int& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const unsigned m = __ballot_sync(0xffffffffu, flag);
  if (lane == 0) warp_tot[w] = __popc(m);
  __syncthreads();
  int before = 0;
  total = 0;
  for (int q = 0; q < nw; q++) {
    const int c = warp_tot[q];
    before += q < w ? c : 0;
    total += c;
  }
  __syncthreads();
  return before + __popc(m & ((1u << lane) - 1u));
}

// An instance's box in output pixels (clipped to its tile on the canvas, mapped, clipped to 0..S,
// flipped), and the box's mapped size before the output clip (w1, h1).  False when nothing of it lies
// inside its tile.
__device__ __forceinline__ bool map_box(const osam_aug_sample& sm, const osam_aug_inst& in, int S, float& X1,
                                        float& Y1, float& X2, float& Y2, float& w1, float& h1) {
  const int t = in.tile;
  const float dx = float(sm.ta[t][0] - sm.tb[t][0]), dy = float(sm.ta[t][1] - sm.tb[t][1]);
  const float x1 = fmaxf(in.box[0] + dx, sm.ta[t][0]), y1 = fmaxf(in.box[1] + dy, sm.ta[t][1]);
  const float x2 = fminf(in.box[2] + dx, sm.ta[t][2]), y2 = fminf(in.box[3] + dy, sm.ta[t][3]);
  if (!(x2 > x1 && y2 > y1)) return false;
  w1 = (x2 - x1) * sm.s;
  h1 = (y2 - y1) * sm.s;
  X1 = fminf(fmaxf(sm.s * x1 + sm.tx, 0.f), float(S));
  X2 = fminf(fmaxf(sm.s * x2 + sm.tx, 0.f), float(S));
  Y1 = fminf(fmaxf(sm.s * y1 + sm.ty, 0.f), float(S));
  Y2 = fminf(fmaxf(sm.s * y2 + sm.ty, 0.f), float(S));
  if (sm.flip) {
    const float a = S - X2, b = S - X1;
    X1 = a;
    X2 = b;
  }
  return true;
}

__global__ void __launch_bounds__(kAugThreads) k_aug_targets(const osam_aug_batch bt, int S, const osam_aug_out o) {
  __shared__ AugShared sh;
  __shared__ int warp_tot[kAugThreads / 32];
  const int i = blockIdx.x;
  stage_sample(sh, bt, i);
  const osam_aug_sample& sm = sh.sm;
  const int ninst = bt.hdr->ninst;
  int n = 0;  // targets found so far (uniform)
  for (int k0 = 0; k0 < ninst && n < o.G; k0 += blockDim.x) {
    const int k = k0 + threadIdx.x;
    bool keep = false;
    float X1 = 0.f, Y1 = 0.f, X2 = 0.f, Y2 = 0.f;
    if (k < ninst) {
      const osam_aug_inst in = bt.inst[k];
      float w1, h1;
      if (in.sample == i && !in.ignore && map_box(sm, in, S, X1, Y1, X2, Y2, w1, h1)) {
        const float w2 = X2 - X1, h2 = Y2 - Y1;
        const float aspect = fmaxf(w2 / (h2 + 1e-16f), h2 / (w2 + 1e-16f));
        keep = w2 > 2.f && h2 > 2.f && w2 * h2 / (w1 * h1 + 1e-16f) > 0.1f && aspect < 100.f;
      }
    }
    int total;
    const int slot = n + block_rank_of(keep, warp_tot, total);
    if (keep && slot < o.G) {
      reinterpret_cast<float4*>(o.box)[(int64_t)i * o.G + slot] = make_float4(X1, Y1, X2, Y2);
      o.gt_inst[(int64_t)i * o.G + slot] = k;
    }
    n += total;
  }
  const int ng = min(n, o.G);
  for (int j = ng + threadIdx.x; j < o.G; j += blockDim.x) {
    reinterpret_cast<float4*>(o.box)[(int64_t)i * o.G + j] = make_float4(0.f, 0.f, 0.f, 0.f);
    o.gt_inst[(int64_t)i * o.G + j] = -1;
  }
  if (threadIdx.x == 0) o.n_gt[i] = ng;
}

// The loss-grid window of an output box: cells [c0, c1) × [r0, r1), one cell of margin, clipped.
__device__ __forceinline__ void box_cells(float x1, float y1, float x2, float y2, float cs, int Hp, int Wp, int& c0,
                                          int& c1, int& r0, int& r1) {
  c0 = max(0, int(floorf(x1 / cs)) - 1);
  c1 = min(Wp, int(ceilf(x2 / cs)) + 1);
  r0 = max(0, int(floorf(y1 / cs)) - 1);
  r1 = min(Hp, int(ceilf(y2 / cs)) + 1);
}

// Mask bit of cell (r, c): the cell centre followed back through flip, affine and tile to the instance's
// bitmap.
__device__ __forceinline__ bool cell_bit(const osam_aug_sample& sm, const osam_aug_inst& in, float kx, float ky,
                                         const uint32_t* __restrict__ mask, int S, float cs, int r, int c) {
  const int t = in.tile;
  const float x = (c + 0.5f) * cs - 0.5f, y = (r + 0.5f) * cs - 0.5f;  // cell centre, output pixels
  const float xs = sm.flip ? S - 1 - x : x;
  const float u = (xs - sm.tx) / sm.s, v = (y - sm.ty) / sm.s;        // canvas
  if (u < sm.ta[t][0] || u >= sm.ta[t][2] || v < sm.ta[t][1] || v >= sm.ta[t][3]) return false;
  const float sx = u - sm.ta[t][0] + sm.tb[t][0], sy = v - sm.ta[t][1] + sm.tb[t][1];  // source pixels
  const int mx = int(floorf((sx + 0.5f) * kx)) - in.mx0, my = int(floorf((sy + 0.5f) * ky)) - in.my0;
  if (mx < 0 || my < 0 || mx >= in.mcw || my >= in.mch) return false;
  return (mask[in.mask_off + (int64_t)my * in.wpr + (mx >> 5)] >> (mx & 31)) & 1u;
}

// One lane per cell, one warp per 32-cell word (a word is 32 cells of one row: Wp % 32 == 0), the word
// formed by a ballot: no per-thread chain of dependent bitmap loads.
constexpr int kMaskThreads = 256;

__global__ void __launch_bounds__(kMaskThreads) k_aug_gtmask(const osam_aug_batch bt, int S, const osam_aug_out o) {
  __shared__ AugShared sh;
  const int i = blockIdx.y, j = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int words = o.Hp * o.Wp / 32, wpr = o.Wp / 32;
  uint32_t* dst = o.mask + ((int64_t)i * o.G + j) * words;
  const int ng = o.n_gt[i];
  if (j >= ng) {
    for (int q = threadIdx.x; q < words; q += blockDim.x) dst[q] = 0u;
    return;
  }
  stage_sample(sh, bt, i);
  const osam_aug_sample& sm = sh.sm;
  const osam_aug_inst in = bt.inst[o.gt_inst[(int64_t)i * o.G + j]];
  const osam_aug_src si = bt.src[in.src];
  const float4 bx = reinterpret_cast<const float4*>(o.box)[(int64_t)i * o.G + j];
  const float cs = float(S) / o.Wp;  // cell size, output pixels
  int c0, c1, r0, r1;
  box_cells(bx.x, bx.y, bx.z, bx.w, cs, o.Hp, o.Wp, c0, c1, r0, r1);
  const float kx = float(si.mw) / si.iw, ky = float(si.mh) / si.ih;
  const int w0 = c0 >> 5, w1 = (c1 + 31) >> 5, nww = w1 > w0 ? w1 - w0 : 0, nwr = r1 > r0 ? r1 - r0 : 0;
  // words outside the window: zero, all threads, coalesced
  for (int q = threadIdx.x; q < words; q += kMaskThreads) {
    const int r = q / wpr, w = q - r * wpr;
    if (r < r0 || r >= r1 || w < w0 || w >= w1) dst[q] = 0u;
  }
  // the window's words: a warp each
  for (int k = warp; k < nwr * nww; k += kMaskThreads / 32) {
    const int r = r0 + k / nww, w = w0 + k % nww, c = w * 32 + lane;
    const bool in_win = c >= c0 && c < c1;
    const unsigned bits = __ballot_sync(0xffffffffu, in_win && cell_bit(sm, in, kx, ky, bt.mask, S, cs, r, c));
    if (lane == 0) dst[r * wpr + w] = bits;
  }
}

// Per image, its ignore instances that reach into their tile, with their cell windows: gathered by each
// block of k_aug_ignore (a scan over the batch's instances, in order).
struct IgnWin {
  int k, c0, c1, r0, r1;
};
constexpr int kIgnoreWords = 8;  // words per warp of k_aug_ignore (a block covers 8 warps × 8 words)

// Grid (word blocks, B): each warp ORs, word by word, the ballots of every ignore instance of its image.
__global__ void __launch_bounds__(kAugThreads) k_aug_ignore(const osam_aug_batch bt, int S, const osam_aug_out o) {
  __shared__ AugShared sh;
  __shared__ IgnWin win[kAugThreads];
  __shared__ int warp_tot[kAugThreads / 32];
  const int i = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int words = o.Hp * o.Wp / 32, wpr = o.Wp / 32;
  const int q0 = (blockIdx.x * (kAugThreads / 32) + warp) * kIgnoreWords;  // this warp's first word
  stage_sample(sh, bt, i);
  const osam_aug_sample& sm = sh.sm;
  const int ninst = bt.hdr->ninst;
  const float cs = float(S) / o.Wp;
  uint32_t acc[kIgnoreWords];
#pragma unroll
  for (int w = 0; w < kIgnoreWords; w++) acc[w] = 0u;
  for (int k0 = 0; k0 < ninst; k0 += blockDim.x) {
    const int k = k0 + threadIdx.x;
    bool hit = false;
    IgnWin wv{};
    if (k < ninst) {
      const osam_aug_inst in = bt.inst[k];
      float X1, Y1, X2, Y2, w1, h1;
      if (in.sample == i && in.ignore && map_box(sm, in, S, X1, Y1, X2, Y2, w1, h1)) {
        hit = true;
        wv.k = k;
        box_cells(X1, Y1, X2, Y2, cs, o.Hp, o.Wp, wv.c0, wv.c1, wv.r0, wv.r1);
      }
    }
    int nl;
    const int slot = block_rank_of(hit, warp_tot, nl);
    if (hit) win[slot] = wv;
    __syncthreads();
    for (int l = 0; l < nl; l++) {
      const IgnWin w = win[l];
      const osam_aug_inst in = bt.inst[w.k];
      const osam_aug_src si = bt.src[in.src];
      const float kx = float(si.mw) / si.iw, ky = float(si.mh) / si.ih;
#pragma unroll
      for (int u = 0; u < kIgnoreWords; u++) {
        const int q = q0 + u;
        if (q >= words) break;
        const int r = q / wpr, c = (q - r * wpr) * 32 + lane;
        const bool in_win = r >= w.r0 && r < w.r1 && c >= w.c0 && c < w.c1;
        if (__ballot_sync(0xffffffffu, in_win))
          acc[u] |= __ballot_sync(0xffffffffu, in_win && cell_bit(sm, in, kx, ky, bt.mask, S, cs, r, c));
      }
    }
    __syncthreads();
  }
  uint32_t* dst = o.ignore + (int64_t)i * words;
#pragma unroll
  for (int u = 0; u < kIgnoreWords; u++)
    if (lane == 0 && q0 + u < words) dst[q0 + u] = acc[u];
}

}  // namespace
}  // namespace osam

using namespace osam;

extern "C" int osam_augment(const osam_aug_batch* batch, int B, int S, const osam_aug_out* out,
                            osam_stream_t stream) {
  if (!batch || !out || B < 1 || S < 8 || S > 16384 || S % 8 || out->G < 1 || out->Hp < 1 || out->Wp < 32 ||
      out->Wp % 32) {
    set_last_error("osam_augment: invalid arguments (need B ≥ 1, 8 ≤ S ≤ 16384, S % 8 == 0, G ≥ 1, Wp % 32 == 0)");
    return OSAM_ERR_INVALID;
  }
  if (!batch->hdr || !batch->smp || !batch->src || !batch->inst || !batch->img || !batch->mask || !out->img ||
      !out->n_gt || !out->box || !out->mask || !out->gt_inst) {
    set_last_error("osam_augment: NULL pointer");
    return OSAM_ERR_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(out->img) & 15) || (reinterpret_cast<uintptr_t>(out->box) & 15)) {
    set_last_error("osam_augment: img and box must be 16-byte aligned");
    return OSAM_ERR_INVALID;
  }
  // records with 64-bit fields must sit on 8-byte boundaries (in the reference's one-block layout that
  // holds for even B: the 148-byte sample records come first)
  if ((reinterpret_cast<uintptr_t>(batch->hdr) & 7) || (reinterpret_cast<uintptr_t>(batch->src) & 7) ||
      (reinterpret_cast<uintptr_t>(batch->inst) & 7) || (reinterpret_cast<uintptr_t>(batch->smp) & 3)) {
    set_last_error("osam_augment: header, source and instance records must be 8-byte aligned");
    return OSAM_ERR_INVALID;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const osam_aug_batch bt = *batch;
  const osam_aug_out o = *out;
  const int64_t npix = (int64_t)S * S;
  k_aug_image<<<dim3((unsigned)((npix + kAugThreads - 1) / kAugThreads), B), kAugThreads, 0, st>>>(
      bt, S, static_cast<__half*>(o.img));
  k_aug_targets<<<B, kAugThreads, 0, st>>>(bt, S, o);
  k_aug_gtmask<<<dim3(o.G, B), kMaskThreads, 0, st>>>(bt, S, o);
  if (o.ignore) {
    const int words = o.Hp * o.Wp / 32, per_block = (kAugThreads / 32) * kIgnoreWords;
    k_aug_ignore<<<dim3((words + per_block - 1) / per_block, B), kAugThreads, 0, st>>>(bt, S, o);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("osam_augment launch: %s", cudaGetErrorString(e));
    return OSAM_ERR_CUDA;
  }
  return OSAM_OK;
}
