// Detection part of the training loss of the segment head: the SegLoss::run steps before the mask loss
// (reference src/loss.cu:123-390 and :590-612 — Ultralytics 8.4 v8SegmentationLoss with one class):
//   1. decode      per anchor: DFL expectation of the four distances (softmax over reg_max bins) → the
//                  predicted box in grid units, and the class score σ(cls);
//   2. top-k       per ground-truth box: the anchors whose centre lies in the box (enlarged to ≥ 16 px per
//                  side) ranked by the alignment metric √score·CIoU⁶ (ties: lower anchor id), the best 10
//                  mark themselves (a count and the gt id);
//   3. resolve     per anchor chosen at least once: its gt (the most-overlapping one when several chose it),
//                  its metric and overlap, and per gt the largest metric and overlap (atomic max);
//   4. positives   per image: the positive anchors in ANCHOR ORDER (a block scan — the reference appends
//                  them with an atomic counter, in no fixed order), their target scores
//                  t = metric·max_overlap(gt)/(max_metric(gt) + 1e-9) and the sum of t;
//   5. loss        per anchor: BCE(cls, t) (negatives whose centre lies in the ignore region excluded) and
//                  its gradient; on positives the CIoU loss and the DFL loss with their gradients through
//                  the softmax into the box head; negatives get zero box and coefficient gradients.
// The gradients are those of (Σ items)·batch with items normalised by the target-score sum, times the
// loss scale (a device float), exactly the reference's; the loss sums go to items[8] (CIoU), [10] (BCE),
// [11] (DFL), with [4] = positives and [5] = target-score sum; osam_seg_loss_items forms items[0..3] once the
// mask loss has added items[9].  All counts stay on the device: no host synchronisation, graph-capturable.
#include "conv_internal.h"

namespace osam {
namespace {

constexpr int kDlT = 256;
constexpr int kDlTopK = 10;
constexpr float kCiouEps = 1e-7f;  // bbox_iou's eps
constexpr float kTalEps = 1e-9f;   // the assigner's eps

struct Levels {
  int off[4];  // first anchor of each level; off[3] = A
  int h[3], w[3], s[3];
};

__device__ __forceinline__ void level_of(const Levels& L, int a, int& l, int& y, int& x) {
  l = a < L.off[1] ? 0 : (a < L.off[2] ? 1 : 2);
  const int r = a - L.off[l];
  y = r / L.w[l];
  x = r - y * L.w[l];
}

__device__ __forceinline__ float sigmoid(float x) { return 1.f / (1.f + expf(-x)); }
// BCE with logits, the numerically stable form max(x, 0) − x·y + log(1 + e^{−|x|})
__device__ __forceinline__ float bce(float x, float y) { return fmaxf(x, 0.f) - x * y + log1pf(expf(-fabsf(x))); }

// CIoU of two xyxy boxes (b1 predicted, b2 target), the Ultralytics bbox_iou(CIoU=True) formula with its eps
// placement; α is treated as a constant.  `grad` (optional): d CIoU / d b1.
__device__ float ciou_of(float4 b1, float4 b2, float4* grad) {
  const float w1 = b1.z - b1.x, h1 = b1.w - b1.y + kCiouEps, w2 = b2.z - b2.x, h2 = b2.w - b2.y + kCiouEps;
  const float ix2 = fminf(b1.z, b2.z), ix1 = fmaxf(b1.x, b2.x), iy2 = fminf(b1.w, b2.w), iy1 = fmaxf(b1.y, b2.y);
  const float iw0 = ix2 - ix1, ih0 = iy2 - iy1;
  const float iw = fmaxf(iw0, 0.f), ih = fmaxf(ih0, 0.f);
  const float inter = iw * ih, uni = w1 * h1 + w2 * h2 - inter + kCiouEps, iou = inter / uni;
  const float cx2 = fmaxf(b1.z, b2.z), cx1 = fminf(b1.x, b2.x), cy2 = fmaxf(b1.w, b2.w), cy1 = fminf(b1.y, b2.y);
  const float cw = cx2 - cx1, ch = cy2 - cy1;
  const float c2 = cw * cw + ch * ch + kCiouEps;
  const float sx = b2.x + b2.z - b1.x - b1.z, sy = b2.y + b2.w - b1.y - b1.w;
  const float rho2 = (sx * sx + sy * sy) * 0.25f;
  const float r1 = w1 / h1;
  const float dv = atanf(w2 / h2) - atanf(r1);
  const float k4 = 0.40528473456935108f;  // 4/π²
  const float v = k4 * dv * dv;
  const float alpha = v / (1.f - iou + v + kCiouEps);
  const float out = iou - (rho2 / c2 + v * alpha);
  if (grad) {
    float dx1 = 0.f, dy1 = 0.f, dx2 = 0.f, dy2 = 0.f, dw1 = 0.f, dh1 = 0.f;
    // iou = inter / (area1 + area2 − inter + eps)
    const float dinter = (uni + inter) / (uni * uni), darea1 = -inter / (uni * uni);
    dw1 += darea1 * h1;
    dh1 += darea1 * w1;
    const float diw = iw0 > 0.f ? dinter * ih : 0.f, dih = ih0 > 0.f ? dinter * iw : 0.f;
    if (b1.z < b2.z) dx2 += diw;
    if (b1.x > b2.x) dx1 -= diw;
    if (b1.w < b2.w) dy2 += dih;
    if (b1.y > b2.y) dy1 -= dih;
    // − ρ²/c²
    const float drho2 = -1.f / c2, dc2 = rho2 / (c2 * c2);
    dx1 += drho2 * (-sx * 0.5f);
    dx2 += drho2 * (-sx * 0.5f);
    dy1 += drho2 * (-sy * 0.5f);
    dy2 += drho2 * (-sy * 0.5f);
    const float dcw = dc2 * 2.f * cw, dch = dc2 * 2.f * ch;
    if (b1.z > b2.z) dx2 += dcw;
    if (b1.x < b2.x) dx1 -= dcw;
    if (b1.w > b2.w) dy2 += dch;
    if (b1.y < b2.y) dy1 -= dch;
    // − α·v with v = (4/π²)(atan(w2/h2) − atan(w1/h1))²
    const float dr1 = -alpha * k4 * 2.f * dv * (-1.f / (1.f + r1 * r1));
    dw1 += dr1 / h1;
    dh1 += dr1 * (-w1 / (h1 * h1));
    dx2 += dw1;
    dx1 -= dw1;
    dy2 += dh1;
    dy1 -= dh1;
    *grad = make_float4(dx1, dy1, dx2, dy2);
  }
  return out;
}

// select_candidates_in_gts: a box side shorter than 16 px (the middle stride) is widened to 16 around its centre
__device__ __forceinline__ float4 enlarged(float4 g) {
  const float cx = (g.x + g.z) * 0.5f, cy = (g.y + g.w) * 0.5f;
  float w = g.z - g.x, h = g.w - g.y;
  if (w < 16.f) w = 16.f;
  if (h < 16.f) h = 16.f;
  return make_float4(cx - w * 0.5f, cy - h * 0.5f, cx + w * 0.5f, cy + h * 0.5f);
}
__device__ __forceinline__ bool centre_in(float4 e, float px, float py) {
  return px - e.x > kTalEps && py - e.y > kTalEps && e.z - px > kTalEps && e.w - py > kTalEps;
}
__device__ __forceinline__ float align_metric(float score, float ov) {
  const float o2 = ov * ov;
  return sqrtf(score) * o2 * o2 * o2;
}

// ------------------------------------------------------------------------------------------------ 1. decode
struct Heads {
  const __half* box[3];
  const __half* cls[3];
};
template <int REG>
__global__ void __launch_bounds__(kDlT) k_dl_decode(const Levels L, int A, int B, const Heads H, float4* pbox,
                                                   float* score) {
  const long long q = (long long)blockIdx.x * kDlT + threadIdx.x;
  if (q >= (long long)B * A) return;
  const int b = (int)(q / A), a = (int)(q - (long long)b * A);
  int l, y, x;
  level_of(L, a, l, y, x);
  const long long pix = ((long long)b * L.h[l] + y) * L.w[l] + x;
  const __half* p = H.box[l] + pix * 4 * REG;
  float d[4];
#pragma unroll
  for (int s = 0; s < 4; s++) {
    float v[REG], m = -INFINITY;
#pragma unroll
    for (int k = 0; k < REG; k++) {
      v[k] = __half2float(p[s * REG + k]);
      m = fmaxf(m, v[k]);
    }
    float z = 0.f, e = 0.f;
#pragma unroll
    for (int k = 0; k < REG; k++) {
      const float t = expf(v[k] - m);
      z += t;
      e += t * k;
    }
    d[s] = e / z;
  }
  const float ax = x + 0.5f, ay = y + 0.5f;
  pbox[q] = make_float4(ax - d[0], ay - d[1], ax + d[2], ay + d[3]);
  score[q] = sigmoid(__half2float(H.cls[l][pix]));
}

// ------------------------------------------------------------------------------------------------ 2. top-k
// (metric, anchor) order of the ranking: larger metric first, then the lower anchor id; anchor −1 = none.
__device__ __forceinline__ bool ranks_before(float m1, int a1, float m2, int a2) {
  if (a1 < 0) return false;
  if (a2 < 0) return true;
  return m1 > m2 || (m1 == m2 && a1 < a2);
}
// the better of this lane's (m, a) and the one `off` lanes away
__device__ __forceinline__ void warp_best(float& m, int& a, int& src) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
    const int a2 = __shfl_xor_sync(0xffffffffu, a, off), s2 = __shfl_xor_sync(0xffffffffu, src, off);
    if (ranks_before(m2, a2, m, a)) {
      m = m2;
      a = a2;
      src = s2;
    }
  }
}

// One CTA per (image, gt slot).  Each thread keeps its own sorted top-10 of the candidates it visits; each warp
// then takes the best 10 of its 32 lists (10 rounds of a warp arg-best, the winning lane advancing its list),
// and warp 0 the best `topk` of the 8 warps' lists the same way.
__global__ void __launch_bounds__(kDlT) k_dl_topk(const Levels L, int A, int G, int topk, const int* n_gt,
                                                 const float4* gt_box, const float4* pbox, const float* score,
                                                 int* cnt, int* who, float* galign, float* govl) {
  __shared__ float s_m[kDlT / 32][kDlTopK];
  __shared__ int s_a[kDlT / 32][kDlTopK];
  const int bj = blockIdx.x, b = bj / G, j = bj - b * G;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    galign[bj] = 0.f;
    govl[bj] = 0.f;
  }
  if (j >= n_gt[b]) return;
  const float4 g = gt_box[bj], e = enlarged(g);
  float tm[kDlTopK];
  int ta[kDlTopK];
#pragma unroll
  for (int k = 0; k < kDlTopK; k++) {
    tm[k] = -1.f;
    ta[k] = -1;
  }
  for (int l = 0; l < 3; l++) {
    const float s = (float)L.s[l];
    const int x0 = max(0, (int)floorf(e.x / s - 0.5f)), x1 = min(L.w[l] - 1, (int)ceilf(e.z / s - 0.5f));
    const int y0 = max(0, (int)floorf(e.y / s - 0.5f)), y1 = min(L.h[l] - 1, (int)ceilf(e.w / s - 0.5f));
    const int nx = x1 - x0 + 1, ny = y1 - y0 + 1;
    if (nx <= 0 || ny <= 0) continue;
    for (int t = tid; t < nx * ny; t += kDlT) {
      const int yy = y0 + t / nx, xx = x0 + t % nx;
      if (!centre_in(e, (xx + 0.5f) * s, (yy + 0.5f) * s)) continue;
      const int a = L.off[l] + yy * L.w[l] + xx;
      const long long q = (long long)b * A + a;
      const float4 pb = pbox[q];
      const float ov = fmaxf(ciou_of(g, make_float4(pb.x * s, pb.y * s, pb.z * s, pb.w * s), nullptr), 0.f);
      const float m = align_metric(score[q], ov);
      if (!ranks_before(m, a, tm[kDlTopK - 1], ta[kDlTopK - 1])) continue;
      int k = kDlTopK - 1;  // sorted insertion
      while (k > 0 && ranks_before(m, a, tm[k - 1], ta[k - 1])) {
        tm[k] = tm[k - 1];
        ta[k] = ta[k - 1];
        k--;
      }
      tm[k] = m;
      ta[k] = a;
    }
  }
  // warp level: the best 10 of the warp's 32 sorted lists
  int head = 0;
  for (int r = 0; r < kDlTopK; r++) {
    float m = -1.f;
    int a = -1;
#pragma unroll
    for (int k = 0; k < kDlTopK; k++)
      if (k == head) {
        m = tm[k];
        a = ta[k];
      }
    int src = lane;
    warp_best(m, a, src);
    if (lane == src && a >= 0) head++;
    if (lane == 0) {
      s_m[warp][r] = m;
      s_a[warp][r] = a;
    }
  }
  __syncthreads();
  if (warp != 0) return;
  // block level: the best `topk` of the warps' sorted lists; lanes 0..7 hold the heads
  int wh = 0;
  for (int r = 0; r < topk; r++) {
    const bool own = lane < kDlT / 32 && wh < kDlTopK;
    float m = own ? s_m[lane][wh] : -1.f;
    int a = own ? s_a[lane][wh] : -1;
    int src = lane;
    warp_best(m, a, src);
    if (a < 0) break;
    if (lane == src) wh++;
    if (lane == 0) {
      atomicAdd(&cnt[(long long)b * A + a], 1);
      who[(long long)b * A + a] = j;
    }
  }
}

// ------------------------------------------------------------------------------------------------ 3. resolve
__global__ void __launch_bounds__(kDlT) k_dl_resolve(const Levels L, int A, int B, int G, const int* n_gt,
                                                    const float4* gt_box, const float4* pbox, const float* score,
                                                    int* cnt, const int* who, int* agt, float* amet, float* aovl,
                                                    float* galign, float* govl) {
  const long long q = (long long)blockIdx.x * kDlT + threadIdx.x;
  if (q >= (long long)B * A) return;
  const int c = cnt[q];
  if (c == 0) {
    agt[q] = -1;
    return;
  }
  const int b = (int)(q / A), a = (int)(q - (long long)b * A);
  int l, y, x;
  level_of(L, a, l, y, x);
  const float s = (float)L.s[l], px = (x + 0.5f) * s, py = (y + 0.5f) * s;
  const float4 pb = pbox[q], pp = make_float4(pb.x * s, pb.y * s, pb.z * s, pb.w * s);
  int j = who[q];
  if (c > 1) {  // chosen by several: the gt it overlaps most (the first maximum); outside a gt's box the overlap is 0
    float best = -1.f;
    for (int k = 0; k < n_gt[b]; k++) {
      const float4 g = gt_box[(long long)b * G + k];
      const float ov = centre_in(enlarged(g), px, py) ? fmaxf(ciou_of(g, pp, nullptr), 0.f) : 0.f;
      if (ov > best) {
        best = ov;
        j = k;
      }
    }
  }
  const float4 g = gt_box[(long long)b * G + j];
  float ov = 0.f, m = 0.f;
  if (centre_in(enlarged(g), px, py)) {
    ov = fmaxf(ciou_of(g, pp, nullptr), 0.f);
    m = align_metric(score[q], ov);
  }
  agt[q] = j;
  amet[q] = m;
  aovl[q] = ov;
  // non-negative floats order like their bit patterns
  atomicMax(reinterpret_cast<int*>(&galign[(long long)b * G + j]), __float_as_int(m));
  atomicMax(reinterpret_cast<int*>(&govl[(long long)b * G + j]), __float_as_int(ov));
}

// ------------------------------------------------------------------------------------------------ 4. positives
// One CTA per image: the positives in anchor order (each thread a contiguous run of anchors, a block scan of
// the counts), the target scores (0 for negatives) and their sum.
constexpr int kDlPosT = 1024;
__global__ void __launch_bounds__(kDlPosT) k_dl_positives(int A, int G, const int* agt, const float* amet,
                                                         const float* galign, const float* govl, float* tsc,
                                                         int* npos, int* pos, float* items) {
  __shared__ int s_cnt[kDlPosT];
  __shared__ float s_t[kDlPosT / 32];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int per = (A + kDlPosT - 1) / kDlPosT, a0 = tid * per, a1 = min(A, a0 + per);
  const long long base = (long long)b * A;
  int c = 0;
  float tsum = 0.f;
  for (int a = a0; a < a1; a++) {
    const int j = agt[base + a];
    float t = 0.f;
    if (j >= 0) {
      c++;
      t = amet[base + a] * govl[(long long)b * G + j] / (galign[(long long)b * G + j] + kTalEps);
      tsum += t;
    }
    tsc[base + a] = t;
  }
  s_cnt[tid] = c;
  __syncthreads();
  for (int off = 1; off < kDlPosT; off <<= 1) {  // inclusive scan (Hillis–Steele)
    const int v = tid >= off ? s_cnt[tid - off] : 0;
    __syncthreads();
    s_cnt[tid] += v;
    __syncthreads();
  }
  int k = s_cnt[tid] - c;
  for (int a = a0; a < a1; a++)
    if (agt[base + a] >= 0) pos[base + k++] = a;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) tsum += __shfl_down_sync(0xffffffffu, tsum, off);
  if ((tid & 31) == 0) s_t[tid >> 5] = tsum;
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    for (int w = 0; w < kDlPosT / 32; w++) t += s_t[w];
    const int n = s_cnt[kDlPosT - 1];
    npos[b] = n;
    atomicAdd(&items[4], (float)n);
    if (t != 0.f) atomicAdd(&items[5], t);
  }
}

// ------------------------------------------------------------------------------------------------ 5. loss
struct LossArgs {
  Levels L;
  int A, B, G, imgsz, Hp, Wp;
  const __half* box[3];
  const __half* cls[3];
  __half* dbox[3];
  __half* dcls[3];
  __half* dcoef[3];
  const int* agt;
  const float* tsc;
  const float4* gt_box;
  const uint32_t* ignore;  // [B][Hp·Wp/32] bits, or null
  float* items;
  const float* scale;
  float box_gain, cls_gain, dfl_gain;
};

__device__ __forceinline__ void block_sum_to(float v, float* dst) {
  __shared__ float red[kDlT / 32];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = threadIdx.x < kDlT / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0 && v != 0.f) atomicAdd(dst, v);
  }
  __syncthreads();
}

__device__ __forceinline__ void store8h(__half* p, const float* v) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

template <int REG>
__global__ void __launch_bounds__(kDlT) k_dl_loss(const LossArgs P) {
  const long long q = (long long)blockIdx.x * kDlT + threadIdx.x;
  float lcls = 0.f, liou = 0.f, ldfl = 0.f;
  if (q < (long long)P.B * P.A) {
    const int b = (int)(q / P.A), a = (int)(q - (long long)b * P.A);
    int l, y, x;
    level_of(P.L, a, l, y, x);
    const long long pix = ((long long)b * P.L.h[l] + y) * P.L.w[l] + x;
    // gradients of (Σ items)·B, items normalised by the target-score sum, times the loss scale
    const float sc = (float)P.B / fmaxf(P.items[5], 1.f) * *P.scale;
    const int j = P.agt[q];
    const float t = j >= 0 ? P.tsc[q] : 0.f;
    const float xl = __half2float(P.cls[l][pix]);
    bool ign = false;
    if (j < 0 && P.ignore) {  // a negative whose centre lies in the ignore region: no class loss
      const int cs = P.imgsz / P.Wp;
      const int cx = min(P.Wp - 1, (int)((x + 0.5f) * P.L.s[l]) / cs);
      const int cy = min(P.Hp - 1, (int)((y + 0.5f) * P.L.s[l]) / cs);
      const long long bit = (long long)cy * P.Wp + cx;
      ign = (P.ignore[(long long)b * (P.Hp * P.Wp / 32) + (bit >> 5)] >> (bit & 31)) & 1u;
    }
    lcls = ign ? 0.f : bce(xl, t);
    P.dcls[l][pix] = __float2half_rn(ign ? 0.f : (sigmoid(xl) - t) * P.cls_gain * sc);
    __half* db = P.dbox[l] + pix * 4 * REG;
    if (j < 0) {
      const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < 4 * REG; k += 8) store8h(db + k, z);
#pragma unroll
      for (int k = 0; k < 32; k += 8) store8h(P.dcoef[l] + pix * 32 + k, z);
    } else {
      const __half* bl = P.box[l] + pix * 4 * REG;
      float pr[4][REG], dist[4];
#pragma unroll
      for (int s = 0; s < 4; s++) {
        float m = -INFINITY;
#pragma unroll
        for (int k = 0; k < REG; k++) {
          pr[s][k] = __half2float(bl[s * REG + k]);
          m = fmaxf(m, pr[s][k]);
        }
        float z = 0.f;
#pragma unroll
        for (int k = 0; k < REG; k++) {
          pr[s][k] = expf(pr[s][k] - m);
          z += pr[s][k];
        }
        float e = 0.f;
#pragma unroll
        for (int k = 0; k < REG; k++) {
          pr[s][k] /= z;
          e += pr[s][k] * k;
        }
        dist[s] = e;
      }
      const float st = (float)P.L.s[l];
      const float ax = x + 0.5f, ay = y + 0.5f;
      const float4 pb = make_float4(ax - dist[0], ay - dist[1], ax + dist[2], ay + dist[3]);
      const float4 tg = P.gt_box[(long long)b * P.G + j];
      const float4 tb = make_float4(tg.x / st, tg.y / st, tg.z / st, tg.w / st);
      float4 gb;
      const float ci = ciou_of(pb, tb, &gb);
      liou = (1.f - ci) * t;
      const float gi = -t * P.box_gain * sc;                             // d loss / d CIoU
      const float dd[4] = {-gb.x * gi, -gb.y * gi, gb.z * gi, gb.w * gi};  // d loss / d (left, top, right, bottom)
      const float tl[4] = {ax - tb.x, ay - tb.y, tb.z - ax, tb.w - ay};   // target distances
      const float gd = t * 0.25f * P.dfl_gain * sc;
      float g[4][REG];
#pragma unroll
      for (int s = 0; s < 4; s++) {
        const float tt = fminf(fmaxf(tl[s], 0.f), REG - 1 - 0.01f);
        const int il = (int)tt, ir = il + 1;
        const float wl = ir - tt, wr = 1.f - wl;
        ldfl += -(logf(pr[s][il]) * wl + logf(pr[s][ir]) * wr) * 0.25f * t;
#pragma unroll
        for (int k = 0; k < REG; k++) {
          const float p = pr[s][k];
          g[s][k] = dd[s] * p * (k - dist[s]) + gd * (p - (k == il ? wl : 0.f) - (k == ir ? wr : 0.f));
        }
      }
#pragma unroll
      for (int k = 0; k < 4 * REG; k += 8) store8h(db + k, &g[0][0] + k);
    }
  }
  block_sum_to(lcls, &P.items[10]);
  block_sum_to(liou, &P.items[8]);
  block_sum_to(ldfl, &P.items[11]);
}

__global__ void k_dl_items(float* items, float box_gain, float cls_gain, float dfl_gain) {
  const float tss = fmaxf(items[5], 1.f), fg = items[4];
  items[0] = items[8] / tss * box_gain;
  items[1] = fg > 0.f ? items[9] / fg * box_gain : 0.f;
  items[2] = items[10] / tss * cls_gain;
  items[3] = items[11] / tss * dfl_gain;
}

// workspace: pbox [B·A] float4, score, amet, aovl [B·A] float, cnt, who [B·A] int, galign, govl [B·G] float
struct DlWs {
  float4* pbox;
  float *score, *amet, *aovl, *galign, *govl;
  int *cnt, *who;
};
size_t al256(size_t n) { return (n + 255) & ~size_t(255); }
size_t dl_ws_bytes(int B, int A, int G) {
  const size_t BA = (size_t)B * A, BG = (size_t)B * G;
  return al256(BA * 16) + 3 * al256(BA * 4) + 2 * al256(BA * 4) + 2 * al256(BG * 4);
}
DlWs dl_ws(void* ws, int B, int A, int G) {
  const size_t BA = (size_t)B * A, BG = (size_t)B * G;
  char* p = static_cast<char*>(ws);
  DlWs w;
  w.pbox = reinterpret_cast<float4*>(p);
  p += al256(BA * 16);
  w.score = reinterpret_cast<float*>(p);
  p += al256(BA * 4);
  w.amet = reinterpret_cast<float*>(p);
  p += al256(BA * 4);
  w.aovl = reinterpret_cast<float*>(p);
  p += al256(BA * 4);
  w.cnt = reinterpret_cast<int*>(p);  // zeroed by every call
  p += al256(BA * 4);
  w.who = reinterpret_cast<int*>(p);
  p += al256(BA * 4);
  w.galign = reinterpret_cast<float*>(p);
  p += al256(BG * 4);
  w.govl = reinterpret_cast<float*>(p);
  return w;
}

int dl_fail(int code, const char* msg) {
  set_last_error("%s", msg);
  return code;
}

}  // namespace
}  // namespace osam

using namespace osam;

extern "C" {

size_t osam_det_loss_workspace_size(int batch, int anchors, int max_gt) {
  return batch > 0 && anchors > 0 && max_gt > 0 ? dl_ws_bytes(batch, anchors, max_gt) : 0;
}

int osam_det_loss(const void* const* box, const void* const* cls, const int* level_hw, int batch, int imgsz,
                  int reg_max, const int* n_gt, const float* gt_box, int max_gt, const uint32_t* ignore, int proto_h,
                  int proto_w, const float* scale, float box_gain, float cls_gain, float dfl_gain, void* const* dbox,
                  void* const* dcls, void* const* dcoef, int* agt, float* tsc, int* npos, int* pos, float* items,
                  void* ws, size_t ws_bytes, osam_stream_t stream) {
  if (!box || !cls || !level_hw || !n_gt || !gt_box || !scale || !dbox || !dcls || !dcoef || !agt || !tsc || !npos ||
      !pos || !items || batch < 1 || max_gt < 1 || imgsz < 32)
    return dl_fail(OSAM_ERR_INVALID, "osam_det_loss: invalid arguments");
  if (reg_max != 16) return dl_fail(OSAM_ERR_UNSUPPORTED, "osam_det_loss: reg_max 16 only");
  if (ignore && (proto_h < 1 || proto_w < 1 || (proto_h * proto_w) % 32 || imgsz % proto_w))
    return dl_fail(OSAM_ERR_INVALID, "osam_det_loss: ignore bits need the proto grid (H·W % 32 == 0)");
  Levels L{};
  L.off[0] = 0;
  for (int l = 0; l < 3; l++) {
    L.h[l] = level_hw[2 * l];
    L.w[l] = level_hw[2 * l + 1];
    if (L.h[l] < 1 || L.w[l] < 1 || imgsz % L.w[l]) return dl_fail(OSAM_ERR_INVALID, "osam_det_loss: level sizes");
    L.s[l] = imgsz / L.w[l];
    L.off[l + 1] = L.off[l] + L.h[l] * L.w[l];
    if (!box[l] || !cls[l] || !dbox[l] || !dcls[l] || !dcoef[l]) return dl_fail(OSAM_ERR_INVALID, "osam_det_loss: null head");
    if ((reinterpret_cast<uintptr_t>(box[l]) | reinterpret_cast<uintptr_t>(dbox[l]) |
         reinterpret_cast<uintptr_t>(dcoef[l])) & 15)
      return dl_fail(OSAM_ERR_INVALID, "osam_det_loss: box / coefficient heads must be 16-byte aligned");
  }
  const int A = L.off[3];
  if ((long long)batch * A >= (1LL << 31)) return dl_fail(OSAM_ERR_UNSUPPORTED, "osam_det_loss: too many anchors");
  if (!ws || ws_bytes < dl_ws_bytes(batch, A, max_gt) || (reinterpret_cast<uintptr_t>(ws) & 255))
    return dl_fail(OSAM_ERR_INVALID, "osam_det_loss: workspace (osam_det_loss_workspace_size, 256-byte aligned)");
  const DlWs w = dl_ws(ws, batch, A, max_gt);
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  Heads H{};
  for (int l = 0; l < 3; l++) {
    H.box[l] = static_cast<const __half*>(box[l]);
    H.cls[l] = static_cast<const __half*>(cls[l]);
  }
  const long long BA = (long long)batch * A;
  const int nq = (int)((BA + kDlT - 1) / kDlT);
  cudaMemsetAsync(items, 0, 16 * sizeof(float), st);
  // the per-anchor selection counts start at zero (the rest of the workspace is written before it is read)
  cudaMemsetAsync(w.cnt, 0, (size_t)BA * sizeof(int), st);
  LossArgs P{};
  P.L = L;
  P.A = A;
  P.B = batch;
  P.G = max_gt;
  P.imgsz = imgsz;
  P.Hp = proto_h;
  P.Wp = proto_w;
  for (int l = 0; l < 3; l++) {
    P.box[l] = H.box[l];
    P.cls[l] = H.cls[l];
    P.dbox[l] = static_cast<__half*>(dbox[l]);
    P.dcls[l] = static_cast<__half*>(dcls[l]);
    P.dcoef[l] = static_cast<__half*>(dcoef[l]);
  }
  P.agt = agt;
  P.tsc = tsc;
  P.gt_box = reinterpret_cast<const float4*>(gt_box);
  P.ignore = ignore;
  P.items = items;
  P.scale = scale;
  P.box_gain = box_gain;
  P.cls_gain = cls_gain;
  P.dfl_gain = dfl_gain;
  k_dl_decode<16><<<nq, kDlT, 0, st>>>(L, A, batch, H, w.pbox, w.score);
  k_dl_topk<<<batch * max_gt, kDlT, 0, st>>>(L, A, max_gt, kDlTopK, n_gt, P.gt_box, w.pbox, w.score, w.cnt, w.who,
                                             w.galign, w.govl);
  k_dl_resolve<<<nq, kDlT, 0, st>>>(L, A, batch, max_gt, n_gt, P.gt_box, w.pbox, w.score, w.cnt, w.who, agt, w.amet,
                                    w.aovl, w.galign, w.govl);
  k_dl_positives<<<batch, kDlPosT, 0, st>>>(A, max_gt, agt, w.amet, w.galign, w.govl, tsc, npos, pos, items);
  k_dl_loss<16><<<nq, kDlT, 0, st>>>(P);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OSAM_OK : dl_fail(OSAM_ERR_CUDA, cudaGetErrorString(e));
}

int osam_seg_loss_items(float* items, float box_gain, float cls_gain, float dfl_gain, osam_stream_t stream) {
  if (!items) return dl_fail(OSAM_ERR_INVALID, "osam_seg_loss_items: null items");
  k_dl_items<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(items, box_gain, cls_gain, dfl_gain);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OSAM_OK : dl_fail(OSAM_ERR_CUDA, cudaGetErrorString(e));
}

}  // extern "C"
