// Inference post-process on the GPU: DFL decode, stable score sort + greedy NMS, and the mask assembly
// (coef · proto on the tensor cores, fused with the logit > 0 test and the box crop).
//
// Semantics follow the reference's only inference post-process, archive/tools/ref_detect.py:37-81, for an
// unpadded S×S input, and its DFL decode (src/loss.cu:128-147):
//   decode   per anchor (levels 8/16/32, row-major cells): softmax expectation of each side's reg_max bins,
//            x1 = ax − l, y1 = ay − t, x2 = ax + r, y2 = ay + b (anchor = cell + 0.5), xywh = ((x1+x2)/2,
//            (y1+y2)/2, x2−x1, y2−y1)·stride — the exported head — and back to xyxy as ref_detect does
//            (cx − w/2, …); conf = sigmoid(cls).
//   NMS      candidates conf > conf_th in stable descending-conf order (ties: lower anchor first); greedy:
//            a candidate is dropped when IoU > nms_iou (strict, and only if union > 0) with a kept box;
//            stop at max_det.  IoU is evaluated with explicitly rounded fp32 operations in ref_detect's
//            order, so the kept indices are bit-exact given the same boxes and scores.
//   masks    logits = coef[kept] (n × 32) · proto (32 × Hp·Wp); mask = logit > 0 (≡ sigmoid > 0.5)
//            ∩ the box scaled to the proto grid (x ≥ x1·g, x < x2·g, y ≥ y1·g, y < y2·g, g = Wp / S).
#include "epilogue.cuh"

#include <algorithm>
#include <cstring>
#include <cmath>

namespace osam {

struct DecodeArgs {
  const __half* box[3];
  const __half* cls[3];
  int h[3], w[3], stride[3];
  int A;        // anchors per image
  int reg_max;  // DFL bins (box channels = 4·reg_max)
  float* xyxy;  // [B][A][4]
  float* conf;  // [B][A]
  int B;
};

__global__ void k_decode(const DecodeArgs a) {
  const long long gid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (gid >= (long long)a.B * a.A) return;
  const int b = (int)(gid / a.A), an = (int)(gid - (long long)b * a.A);
  // level by anchor range; the per-level fields are picked with selects (no dynamic parameter indexing)
  const int n0 = a.h[0] * a.w[0], n1 = a.h[1] * a.w[1];
  const int l = an < n0 ? 0 : (an < n0 + n1 ? 1 : 2);
  const int rem = an - (l == 0 ? 0 : (l == 1 ? n0 : n0 + n1));
  const int lh = l == 0 ? a.h[0] : (l == 1 ? a.h[1] : a.h[2]);
  const int lw = l == 0 ? a.w[0] : (l == 1 ? a.w[1] : a.w[2]);
  const int lstride = l == 0 ? a.stride[0] : (l == 1 ? a.stride[1] : a.stride[2]);
  const __half* lbox = l == 0 ? a.box[0] : (l == 1 ? a.box[1] : a.box[2]);
  const __half* lcls = l == 0 ? a.cls[0] : (l == 1 ? a.cls[1] : a.cls[2]);
  const int cy = rem / lw, cx = rem - cy * lw;
  const long long pix = ((long long)b * lh + cy) * lw + cx;
  const __half* p = lbox + pix * 4 * a.reg_max;
  float d[4];
  if (a.reg_max == 16) {  // 4 sides × 16 bins = eight 16-byte loads
    const uint4* p4 = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int s = 0; s < 4; s++) {
      float v[16];
      unpack8h(p4[2 * s], v);
      unpack8h(p4[2 * s + 1], v + 8);
      float mx = v[0];
#pragma unroll
      for (int k = 1; k < 16; k++) mx = fmaxf(mx, v[k]);
      float z = 0.f, e = 0.f;
#pragma unroll
      for (int k = 0; k < 16; k++) {
        const float t = __expf(v[k] - mx);
        z += t;
        e += t * (float)k;
      }
      d[s] = e / z;
    }
  } else {
#pragma unroll
    for (int s = 0; s < 4; s++) {
      float mx = -INFINITY;
      for (int k = 0; k < a.reg_max; k++) mx = fmaxf(mx, __half2float(p[s * a.reg_max + k]));
      float z = 0.f, e = 0.f;
      for (int k = 0; k < a.reg_max; k++) {
        const float t = __expf(__half2float(p[s * a.reg_max + k]) - mx);
        z += t;
        e += t * (float)k;
      }
      d[s] = e / z;
    }
  }
  const float ax = (float)cx + 0.5f, ay = (float)cy + 0.5f, st = (float)lstride;
  const float x1 = __fsub_rn(ax, d[0]), y1 = __fsub_rn(ay, d[1]);
  const float x2 = __fadd_rn(ax, d[2]), y2 = __fadd_rn(ay, d[3]);
  // exported xywh (dist2bbox) × stride, then ref_detect's xywh → xyxy
  const float cxw = __fmul_rn(__fdiv_rn(__fadd_rn(x1, x2), 2.f), st);
  const float cyw = __fmul_rn(__fdiv_rn(__fadd_rn(y1, y2), 2.f), st);
  const float ww = __fmul_rn(__fsub_rn(x2, x1), st), hh = __fmul_rn(__fsub_rn(y2, y1), st);
  float4 o;
  o.x = __fsub_rn(cxw, __fdiv_rn(ww, 2.f));
  o.y = __fsub_rn(cyw, __fdiv_rn(hh, 2.f));
  o.z = __fadd_rn(cxw, __fdiv_rn(ww, 2.f));
  o.w = __fadd_rn(cyw, __fdiv_rn(hh, 2.f));
  reinterpret_cast<float4*>(a.xyxy)[gid] = o;
  const float c = __half2float(lcls[pix]);
  a.conf[gid] = 1.f / (1.f + expf(-c));
}

// --------------------------------------------------------------------------------------------- NMS
struct NmsArgs {
  const float* xyxy;   // [B][A][4]
  const float* conf;   // [B][A]
  int A;               // anchors per image (< 65536: shared order arrays hold 16-bit anchor ids)
  float conf_th;
  int max_det;
  int forced;          // 1: no threshold and no suppression — the max_det highest scores
  int* n_det;          // [B]
  int* keep;           // [B][max_det] anchor indices, in score order
  float* det_box;      // [B][max_det][4] xyxy px
  float* det_score;    // [B][max_det]
  // coefficient gather for the mask GEMM: coef[l] NHWC (32 ch), level geometry
  const __half* coef[3];
  int h[3], w[3];
  __half* coef_g;      // [B][max_det_pad][32]
  int max_det_pad;
  int mblk;            // survivors per suppression-matrix block (512, 256 or 128: what shared memory holds)
  // the IoU threshold as an exact test (see iou_gt)
  float thr;           // iou_th
  float thr_h;         // half the gap from iou_th to the next float (a power of two)
  int thr_fast;        // iou_th finite in [1e-3, 1e3]: iou_gt's single-rounding pre-test applies
  double thr_mid;      // midpoint between iou_th and the next float above it
  int thr_odd;         // iou_th's last significand bit (a quotient exactly at thr_mid rounds up iff set)
  int thr_nonneg;      // iou_th ≥ 0: disjoint boxes (IoU 0) never pass
  int thr_nan;         // iou_th is NaN: nothing passes
  int smem_sort;       // byte offset of the phase-shared region in dynamic shared memory
};

// ref_detect's IoU test: RN(inter / union) > thr, with inter and union rounded as numpy's float32 ops round
// them (b = candidate, c = kept box, ab / ac their areas, computed as (x2 − x1)·(y2 − y1)).  The rounded
// quotient exceeds thr exactly when the real quotient exceeds the midpoint m = thr + h between thr and the
// next float, or equals m and round-to-even picks the upper neighbour (thr's last bit is 1); with union > 0
// that is D = inter − union·thr > union·h.  D is first formed with one rounding (an FMA, relative error
// ≤ 2⁻²⁴), which settles every pair farther than a factor 2 from the boundary; the rest are decided by
// inter > union·m in double, where the 24-bit × 25-bit product is exact.  No division is needed.
__device__ __forceinline__ bool iou_gt_exact(float inter, float u, const NmsArgs& a) {
  if (inter == 0.f && a.thr_nonneg) return false;
  if (!(u > 0.f) || a.thr_nan) return false;
  const double p = __dmul_rn((double)u, a.thr_mid), in = (double)inter;
  return in > p || (in == p && a.thr_odd);
}

__device__ __forceinline__ bool iou_gt(const float4 b, float ab, const float4 c, float ac, const NmsArgs& a) {
  const float iw = fmaxf(0.f, __fsub_rn(fminf(b.z, c.z), fmaxf(b.x, c.x)));
  const float ih = fmaxf(0.f, __fsub_rn(fminf(b.w, c.w), fmaxf(b.y, c.y)));
  const float inter = __fmul_rn(iw, ih);
  const float u = __fsub_rn(__fadd_rn(ab, ac), inter);
  const float dd = __fmaf_rn(-u, a.thr, inter);
  const float uh = __fmul_rn(u, a.thr_h);
  const bool above = dd > 2.f * uh, below = dd < 0.5f * uh;
  if (a.thr_fast && u >= 1e-20f && u <= 1e30f && (above || below)) return above;
  return iou_gt_exact(inter, u, a);
}

__device__ __forceinline__ float box_area(const float4 b) { return __fmul_rn(__fsub_rn(b.z, b.x), __fsub_rn(b.w, b.y)); }

// Sort key whose ascending order is numpy's stable argsort of −conf: descending conf, NaN last, −0 = +0.
__device__ __forceinline__ uint32_t desc_key(float c) {
  if (c != c) return 0xFFFFFFFFu;
  if (c == 0.f) c = 0.f;
  uint32_t u = __float_as_uint(c);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // monotone in the float's value
  return ~u;
}

constexpr int kNmsThreads = 1024;
constexpr int kNmsWarps = kNmsThreads / 32;
constexpr int kRadixBins = 256;  // 8-bit digits

// Exclusive block-wide prefix sum of one int per thread; `tot` holds ≥ 33 ints.  All threads must call it.
__device__ __forceinline__ int block_scan_excl(int v, int* tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int t = tot[lane];
    int ti = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, ti, o);
      if (lane >= o) ti += x;
    }
    tot[lane] = ti - t;
    if (lane == 31) tot[32] = ti;
  }
  __syncthreads();
  const int r = tot[warp] + incl - v;
  *total = tot[32];
  __syncthreads();
  return r;
}

// One CTA per image.
//  (0) the candidates (conf > conf_th, or every anchor when forced) are compacted in anchor order;
//  (1) a stable LSD radix sort (8-bit digits of desc_key, only as many passes as the keys' range needs)
//      puts them in numpy's stable descending-conf order.  Each warp owns a contiguous segment and ranks
//      32 elements per step with __match_any_sync, so ties keep anchor order;
//  (2) greedy NMS in rounds of 1024 sorted candidates: every thread tests its candidate against the boxes
//      kept before the round and the survivors are compacted in order; then, per block of `mblk`
//      survivors, the whole CTA tests the block against the boxes kept earlier in the round and fills the
//      block's suppression bit-matrix (row i: survivors j > i whose IoU with i passes), and warp 0 walks
//      the block in order, keeping the first survivor not yet removed and OR-ing its row into the removed
//      set — one step per kept box.  This keeps exactly the boxes of the sequential greedy loop.
__global__ void __launch_bounds__(kNmsThreads, 1) k_nms(const NmsArgs a) {
  extern __shared__ __align__(16) uint8_t nsm[];
  unsigned short* ord0 = reinterpret_cast<unsigned short*>(nsm);  // [A] candidate anchors
  unsigned short* ord1 = ord0 + a.A;                               // [A] radix ping-pong buffer
  uint8_t* ph = nsm + a.smem_sort;                                  // phase-shared region
  // sort phase
  uint32_t* key_of = reinterpret_cast<uint32_t*>(ph);              // [A] desc_key by anchor
  uint32_t* cnt = key_of + ((a.A + 3) & ~3);                        // [kRadixBins][kNmsWarps]
  // greedy phase
  float4* kept = reinterpret_cast<float4*>(ph);                     // [max_det]
  float* kept_area = reinterpret_cast<float*>(kept + a.max_det);    // [max_det]
  int* kept_src = reinterpret_cast<int*>(kept_area + ((a.max_det + 3) & ~3));  // [max_det] survivor slot
  float4* surv_box = reinterpret_cast<float4*>(kept_src + ((a.max_det + 3) & ~3));  // [kNmsThreads]
  float* surv_area = reinterpret_cast<float*>(surv_box + kNmsThreads);                // [kNmsThreads]
  int* surv_an = reinterpret_cast<int*>(surv_area + kNmsThreads);                     // [kNmsThreads]
  uint32_t* mat = reinterpret_cast<uint32_t*>(surv_an + kNmsThreads);                 // [mblk][mblk / 32]
  __shared__ int tot[33], nkept;
  __shared__ uint32_t kmin_s, kmax_s, blk_dead[kNmsWarps];
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned lt = (1u << lane) - 1u;
  const float* conf = a.conf + (long long)b * a.A;
  const float4* box = reinterpret_cast<const float4*>(a.xyxy) + (long long)b * a.A;
  if (tid == 0) {
    nkept = 0;
    kmin_s = 0xFFFFFFFFu;
    kmax_s = 0u;
  }
  // (0) order-preserving compaction
  int nc = 0;
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
  for (int base = 0; base < a.A; base += kNmsThreads) {
    const int i = base + tid;
    bool valid = false;
    uint32_t k = 0u;
    if (i < a.A) {
      const float c = conf[i];
      valid = a.forced || c > a.conf_th;
      k = desc_key(c);
    }
    int total;
    const int pos = nc + block_scan_excl(valid ? 1 : 0, tot, &total);
    if (valid) {
      ord0[pos] = (unsigned short)i;
      key_of[i] = k;
      kmin = min(kmin, k);
      kmax = max(kmax, k);
    }
    nc += total;
  }
  kmin = __reduce_min_sync(0xffffffffu, kmin);
  kmax = __reduce_max_sync(0xffffffffu, kmax);
  if (lane == 0) {
    atomicMin(&kmin_s, kmin);
    atomicMax(&kmax_s, kmax);
  }
  __syncthreads();
  kmin = kmin_s;
  kmax = kmax_s;
  // (1) stable LSD radix sort of ord0[0, nc) by key_of
  unsigned short* src = ord0;
  unsigned short* dst = ord1;
  if (nc > 1) {
    const uint32_t range = kmax - kmin;
    const int passes = range ? (32 - __clz(range) + 7) / 8 : 0;
    const int seg = (nc + kNmsWarps - 1) / kNmsWarps;
    const int seg_lo = min(nc, warp * seg), seg_hi = min(nc, seg_lo + seg);
    for (int pass = 0; pass < passes; pass++) {
      const int shift = 8 * pass;
      for (int e = tid; e < kRadixBins * kNmsWarps; e += kNmsThreads) cnt[e] = 0u;
      __syncthreads();
      for (int p0 = seg_lo; p0 < seg_hi; p0 += 32) {  // per-warp digit counts
        const int pos = p0 + lane;
        const bool v = pos < seg_hi;
        const uint32_t d = v ? ((key_of[src[pos]] - kmin) >> shift) & 0xFFu : 0x100u;
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        if (v && (peers & lt) == 0u) cnt[d * kNmsWarps + warp] += __popc(peers);
        __syncwarp();
      }
      __syncthreads();
      {  // exclusive scan of cnt in (digit, warp) order: 8 entries per thread
        constexpr int per = kRadixBins * kNmsWarps / kNmsThreads;
        uint32_t v[per];
        int sum = 0;
#pragma unroll
        for (int q = 0; q < per; q++) {
          v[q] = cnt[tid * per + q];
          sum += (int)v[q];
        }
        int total;
        int run = block_scan_excl(sum, tot, &total);
#pragma unroll
        for (int q = 0; q < per; q++) {
          cnt[tid * per + q] = (uint32_t)run;
          run += (int)v[q];
        }
      }
      __syncthreads();
      for (int p0 = seg_lo; p0 < seg_hi; p0 += 32) {  // stable scatter
        const int pos = p0 + lane;
        const bool v = pos < seg_hi;
        const unsigned short an = v ? src[pos] : (unsigned short)0;
        const uint32_t d = v ? ((key_of[an] - kmin) >> shift) & 0xFFu : 0x100u;
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        uint32_t base = 0u;
        if (v) {
          base = cnt[d * kNmsWarps + warp];
          dst[base + __popc(peers & lt)] = an;
        }
        __syncwarp();
        if (v && (peers & lt) == 0u) cnt[d * kNmsWarps + warp] = base + __popc(peers);
        __syncwarp();
      }
      __syncthreads();
      unsigned short* t = src;
      src = dst;
      dst = t;
    }
  }
  const unsigned short* order = src;
  __syncthreads();  // the sort's shared region becomes the greedy's
  // (2) greedy NMS
  if (a.forced) {
    const int n = nc < a.max_det ? nc : a.max_det;
    for (int i = tid; i < n; i += kNmsThreads) kept[i] = box[order[i]];
    if (tid == 0) nkept = n;
    __syncthreads();
  } else {
    const int mblk = a.mblk, mw = a.mblk / 32;
    for (int r0 = 0; r0 < nc; r0 += kNmsThreads) {
      const int nk0 = nkept;  // uniform: written before the last barrier
      if (nk0 >= a.max_det) break;
      // (a) the round's candidates against every box kept before the round
      const int ci = r0 + tid;
      bool alive = ci < nc;
      int an = 0;
      float4 bx = make_float4(0.f, 0.f, 0.f, 0.f);
      float ab = 0.f;
      if (alive) {
        an = order[ci];
        bx = box[an];
        ab = box_area(bx);
      }
      for (int k = 0; k < nk0 && alive; k += 4) {  // 4 independent tests per step (order-free: any one kills)
        const int k1 = min(k + 1, nk0 - 1), k2 = min(k + 2, nk0 - 1), k3 = min(k + 3, nk0 - 1);
        const bool s0 = iou_gt(bx, ab, kept[k], kept_area[k], a);
        const bool s1 = iou_gt(bx, ab, kept[k1], kept_area[k1], a);
        const bool s2 = iou_gt(bx, ab, kept[k2], kept_area[k2], a);
        const bool s3 = iou_gt(bx, ab, kept[k3], kept_area[k3], a);
        alive = !(s0 || s1 || s2 || s3);
      }
      int ms;
      const int pos = block_scan_excl(alive ? 1 : 0, tot, &ms);
      if (alive) {
        surv_an[pos] = an;
        surv_box[pos] = bx;
        surv_area[pos] = ab;
      }
      __syncthreads();
      for (int s0 = 0; s0 < ms; s0 += mblk) {
        const int nkb = nkept;  // uniform
        if (nkb >= a.max_det) break;
        const int nb = min(mblk, ms - s0), nwb = (nb + 31) / 32;
        // (b) block members against the boxes kept earlier in this round; members past nb count as removed
        if (warp < mw) {
          bool d = tid >= nb;
          if (!d) {
            const float4 me = surv_box[s0 + tid];
            const float ma = surv_area[s0 + tid];
            for (int k = nk0; k < nkb && !d; k += 4) {
              const int k1 = min(k + 1, nkb - 1), k2 = min(k + 2, nkb - 1), k3 = min(k + 3, nkb - 1);
              const bool s0 = iou_gt(me, ma, kept[k], kept_area[k], a);
              const bool s1 = iou_gt(me, ma, kept[k1], kept_area[k1], a);
              const bool s2 = iou_gt(me, ma, kept[k2], kept_area[k2], a);
              const bool s3 = iou_gt(me, ma, kept[k3], kept_area[k3], a);
              d = s0 || s1 || s2 || s3;
            }
          }
          const unsigned dm = __ballot_sync(0xffffffffu, d);
          if (lane == 0) blk_dead[warp] = dm;
        }
        // (c) suppression bit-matrix, upper triangle, one warp per (word w, 32-row group g ≤ w): lane = row,
        //     the 32 columns of word w are read by all lanes at once (shared-memory broadcast)
        const int units = nwb * (nwb + 1) / 2;
        for (int u = warp; u < units; u += kNmsWarps) {
          int w = (int)((sqrtf(8.f * (float)u + 1.f) - 1.f) * 0.5f);
          while ((w + 1) * (w + 2) / 2 <= u) w++;
          while (w * (w + 1) / 2 > u) w--;
          const int g = u - w * (w + 1) / 2;
          const int i = 32 * g + lane;
          const bool row = i < nb;
          const float4 bi = row ? surv_box[s0 + i] : make_float4(0.f, 0.f, 0.f, 0.f);
          const float ai = row ? surv_area[s0 + i] : 0.f;
          uint32_t bits = 0u;
          const int jend = min(32 * w + 32, nb);
#pragma unroll 4
          for (int j = 32 * w; j < jend; j++) {
            const bool s = row && j > i && iou_gt(surv_box[s0 + j], surv_area[s0 + j], bi, ai, a);
            bits |= (s ? 1u : 0u) << (j - 32 * w);
          }
          if (row) mat[i * mw + w] = bits;
        }
        __syncthreads();
        // (d) in-order walk (warp 0): lane w holds removed-word w
        if (warp == 0) {
          uint32_t removed = lane < nwb ? blk_dead[lane] : 0xffffffffu;
          int nk = nkb;
          for (int w = 0; w < nwb && nk < a.max_det; w++) {
            uint32_t live = ~__shfl_sync(0xffffffffu, removed, w);
            while (live != 0u && nk < a.max_det) {
              const int bit = __ffs(live) - 1, i = 32 * w + bit;
              if (lane == 0) kept_src[nk] = s0 + i;  // boxes and outputs are filled in after the walk
              nk++;
              if (lane >= w && lane < nwb) removed |= mat[i * mw + lane];
              const uint32_t above = bit == 31 ? 0u : (0xffffffffu << (bit + 1));
              live = ~__shfl_sync(0xffffffffu, removed, w) & above;
            }
          }
          __syncwarp();
          if (lane == 0) nkept = nk;
        }
        __syncthreads();
        const int nke = nkept;
        for (int t = nkb + tid; t < nke; t += kNmsThreads) {
          const int si = kept_src[t], ai = surv_an[si];
          kept[t] = surv_box[si];
          kept_area[t] = surv_area[si];
          a.keep[(long long)b * a.max_det + t] = ai;
          a.det_score[(long long)b * a.max_det + t] = conf[ai];
        }
        __syncthreads();
      }
    }
  }
  const int n = nkept;
  if (a.forced) {
    for (int i = tid; i < n; i += kNmsThreads) {
      a.keep[(long long)b * a.max_det + i] = order[i];
      a.det_score[(long long)b * a.max_det + i] = conf[order[i]];
    }
  }
  for (int i = tid; i < a.max_det; i += kNmsThreads) {
    const float4 o = i < n ? kept[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    reinterpret_cast<float4*>(a.det_box)[(long long)b * a.max_det + i] = o;
    if (i >= n) {
      a.keep[(long long)b * a.max_det + i] = -1;
      a.det_score[(long long)b * a.max_det + i] = 0.f;
    }
  }
  __syncthreads();
  // gather the kept anchors' mask coefficients (32 fp16 = 4 × 16 B) into the GEMM's A rows
  const int n0 = a.h[0] * a.w[0], n1 = a.h[1] * a.w[1];
  for (int t = tid; t < a.max_det_pad * 4; t += kNmsThreads) {
    const int i = t >> 2, ch = t & 3;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (i < n) {
      const int an = a.keep[(long long)b * a.max_det + i];
      const int l = an < n0 ? 0 : (an < n0 + n1 ? 1 : 2);
      const int rem = an - (l == 0 ? 0 : (l == 1 ? n0 : n0 + n1));
      const int lhw = l == 0 ? n0 : (l == 1 ? n1 : a.h[2] * a.w[2]);
      const __half* lc = l == 0 ? a.coef[0] : (l == 1 ? a.coef[1] : a.coef[2]);
      v = *reinterpret_cast<const uint4*>(lc + ((long long)b * lhw + rem) * 32 + ch * 8);
    }
    *reinterpret_cast<uint4*>(a.coef_g + ((long long)b * a.max_det_pad + i) * 32 + ch * 8) = v;
  }
  if (tid == 0) a.n_det[b] = n;
}

// --------------------------------------------------------------------------------------------- masks
struct MaskArgs {
  const __half* coef_g;  // [B][max_det_pad][32]
  const __half* proto;   // [B][Hp·Wp][32]
  const float* det_box;  // [B][max_det][4]
  const int* n_det;
  uint8_t* masks;        // [B][max_det][Hp·Wp] bytes, or packed bits [B][max_det][ceil32(Hp·Wp)/32] u32
  int packed;            // 1: one bit per pixel (bit k of word j = pixel 32·j + k)
  int Hp, Wp, max_det, max_det_pad;
  float g;               // proto grid units per input pixel (Wp / S)
  int ptiles;            // pixel tiles of kMaskPix per image
  int tiles_per_cta;     // consecutive pixel tiles one CTA walks
  int nsplit;            // CTAs per (image, detection tile) = ceil(ptiles / tiles_per_cta)
  int vec_rows;          // every output row starts 16-byte aligned (16-byte stores allowed)
  int* err;
};

constexpr int kMaskPix = 128;  // pixels per tile = UMMA N = TMEM columns
constexpr int kMaskBufs = 4;   // prototype tile ring: tiles t+1 … t+3 stream in while tile t is computed


// ⌈v⌉ clamped to [lo, hi]; NaN maps to `nan_to` (an empty range, as every comparison with NaN is false).
__device__ __forceinline__ int ceil_clamp(float v, int lo, int hi, int nan_to) {
  if (v != v) return nan_to;
  const float c = ceilf(v);
  return c < (float)lo ? lo : (c > (float)hi ? hi : (int)c);
}

// One CTA = 128 detections (one per thread) × a run of `tiles_per_cta` consecutive 128-pixel tiles of one
// image.  Per tile: two K=16 UMMAs (M=128, N=128) of coef · proto into TMEM while the next three tiles'
// prototypes stream into a four-deep shared ring (cp.async; one tile in flight left the load latency
// exposed at every tile), then each thread turns its detection's 128 logits into
// bits: (logit > 0) ∧ inside the cropped box.  The crop x ≥ x1·g ∧ x < x2·g is tested on integers (for an
// integer x and a float b, x ≥ b ⟺ x ≥ ⌈b⌉ and x < b ⟺ x < ⌈b⌉), one image row per 16-pixel chunk when
// Wp % 16 == 0.  Detection tiles with no live detection only write zeros.  ≤ 128 TMEM columns and ~41 KB
// of shared memory per CTA, so four CTAs share an SM.
__global__ void __launch_bounds__(128, 4) k_mask(const MaskArgs a) {
  __shared__ __align__(1024) uint8_t sA[128 * 64];
  __shared__ __align__(1024) uint8_t sB[kMaskBufs][kMaskPix * 64];
  __shared__ uint64_t bar;
  __shared__ uint32_t tslot;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int dtiles = a.max_det_pad / 128;
  const int sp = blockIdx.x % a.nsplit, rest = blockIdx.x / a.nsplit;
  const int dtile = rest % dtiles, b = rest / dtiles;
  const int ndet = a.n_det[b];
  const int d0 = dtile * 128, npix = a.Hp * a.Wp, nwords = (npix + 31) / 32;
  const int t_begin = sp * a.tiles_per_cta, t_end = min(a.ptiles, t_begin + a.tiles_per_cta);
  const int det = d0 + tid;
  const bool row_out = det < a.max_det;
  const long long row = (long long)b * a.max_det + det;
  uint32_t* outw = reinterpret_cast<uint32_t*>(a.masks) + row * nwords;
  uint8_t* outb = a.masks + row * npix;
  if (t_begin >= t_end) return;

  if (d0 >= ndet) {  // no live detection in this tile: zero the rows' pixel range
    if (!row_out) return;
    if (a.packed) {
      for (int j = t_begin * (kMaskPix / 32); j < min(t_end * (kMaskPix / 32), nwords); j++) outw[j] = 0u;
    } else {
      for (int j = t_begin * kMaskPix; j < min(t_end * kMaskPix, npix); j++) outb[j] = 0;
    }
    return;
  }

  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tslot, kMaskPix);
    tmem_relinquish();
    tc_fence_before();
  }
  // operands: 64-byte K-major rows, 64-byte swizzle (coef rows; proto pixels, zero beyond the image)
  const __half* ca = a.coef_g + ((long long)b * a.max_det_pad + d0) * 32;
  const __half* pimg = a.proto + (long long)b * npix * 32;
#pragma unroll
  for (int q = 0; q < 4; q++) {
    const int r = (tid >> 2) + 32 * q, ch = tid & 3;
    cp_async16(smem_u32(sA + r * 64 + ((ch ^ ((r >> 1) & 3)) << 4)), ca + r * 32 + ch * 8, 16u);
  }
  auto load_b = [&](int t, int buf) {
#pragma unroll
    for (int q = 0; q < kMaskPix / 32; q++) {
      const int r = (tid >> 2) + 32 * q, ch = tid & 3, pix = t * kMaskPix + r;
      const bool in = pix < npix;
      cp_async16(smem_u32(sB[buf] + r * 64 + ((ch ^ ((r >> 1) & 3)) << 4)),
                 pimg + (long long)(in ? pix : 0) * 32 + ch * 8, in ? 16u : 0u);
    }
  };
  // prologue: tiles t_begin … t_begin + kMaskBufs − 2, one commit group each (empty groups past the end
  // keep the count uniform: at tile i, group i is complete once at most kMaskBufs − 2 are pending)
  for (int j = 0; j < kMaskBufs - 1; j++) {
    if (t_begin + j < t_end) load_b(t_begin + j, j);
    cp_async_commit();
  }

  // crop rectangle on the proto grid as integer half-open ranges [xlo, xhi) × [ylo, yhi)
  const bool live = det < ndet;
  int xlo = 0, xhi = 0, ylo = 0, yhi = 0;
  if (live) {
    const float4 o = reinterpret_cast<const float4*>(a.det_box)[row];
    xlo = ceil_clamp(__fmul_rn(o.x, a.g), 0, a.Wp, a.Wp);
    xhi = ceil_clamp(__fmul_rn(o.z, a.g), 0, a.Wp, 0);
    ylo = ceil_clamp(__fmul_rn(o.y, a.g), 0, a.Hp, a.Hp);
    yhi = ceil_clamp(__fmul_rn(o.w, a.g), 0, a.Hp, 0);
  }
  const bool fast = (a.Wp & 15) == 0;
  const bool vec = a.vec_rows != 0;
  const uint32_t trow = (uint32_t)(warp * 32) << 16;  // this warp's 32 TMEM lanes
  bool fail = false;
#pragma unroll 1
  for (int t = t_begin, i = 0; t < t_end; t++, i++) {
    cp_async_wait_n<kMaskBufs - 2>();
    fence_proxy_async_smem();
    if (__syncthreads_or(fail)) break;  // B(t) visible; the previous tile's TMEM reads are done
    tc_fence_after();
    const uint32_t tmem = tslot + trow;
    if (tid == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, kMaskPix);
      const uint32_t sa = smem_u32(sA), sb = smem_u32(sB[i % kMaskBufs]);
      umma_f16(tslot, smem_desc_kmajor(sa, 64), smem_desc_kmajor(sb, 64), idesc, 0);
      umma_f16(tslot, smem_desc_kmajor(sa + 32, 64), smem_desc_kmajor(sb + 32, 64), idesc, 1);
      umma_commit(&bar);
    }
    // buffer (i − 1) mod kMaskBufs was last read by tile t−1's UMMAs, whose commit every thread has waited for
    if (t + kMaskBufs - 1 < t_end) load_b(t + kMaskBufs - 1, (i + kMaskBufs - 1) % kMaskBufs);
    cp_async_commit();
    fail = !mbar_wait(&bar, i & 1, a.err);
    tc_fence_after();
    if (!fail) {
      const int p0 = t * kMaskPix;
      int y = 0, x = 0;
      if (fast) {
        y = p0 / a.Wp;
        x = p0 - y * a.Wp;
      }
      uint32_t words[kMaskPix / 32];
#pragma unroll
      for (int w = 0; w < kMaskPix / 32; w++) {
        uint32_t r0[16], r1[16];
        tmem_ld16_nowait(tmem + 32 * w, r0);
        tmem_ld16_nowait(tmem + 32 * w + 16, r1);
        tmem_wait_ld();
        uint32_t word = 0u;
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const uint32_t* r = h ? r1 : r0;
          const int c0 = p0 + 32 * w + 16 * h;  // first pixel of this chunk
          uint32_t m16 = 0u;
          if (fast) {  // the 16 pixels lie in image row y, columns [x, x + 16)
            // the sign bits of the 16 logits, pixel k at bit k, one funnel shift each (pixel 15 first); a
            // logit counts when its sign bit is clear — logit > 0 except for an exact +0.0, which a sum of
            // 32 products only reaches with a zero coefficient row (dead rows are masked by `live`)
            uint32_t neg = 0u;
#pragma unroll
            for (int k = 15; k >= 0; k--) neg = __funnelshift_l(r[k], neg, 1);
            const uint32_t pos = ~neg & 0xFFFFu;
            const int lo = min(max(xlo - x, 0), 16), hi = min(max(xhi - x, 0), 16);
            const uint32_t cols = hi > lo ? (0xFFFFu >> (16 - hi)) & ~((1u << lo) - 1u) : 0u;
            m16 = (live && y >= ylo && y < yhi && c0 < npix) ? (pos & cols) : 0u;
            x += 16;
            if (x >= a.Wp) {
              x = 0;
              y++;
            }
          } else {
#pragma unroll
            for (int k = 0; k < 16; k++) {
              const int pix = c0 + k, yy = pix / a.Wp, xx = pix - yy * a.Wp;
              const bool m = live && pix < npix && __uint_as_float(r[k]) > 0.f && xx >= xlo && xx < xhi &&
                             yy >= ylo && yy < yhi;
              m16 |= (m ? 1u : 0u) << k;
            }
          }
          word |= m16 << (16 * h);
        }
        words[w] = word;
      }
      if (row_out) {
        if (a.packed) {
          const int j0 = p0 / 32;
          if (vec && j0 + kMaskPix / 32 <= nwords) {
            *reinterpret_cast<uint4*>(outw + j0) = make_uint4(words[0], words[1], words[2], words[3]);
          } else {
            for (int w = 0; w < kMaskPix / 32 && j0 + w < nwords; w++) outw[j0 + w] = words[w];
          }
        } else {
#pragma unroll
          for (int c = 0; c < kMaskPix; c += 16) {
            const uint32_t m16 = (words[c / 32] >> (c & 16)) & 0xFFFFu;
            uint32_t w4[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
              const uint32_t nib = (m16 >> (4 * q)) & 0xFu;
              w4[q] = (nib & 1u) | ((nib >> 1) & 1u) << 8 | ((nib >> 2) & 1u) << 16 | ((nib >> 3) & 1u) << 24;
            }
            if (vec && p0 + c + 16 <= npix) {
              *reinterpret_cast<uint4*>(outb + p0 + c) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            } else {
              for (int k = 0; k < 16 && p0 + c + k < npix; k++) outb[p0 + c + k] = (m16 >> k) & 1u;
            }
          }
        }
      }
    }
    tc_fence_before();
  }
  cp_async_wait_all();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tslot, kMaskPix);
  }
}

}  // namespace osam

using namespace osam;

namespace {
int pp_fail(int code, const char* msg) {
  set_last_error("%s", msg);
  return code;
}
}  // namespace

extern "C" {

int osam_decode(const void* const* box, const void* const* cls, const int* level_hw, int batch, int imgsz,
                int reg_max, float* xyxy, float* conf, osam_stream_t stream) {
  if (!box || !cls || !level_hw || !xyxy || !conf || batch < 1 || imgsz < 32 || reg_max < 1 || reg_max > 64)
    return pp_fail(OSAM_ERR_INVALID, "osam_decode: invalid arguments");
  DecodeArgs a{};
  a.A = 0;
  for (int l = 0; l < 3; l++) {
    a.box[l] = static_cast<const __half*>(box[l]);
    a.cls[l] = static_cast<const __half*>(cls[l]);
    a.h[l] = level_hw[2 * l];
    a.w[l] = level_hw[2 * l + 1];
    if (a.h[l] < 1 || a.w[l] < 1) return pp_fail(OSAM_ERR_INVALID, "osam_decode: level size");
    a.stride[l] = imgsz / a.w[l];
    a.A += a.h[l] * a.w[l];
  }
  a.reg_max = reg_max;
  a.xyxy = xyxy;
  a.conf = conf;
  a.B = batch;
  const long long n = (long long)batch * a.A;
  k_decode<<<(unsigned)((n + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OSAM_OK : pp_fail(OSAM_ERR_CUDA, cudaGetErrorString(e));
}

}  // extern "C"

// the 227 KiB opt-in limit covers static and dynamic shared memory: leave 1 KiB for k_nms's static part
constexpr size_t kNmsSmemMax = 226 * 1024;

static size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

// dynamic shared memory of k_nms: two 16-bit anchor orders, then one region that the sort (keys by anchor,
// radix counters) and the greedy pass (kept boxes and areas, a round's survivors, the bit-matrix) share
static size_t nms_smem_sort_offset(int anchors) { return align16((size_t)anchors * 4); }
static size_t nms_smem_bytes(int anchors, int max_det, int mblk) {
  const size_t md4 = (size_t)((max_det + 3) & ~3);
  const size_t sort = (size_t)((anchors + 3) & ~3) * 4 + (size_t)kRadixBins * kNmsWarps * 4;
  const size_t greedy = (size_t)max_det * 16 + md4 * 8 + (size_t)kNmsThreads * 24 + (size_t)mblk * (mblk / 32) * 4;
  return nms_smem_sort_offset(anchors) + std::max(sort, greedy);
}

// iou_gt's exact form of "RN(q) > thr": the midpoint to the next float up and thr's last significand bit
static void nms_threshold(float thr, NmsArgs& a) {
  a.thr_nan = thr != thr;
  a.thr_nonneg = thr >= 0.f;
  a.thr = thr;
  a.thr_fast = thr >= 1e-3f && thr <= 1e3f;
  const float nx = std::nextafter(thr, INFINITY);
  a.thr_h = a.thr_fast ? (nx - thr) * 0.5f : 0.f;
  const double nxd = std::isinf(nx) && !std::isinf(thr) ? std::ldexp(1.0, 128) : (double)nx;
  a.thr_mid = ((double)thr + nxd) * 0.5;
  uint32_t bits;
  std::memcpy(&bits, &thr, 4);
  a.thr_odd = (int)(bits & 1u);
}

extern "C" {

int osam_nms(const float* xyxy, const float* conf, int batch, int anchors, float conf_th, float iou_th, int max_det,
             int forced, const void* const* coef, const int* level_hw, int* n_det, int* keep, float* det_box,
             float* det_score, void* coef_g, osam_stream_t stream) {
  if (!xyxy || !conf || batch < 1 || anchors < 1 || anchors > 65535 || max_det < 1 || max_det > 1024 || !n_det ||
      !keep || !det_box || !det_score)
    return pp_fail(OSAM_ERR_INVALID, "osam_nms: invalid arguments");
  NmsArgs a{};
  a.xyxy = xyxy;
  a.conf = conf;
  a.A = anchors;
  a.conf_th = conf_th;
  nms_threshold(iou_th, a);
  a.max_det = max_det;
  a.forced = forced;
  a.n_det = n_det;
  a.keep = keep;
  a.det_box = det_box;
  a.det_score = det_score;
  a.max_det_pad = (max_det + 127) / 128 * 128;
  a.coef_g = static_cast<__half*>(coef_g);
  if (coef_g) {
    if (!coef || !level_hw) return pp_fail(OSAM_ERR_INVALID, "osam_nms: coef gather needs coef heads");
    int tot = 0;
    for (int l = 0; l < 3; l++) {
      a.coef[l] = static_cast<const __half*>(coef[l]);
      a.h[l] = level_hw[2 * l];
      a.w[l] = level_hw[2 * l + 1];
      tot += a.h[l] * a.w[l];
    }
    if (tot != anchors) return pp_fail(OSAM_ERR_INVALID, "osam_nms: level sizes do not sum to the anchor count");
  } else {
    a.max_det_pad = 0;
  }
  a.mblk = 512;
  while (a.mblk > 128 && nms_smem_bytes(anchors, max_det, a.mblk) > kNmsSmemMax) a.mblk >>= 1;
  const size_t smem = nms_smem_bytes(anchors, max_det, a.mblk);
  a.smem_sort = (int)nms_smem_sort_offset(anchors);
  if (smem > kNmsSmemMax) return pp_fail(OSAM_ERR_UNSUPPORTED, "osam_nms: too many anchors for one CTA");
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_nms, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kNmsSmemMax);
    if (e != cudaSuccess) return pp_fail(OSAM_ERR_CUDA, cudaGetErrorString(e));
    attr = true;
  }
  k_nms<<<batch, kNmsThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OSAM_OK : pp_fail(OSAM_ERR_CUDA, cudaGetErrorString(e));
}

int osam_mask_assemble(const void* coef_g, const void* proto, const float* det_box, const int* n_det, int batch,
                       int proto_h, int proto_w, int imgsz, int max_det, int packed, void* masks,
                       osam_stream_t stream) {
  if (!coef_g || !proto || !det_box || !n_det || !masks || batch < 1 || proto_h < 1 || proto_w < 1 || max_det < 1)
    return pp_fail(OSAM_ERR_INVALID, "osam_mask_assemble: invalid arguments");
  if ((reinterpret_cast<uintptr_t>(coef_g) | reinterpret_cast<uintptr_t>(proto)) & 15)
    return pp_fail(OSAM_ERR_INVALID, "osam_mask_assemble: operands must be 16-byte aligned");
  MaskArgs a{};
  a.coef_g = static_cast<const __half*>(coef_g);
  a.proto = static_cast<const __half*>(proto);
  a.det_box = det_box;
  a.n_det = n_det;
  a.masks = static_cast<uint8_t*>(masks);
  a.packed = packed;
  a.Hp = proto_h;
  a.Wp = proto_w;
  a.max_det = max_det;
  a.max_det_pad = (max_det + 127) / 128 * 128;
  a.g = (float)proto_w / (float)imgsz;
  a.ptiles = (proto_h * proto_w + kMaskPix - 1) / kMaskPix;
  // about four waves of 4 CTAs per SM, each CTA walking 2..32 consecutive pixel tiles
  const long long pairs = (long long)batch * (a.max_det_pad / 128);
  const long long want = 148LL * 4 * 4;
  a.tiles_per_cta = (int)std::min<long long>(32, std::max<long long>(2, (pairs * a.ptiles + want - 1) / want));
  a.nsplit = (a.ptiles + a.tiles_per_cta - 1) / a.tiles_per_cta;
  const long long row_bytes = packed ? 4LL * ((proto_h * proto_w + 31) / 32) : (long long)proto_h * proto_w;
  a.vec_rows = (row_bytes % 16 == 0) && (reinterpret_cast<uintptr_t>(masks) % 16 == 0);
  a.err = device_error_word();
  if (!a.err) return pp_fail(OSAM_ERR_CUDA, "osam_mask_assemble: device error word");
  const long long grid = pairs * a.nsplit;
  k_mask<<<(unsigned)grid, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OSAM_OK : pp_fail(OSAM_ERR_CUDA, cudaGetErrorString(e));
}

}  // extern "C"
