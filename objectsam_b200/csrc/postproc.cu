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
  int l = 0, rem = an;
  while (l < 2 && rem >= a.h[l] * a.w[l]) {
    rem -= a.h[l] * a.w[l];
    l++;
  }
  const int cy = rem / a.w[l], cx = rem - cy * a.w[l];
  const long long pix = ((long long)b * a.h[l] + cy) * a.w[l] + cx;
  const __half* p = a.box[l] + pix * 4 * a.reg_max;
  float d[4];
  for (int s = 0; s < 4; s++) {
    float mx = -INFINITY;
    for (int k = 0; k < a.reg_max; k++) mx = fmaxf(mx, __half2float(p[s * a.reg_max + k]));
    float z = 0.f, e = 0.f;
    for (int k = 0; k < a.reg_max; k++) {
      const float t = expf(__half2float(p[s * a.reg_max + k]) - mx);
      z += t;
      e += t * (float)k;
    }
    d[s] = e / z;
  }
  const float ax = (float)cx + 0.5f, ay = (float)cy + 0.5f, st = (float)a.stride[l];
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
  const float c = __half2float(a.cls[l][pix]);
  a.conf[gid] = 1.f / (1.f + expf(-c));
}

// --------------------------------------------------------------------------------------------- NMS
struct NmsArgs {
  const float* xyxy;   // [B][A][4]
  const float* conf;   // [B][A]
  int A, n2;           // anchors, sort size (power of two ≥ A)
  float conf_th, iou_th;
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
};

// ref_detect's IoU test in its exact fp32 operation order (b = candidate, c = kept box).
__device__ __forceinline__ bool suppresses(const float4 b, const float4 c, float thr) {
  const float iw = fmaxf(0.f, __fsub_rn(fminf(b.z, c.z), fmaxf(b.x, c.x)));
  const float ih = fmaxf(0.f, __fsub_rn(fminf(b.w, c.w), fmaxf(b.y, c.y)));
  const float inter = __fmul_rn(iw, ih);
  const float ab = __fmul_rn(__fsub_rn(b.z, b.x), __fsub_rn(b.w, b.y));
  const float ac = __fmul_rn(__fsub_rn(c.z, c.x), __fsub_rn(c.w, c.y));
  const float u = __fsub_rn(__fadd_rn(ab, ac), inter);
  return u > 0.f && __fdiv_rn(inter, u) > thr;
}

// (conf, anchor) ordering of the sort: higher conf first, then lower anchor (numpy's stable argsort of −conf)
__device__ __forceinline__ bool before(float ca, int ia, float cb, int ib) { return ca > cb || (ca == cb && ia < ib); }

constexpr int kNmsThreads = 1024;

__global__ void __launch_bounds__(kNmsThreads) k_nms(const NmsArgs a) {
  extern __shared__ uint8_t nsm[];
  float* key = reinterpret_cast<float*>(nsm);                      // [n2]
  unsigned short* idx = reinterpret_cast<unsigned short*>(key + a.n2);  // [n2] (anchors < 65536)
  float4* kept = reinterpret_cast<float4*>(idx + a.n2);            // [max_det] (n2·6 B is 16-B aligned)
  __shared__ unsigned supp;                                    // candidates of the block suppressed by kept boxes
  __shared__ int nkept, cand_idx[32];
  __shared__ float4 cand_box[32];
  __shared__ int n_valid;
  const int b = blockIdx.x, tid = threadIdx.x;
  const float* conf = a.conf + (long long)b * a.A;
  const float4* box = reinterpret_cast<const float4*>(a.xyxy) + (long long)b * a.A;
  if (tid == 0) {
    nkept = 0;
    n_valid = 0;
  }
  __syncthreads();
  int local_valid = 0;
  for (int i = tid; i < a.n2; i += blockDim.x) {
    float c = -1.f;
    if (i < a.A) {
      c = conf[i];
      if (!a.forced && !(c > a.conf_th)) c = -1.f;
      if (c >= 0.f) local_valid++;
    }
    key[i] = c;
    idx[i] = i;
  }
  atomicAdd(&n_valid, local_valid);
  __syncthreads();
  // bitonic sort, descending by (conf, then ascending anchor)
  for (int k = 2; k <= a.n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < a.n2; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const float ki = key[i], kj = key[ixj];
          const int ii = idx[i], ij = idx[ixj];
          const bool up = (i & k) == 0;  // this sub-sequence sorts in "before" order
          const bool swap = up ? before(kj, ij, ki, ii) : before(ki, ii, kj, ij);
          if (swap) {
            key[i] = kj;
            key[ixj] = ki;
            idx[i] = ij;
            idx[ixj] = ii;
          }
        }
      }
      __syncthreads();
    }
  }
  const int nc = n_valid;
  const int lane = tid & 31, warp = tid >> 5;
  if (a.forced) {
    const int n = nc < a.max_det ? nc : a.max_det;
    for (int i = tid; i < n; i += blockDim.x) kept[i] = box[idx[i]];
    if (tid == 0) nkept = n;
    __syncthreads();
  } else {
    // greedy NMS, 32 candidates per round
    for (int c0 = 0; c0 < nc; c0 += 32) {
      if (nkept >= a.max_det) break;  // uniform: read after a barrier
      if (tid < 32) {
        const int ci = c0 + tid;
        cand_idx[tid] = ci < nc ? idx[ci] : -1;
        cand_box[tid] = ci < nc ? box[idx[ci]] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      if (tid == 0) supp = 0u;
      __syncthreads();
      // (1) against the boxes kept so far: candidate = lane, kept boxes strided over the warps
      {
        const int nk = nkept;
        const float4 cb = cand_box[lane];
        bool s = false;
        if (cand_idx[lane] >= 0)
          for (int k = warp; k < nk && !s; k += blockDim.x / 32) s = suppresses(cb, kept[k], a.iou_th);
        const unsigned m = __ballot_sync(0xffffffffu, s);
        if (lane == 0 && m) atomicOr(&supp, m);
      }
      __syncthreads();
      // (2) in candidate order within the round (warp 0)
      if (warp == 0) {
        unsigned dead = supp;
        const float4 mine = cand_box[lane];
        const bool valid = cand_idx[lane] >= 0;
        int nk = nkept;
        for (int i = 0; i < 32; i++) {
          const bool alive_i = ((dead >> i) & 1u) == 0 && cand_idx[i] >= 0;  // uniform across the warp
          if (!alive_i) continue;
          if (nk >= a.max_det) break;
          if (lane == 0) kept[nk] = cand_box[i];
          // record the kept anchor in the output order
          if (lane == 0) {
            a.keep[(long long)b * a.max_det + nk] = cand_idx[i];
            a.det_score[(long long)b * a.max_det + nk] = conf[cand_idx[i]];
          }
          nk++;
          const bool s = valid && lane > i && suppresses(mine, cand_box[i], a.iou_th);
          dead |= __ballot_sync(0xffffffffu, s);
        }
        if (lane == 0) nkept = nk;
        __syncwarp();
      }
      __syncthreads();
    }
  }
  const int n = nkept;
  if (a.forced) {
    for (int i = tid; i < n; i += blockDim.x) {
      a.keep[(long long)b * a.max_det + i] = idx[i];
      a.det_score[(long long)b * a.max_det + i] = conf[idx[i]];
    }
  }
  for (int i = tid; i < a.max_det; i += blockDim.x) {
    const float4 o = i < n ? kept[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    reinterpret_cast<float4*>(a.det_box)[(long long)b * a.max_det + i] = o;
    if (i >= n) {
      a.keep[(long long)b * a.max_det + i] = -1;
      a.det_score[(long long)b * a.max_det + i] = 0.f;
    }
  }
  __syncthreads();
  // gather the kept anchors' mask coefficients (32 fp16 = 4 × 16 B) into the GEMM's A rows
  for (int t = tid; t < a.max_det_pad * 4; t += blockDim.x) {
    const int i = t >> 2, ch = t & 3;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (i < n) {
      const int an = a.keep[(long long)b * a.max_det + i];
      int l = 0, rem = an;
      while (l < 2 && rem >= a.h[l] * a.w[l]) {
        rem -= a.h[l] * a.w[l];
        l++;
      }
      const long long pix = (long long)b * a.h[l] * a.w[l] + rem;
      v = *reinterpret_cast<const uint4*>(a.coef[l] + pix * 32 + ch * 8);
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
  int ptiles;            // pixel tiles of 256 per image
  int* err;
};

// One CTA = 128 detections × 256 proto pixels of one image: two K=16 UMMAs (M=128, N=256) into TMEM,
// then each of the 4 warps writes its 32 detection rows: byte = (logit > 0) ∧ inside the cropped box.
__global__ void __launch_bounds__(128) k_mask(const MaskArgs a) {
  __shared__ __align__(1024) uint8_t sA[128 * 64];
  __shared__ __align__(1024) uint8_t sB[256 * 64];
  __shared__ uint64_t bar;
  __shared__ uint32_t tslot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pt = blockIdx.x % a.ptiles, rest = blockIdx.x / a.ptiles;
  const int dtile = rest % (a.max_det_pad / 128), b = rest / (a.max_det_pad / 128);
  const int ndet = a.n_det[b];
  const int d0 = dtile * 128, p0 = pt * 256, npix = a.Hp * a.Wp;
  if (d0 >= a.max_det) return;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tslot, 256);
    tmem_relinquish();
  }
  // operands: 64-byte K-major rows, 64-byte swizzle (coef rows; proto pixels, zero beyond the image)
  const __half* ca = a.coef_g + ((long long)b * a.max_det_pad + d0) * 32;
  for (int t = tid; t < 128 * 4; t += 128) {
    const int r = t >> 2, ch = t & 3;
    const uint4 v = *reinterpret_cast<const uint4*>(ca + r * 32 + ch * 8);
    *reinterpret_cast<uint4*>(sA + r * 64 + ((ch ^ ((r >> 1) & 3)) << 4)) = v;
  }
  const __half* pb = a.proto + ((long long)b * npix + p0) * 32;
  for (int t = tid; t < 256 * 4; t += 128) {
    const int r = t >> 2, ch = t & 3;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (p0 + r < npix) v = *reinterpret_cast<const uint4*>(pb + r * 32 + ch * 8);
    *reinterpret_cast<uint4*>(sB + r * 64 + ((ch ^ ((r >> 1) & 3)) << 4)) = v;
  }
  fence_proxy_async_smem();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  if (tid == 0) {
    constexpr uint32_t idesc = idesc_f16_f32(128, 256);
    const uint32_t sa = smem_u32(sA), sb = smem_u32(sB);
    umma_f16(tmem, smem_desc_kmajor(sa, 64), smem_desc_kmajor(sb, 64), idesc, 0);
    umma_f16(tmem, smem_desc_kmajor(sa + 32, 64), smem_desc_kmajor(sb + 32, 64), idesc, 1);
    umma_commit(&bar);
  }
  const bool ok = mbar_wait(&bar, 0, a.err);
  tc_fence_after();
  if (ok) {
    const int det = d0 + warp * 32 + lane;
    const bool live = det < ndet;
    float4 bx = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) {
      const float4 o = reinterpret_cast<const float4*>(a.det_box)[(long long)b * a.max_det + det];
      bx = make_float4(__fmul_rn(o.x, a.g), __fmul_rn(o.y, a.g), __fmul_rn(o.z, a.g), __fmul_rn(o.w, a.g));
    }
    const int nwords = (npix + 31) / 32;
    uint8_t* out = a.masks + ((long long)b * a.max_det + det) * npix + p0;
    uint32_t* outw = reinterpret_cast<uint32_t*>(a.masks) + ((long long)b * a.max_det + det) * nwords + p0 / 32;
    uint32_t bits = 0u;
#pragma unroll 1
    for (int c = 0; c < 256; c += 16) {
      __syncwarp();
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + c, v);
      if (det >= a.max_det || p0 + c >= npix) continue;
      uint32_t w4[4] = {0u, 0u, 0u, 0u};
      uint32_t m16 = 0u;
#pragma unroll
      for (int k = 0; k < 16; k++) {
        const int pix = p0 + c + k;
        const float yy = (float)(pix / a.Wp), xx = (float)(pix - (pix / a.Wp) * a.Wp);
        const bool m = live && pix < npix && v[k] > 0.f && xx >= bx.x && xx < bx.z && yy >= bx.y && yy < bx.w;
        w4[k >> 2] |= (m ? 1u : 0u) << ((k & 3) * 8);
        m16 |= (m ? 1u : 0u) << k;
      }
      if (a.packed) {
        bits |= m16 << (c & 16);
        if ((c & 16) || p0 + c + 16 >= npix) {
          outw[c / 32] = bits;
          bits = 0u;
        }
      } else if (p0 + c + 16 <= npix && (npix & 15) == 0) {
        *reinterpret_cast<uint4*>(out + c) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      } else {
        for (int k = 0; k < 16 && p0 + c + k < npix; k++) out[c + k] = (w4[k >> 2] >> ((k & 3) * 8)) & 0xff;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace osam

using namespace osam;

namespace {
int pp_fail(int code, const char* msg) {
  set_last_error("%s", msg);
  return code;
}
int next_pow2(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
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

static size_t nms_smem_bytes(int anchors, int max_det) {
  const int n2 = next_pow2(anchors) < 16 ? 16 : next_pow2(anchors);
  return (size_t)(n2 < 16 ? 16 : n2) * 6 + (size_t)max_det * 16;
}

extern "C" {

int osam_nms(const float* xyxy, const float* conf, int batch, int anchors, float conf_th, float iou_th, int max_det,
             int forced, const void* const* coef, const int* level_hw, int* n_det, int* keep, float* det_box,
             float* det_score, void* coef_g, osam_stream_t stream) {
  if (!xyxy || !conf || batch < 1 || anchors < 1 || anchors > 65536 || max_det < 1 || max_det > 1024 || !n_det ||
      !keep || !det_box || !det_score)
    return pp_fail(OSAM_ERR_INVALID, "osam_nms: invalid arguments");
  NmsArgs a{};
  a.xyxy = xyxy;
  a.conf = conf;
  a.A = anchors;
  a.n2 = next_pow2(anchors) < 16 ? 16 : next_pow2(anchors);
  a.conf_th = conf_th;
  a.iou_th = iou_th;
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
  const size_t smem = nms_smem_bytes(anchors, max_det);
  if (smem > 220 * 1024) return pp_fail(OSAM_ERR_UNSUPPORTED, "osam_nms: too many anchors for one CTA");
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_nms, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
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
  a.ptiles = (proto_h * proto_w + 255) / 256;
  a.err = device_error_word();
  if (!a.err) return pp_fail(OSAM_ERR_CUDA, "osam_mask_assemble: device error word");
  const long long grid = (long long)batch * (a.max_det_pad / 128) * a.ptiles;
  k_mask<<<(unsigned)grid, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OSAM_OK : pp_fail(OSAM_ERR_CUDA, cudaGetErrorString(e));
}

}  // extern "C"
