// Test infrastructure: runs the reference's own training-mode BN / bias / stem-wgrad / loss kernels (built from
// its sources src/bn.cu, src/misc.cu and src/loss.cu by oracle/Makefile into oracle/_ref/ref_bn) on inputs read
// from an FSOW file, and writes their outputs to another, so the GPU tests can compare this build's kernels and
// the CPU restatements (oracle/bn_ref.py, oracle/mask_loss_ref.py) with the reference itself on identical inputs.
//
//   ref_bn <in.fsow> <out.fsow>
//
// Cases are named "c<i>.*".  c<i>.meta (int32) = {op, ...}:
//   op 0  CONVBN training node: meta = {0, N, H, W, C, act, has_res, ndest, accum, res_accum,
//         (ctot, choff, c0, c1, up) × ndest}; c<i>.f = {momentum, eps}; inputs z, gamma, beta, run_mean,
//         run_var, [res], dest<k> (initial destination contents), grad<k> (destination gradients),
//         gw_gamma0, gw_beta0, [res_grad0].  Runs bn_forward_stats → bn_forward_apply → bn_backward
//         (src/model.cpp:388-400, :440-444) and writes mean, istd, scale, shift, run_mean, run_var,
//         dest<k>, dz, gw_gamma, gw_beta, [res_grad].
//   op 1  chan_sum: meta = {1, M, C, accum}; x (M, C), out0 (C) → out.
//   op 2  add_bias: meta = {2, M, C}; y (M, C), bias (C) → y.
//   op 3  wgrad_rgb_s2: meta = {3, N, H, W, K}; x (N, H, W, 3), dz (N, P, Q, K) → dw (K, 3, 3, 3) and
//         ran (1 if the reference took its own kernel, 0 if it declined the shape).
//   op 4  sppf_pool_bwd: meta = {4, N, H, W, c}; cat, dcat (N, H, W, 4c) → dcat.
//   op 6  augment (src/augment.cuh:19): meta = {6, B, S, G, Hp, Wp, with_ignore, iters}; blob (u8: the
//         batch's header, B sample records, 4B source records and its instance records, laid out as
//         BatchBuf::alloc_dev lays them out), img (u8 source pixels), mask (int32 instance bitmaps) →
//         img (fp16 values as f32 [B, S, S, 3]), n_gt, box [B, G, 4], gt_inst [B, G], mask (int32
//         [B, G, Hp·Wp/32]), [ignore (int32 [B, Hp·Wp/32])], (iters > 0: ms, the mean time of augment).
//   op 5  SegLoss::run (src/loss.cu:590-621): meta = {5, B, imgsz, G}; box<l>, cls<l>, coef<l> heads, proto,
//         n_gt (int32 [B]), gt_box (B, G, 4), gt_mask (int32 [B, G, Hp·Wp/32]), scale (1) → dproto, dcoef<l>,
//         dbox<l>, dcls<l>, tsc (target scores),  (meta[4] = iters > 0: also ms, the mean time of run)
//         items (16), agt (int32 [B, A]).
// Timing ops (device time with CUDA events per call, L2 flushed by reading 256 MiB before each call; inputs
// are seeded pseudo-random fp16 made on the host):
//   op 10 BN passes of one conv+BN+SiLU node: meta = {10, N, H, W, C, iters} → ms = {stats, apply, backward,
//         stats and apply back to back} (one plain destination, no residual).
//   op 13 wgrad_rgb_s2: meta = {13, N, H, W, iters} → ms = {wgrad} (K = 32).
// Activations are converted to the reference's act_t (fp16) on upload; every value the tests send is
// fp16-representable.
#include <cstdio>
#include <string>
#include <vector>

#include <cstddef>

#include "augment.cuh"
#include "bn.cuh"
#include "fsow.h"
#include "osam.h"
#include "loss.cuh"
#include "misc.cuh"

namespace {

const HostTensor& need(const TensorMap& m, const std::string& k) {
  auto it = m.find(k);
  FSO_ASSERT(it != m.end(), "missing %s", k.c_str());
  return it->second;
}
bool has(const TensorMap& m, const std::string& k) { return m.count(k) > 0; }

act_t* up_act(const HostTensor& t) {
  const int64_t n = t.numel();
  std::vector<act_t> h(n);
  for (int64_t i = 0; i < n; i++) h[i] = from_f<act_t>(t.f32()[i]);
  act_t* d = dalloc<act_t>(n);
  CUDA_CHECK(cudaMemcpy(d, h.data(), n * sizeof(act_t), cudaMemcpyHostToDevice));
  return d;
}
float* up_f32(const HostTensor& t) {
  float* d = dalloc<float>(t.numel());
  CUDA_CHECK(cudaMemcpy(d, t.f32(), t.numel() * sizeof(float), cudaMemcpyHostToDevice));
  return d;
}
HostTensor down_act(const act_t* d, const std::vector<int64_t>& shape) {
  HostTensor t = HostTensor::make_f32(shape, nullptr);
  const int64_t n = t.numel();
  std::vector<act_t> h(n);
  CUDA_CHECK(cudaMemcpy(h.data(), d, n * sizeof(act_t), cudaMemcpyDeviceToHost));
  float* o = reinterpret_cast<float*>(t.data.data());
  for (int64_t i = 0; i < n; i++) o[i] = to_f(h[i]);
  return t;
}
int32_t* up_i32(const HostTensor& t) {
  int32_t* d = dalloc<int32_t>(t.numel());
  CUDA_CHECK(cudaMemcpy(d, t.i32(), t.numel() * sizeof(int32_t), cudaMemcpyHostToDevice));
  return d;
}
HostTensor down_i32(const int32_t* d, const std::vector<int64_t>& shape) {
  HostTensor t;
  t.shape = shape;
  t.dtype = 1;
  t.data.resize(size_t(t.numel()) * 4);
  CUDA_CHECK(cudaMemcpy(t.data.data(), d, t.data.size(), cudaMemcpyDeviceToHost));
  return t;
}
act_t* rand_act(int64_t n, uint32_t seed, float lo, float hi) {
  std::vector<act_t> h(n);
  uint32_t x = seed * 2654435761u + 1u;
  for (int64_t i = 0; i < n; i++) {
    x = x * 1664525u + 1013904223u;
    h[i] = from_f<act_t>(lo + (hi - lo) * float(x >> 8) * (1.f / 16777216.f));
  }
  act_t* d = dalloc<act_t>(n);
  CUDA_CHECK(cudaMemcpy(d, h.data(), n * sizeof(act_t), cudaMemcpyHostToDevice));
  return d;
}
float* const_f32(int64_t n, float v) {
  std::vector<float> h(n, v);
  float* d = dalloc<float>(n);
  CUDA_CHECK(cudaMemcpy(d, h.data(), n * sizeof(float), cudaMemcpyHostToDevice));
  return d;
}
// Reads a buffer larger than L2 so that the timed call finds none of its inputs there (reads leave clean
// lines: nothing is written back during the timed call).
__global__ void k_flush_read(const uint4* p, size_t n, unsigned* sink) {
  unsigned x = 0;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    const uint4 v = p[i];
    x ^= v.x ^ v.y ^ v.z ^ v.w;
  }
  if (x == 0x9e3779b9u) *sink = x;
}
// Mean device time (ms) of fn over iters calls, each after an L2 flush.
template <class F>
float time_flushed(F fn, int iters, void* flush, size_t flush_bytes, cudaStream_t st) {
  cudaEvent_t e0, e1;
  CUDA_CHECK(cudaEventCreate(&e0));
  CUDA_CHECK(cudaEventCreate(&e1));
  fn();
  fn();
  float tot = 0.f;
  for (int i = 0; i < iters; i++) {
    k_flush_read<<<148 * 8, 256, 0, st>>>(static_cast<const uint4*>(flush), flush_bytes / 16,
                                         reinterpret_cast<unsigned*>(static_cast<char*>(flush)));
    CUDA_CHECK(cudaEventRecord(e0, st));
    fn();
    CUDA_CHECK(cudaEventRecord(e1, st));
    CUDA_CHECK(cudaEventSynchronize(e1));
    float ms = 0.f;
    CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
    tot += ms;
  }
  CUDA_CHECK(cudaEventDestroy(e0));
  CUDA_CHECK(cudaEventDestroy(e1));
  return tot / iters;
}
HostTensor down_f32(const float* d, int64_t n) {
  HostTensor t = HostTensor::make_f32({n}, nullptr);
  CUDA_CHECK(cudaMemcpy(t.data.data(), d, n * sizeof(float), cudaMemcpyDeviceToHost));
  return t;
}

// The C ABI's batch records must be the reference's, byte for byte (its loader fills them).
#define SAME_FIELD(A, B, f) static_assert(offsetof(A, f) == offsetof(B, f), #A "." #f)
static_assert(sizeof(osam_aug_src) == sizeof(SrcInfo), "SrcInfo size");
SAME_FIELD(osam_aug_src, SrcInfo, img_off); SAME_FIELD(osam_aug_src, SrcInfo, iw); SAME_FIELD(osam_aug_src, SrcInfo, mh);
static_assert(sizeof(osam_aug_inst) == sizeof(InstInfo), "InstInfo size");
SAME_FIELD(osam_aug_inst, InstInfo, src); SAME_FIELD(osam_aug_inst, InstInfo, box);
SAME_FIELD(osam_aug_inst, InstInfo, mx0); SAME_FIELD(osam_aug_inst, InstInfo, wpr);
SAME_FIELD(osam_aug_inst, InstInfo, mask_off); SAME_FIELD(osam_aug_inst, InstInfo, ignore);
static_assert(sizeof(osam_aug_sample) == sizeof(SampleInfo), "SampleInfo size");
SAME_FIELD(osam_aug_sample, SampleInfo, ta); SAME_FIELD(osam_aug_sample, SampleInfo, tb);
SAME_FIELD(osam_aug_sample, SampleInfo, s); SAME_FIELD(osam_aug_sample, SampleInfo, hsv);
SAME_FIELD(osam_aug_sample, SampleInfo, flip); SAME_FIELD(osam_aug_sample, SampleInfo, ninst);
static_assert(sizeof(osam_aug_header) == sizeof(BatchHeader), "BatchHeader size");
SAME_FIELD(osam_aug_header, BatchHeader, ninst); SAME_FIELD(osam_aug_header, BatchHeader, mask_words);

}  // namespace

int main(int argc, char** argv) {
  FSO_ASSERT(argc == 3, "usage: ref_bn <in.fsow> <out.fsow>");
  const TensorMap in = fsow_load(argv[1]);
  TensorMap out;
  bn_init();
  cudaStream_t st;
  CUDA_CHECK(cudaStreamCreate(&st));
  for (int ci = 0;; ci++) {
    const std::string p = "c" + std::to_string(ci) + ".";
    if (!has(in, p + "meta")) break;
    const int32_t* m = need(in, p + "meta").i32();
    const int64_t m_len = need(in, p + "meta").numel();
    const int op = m[0];
    if (op == 0) {
      const int N = m[1], H = m[2], W = m[3], C = m[4], act = m[5], has_res = m[6], nd = m[7];
      const bool accum = m[8] != 0, res_accum = m[9] != 0;
      const float* f = need(in, p + "f").f32();
      BnShape s{N, H, W, C};
      const int64_t M = s.M();
      act_t* z = up_act(need(in, p + "z"));
      float* gamma = up_f32(need(in, p + "gamma"));
      float* beta = up_f32(need(in, p + "beta"));
      float* rm = up_f32(need(in, p + "run_mean"));
      float* rv = up_f32(need(in, p + "run_var"));
      act_t* res = has_res ? up_act(need(in, p + "res")) : nullptr;
      float *mean = dalloc<float>(C), *istd = dalloc<float>(C), *scale = dalloc<float>(C), *shift = dalloc<float>(C);
      DestList fl, gl;
      std::vector<std::vector<int64_t>> dshape;
      for (int k = 0; k < nd; k++) {
        const int* d = m + 10 + 5 * k;
        const HostTensor& d0 = need(in, p + "dest" + std::to_string(k));
        const HostTensor& g0 = need(in, p + "grad" + std::to_string(k));
        Dest& a = fl.d[fl.n++];
        a.p = up_act(d0);
        a.ctot = d[0]; a.choff = d[1]; a.c0 = d[2]; a.c1 = d[3]; a.up = d[4];
        Dest& b = gl.d[gl.n++];
        b = a;
        b.g = up_act(g0);
        dshape.push_back(d0.shape);
      }
      bn_forward_stats(z, s, gamma, beta, rm, rv, f[0], f[1], mean, istd, scale, shift, st);
      bn_forward_apply(z, s, scale, shift, res, fl, act != 0, st);
      float* sums = dalloc<float>(2 * C);
      act_t* dz = dalloc<act_t>(M * C);
      float* gwg = up_f32(need(in, p + "gw_gamma0"));
      float* gwb = up_f32(need(in, p + "gw_beta0"));
      act_t* rg = nullptr;
      if (has_res) rg = has(in, p + "res_grad0") ? up_act(need(in, p + "res_grad0")) : dalloc<act_t>(M * C);
      bn_backward(z, s, gamma, mean, istd, scale, shift, gl, act != 0, sums, dz, gwg, gwb, accum, rg, res_accum, st);
      CUDA_CHECK(cudaStreamSynchronize(st));
      out[p + "mean"] = down_f32(mean, C);
      out[p + "istd"] = down_f32(istd, C);
      out[p + "scale"] = down_f32(scale, C);
      out[p + "shift"] = down_f32(shift, C);
      out[p + "run_mean"] = down_f32(rm, C);
      out[p + "run_var"] = down_f32(rv, C);
      for (int k = 0; k < nd; k++) out[p + "dest" + std::to_string(k)] = down_act(fl.d[k].p, dshape[k]);
      out[p + "dz"] = down_act(dz, {N, H, W, C});
      out[p + "gw_gamma"] = down_f32(gwg, C);
      out[p + "gw_beta"] = down_f32(gwb, C);
      if (rg) out[p + "res_grad"] = down_act(rg, {N, H, W, C});
    } else if (op == 1) {
      const int64_t M = m[1];
      const int C = m[2];
      act_t* x = up_act(need(in, p + "x"));
      float* o = up_f32(need(in, p + "out0"));
      float* part = dalloc<float>(int64_t(chan_sum_blocks(M, C)) * C);
      chan_sum(x, M, C, part, o, m[3] != 0, st);
      CUDA_CHECK(cudaStreamSynchronize(st));
      out[p + "out"] = down_f32(o, C);
    } else if (op == 2) {
      const int64_t M = m[1];
      const int C = m[2];
      act_t* y = up_act(need(in, p + "y"));
      float* b = up_f32(need(in, p + "bias"));
      add_bias(y, M, C, b, st);
      CUDA_CHECK(cudaStreamSynchronize(st));
      out[p + "y"] = down_act(y, {M, C});
    } else if (op == 3) {
      const int N = m[1], H = m[2], W = m[3], K = m[4];
      act_t* x = up_act(need(in, p + "x"));
      act_t* dz = up_act(need(in, p + "dz"));
      float* tmp = dalloc<float>(int64_t(K) * 27);
      act_t* dw = dalloc<act_t>(int64_t(K) * 27);
      CUDA_CHECK(cudaMemset(dw, 0, size_t(K) * 27 * sizeof(act_t)));
      const bool ran = wgrad_rgb_s2(x, dz, N, H, W, K, tmp, dw, st);
      CUDA_CHECK(cudaStreamSynchronize(st));
      out[p + "dw"] = down_act(dw, {K, 3, 3, 3});
      const float r = ran ? 1.f : 0.f;
      out[p + "ran"] = HostTensor::make_f32({1}, &r);
    } else if (op == 4) {
      const int N = m[1], H = m[2], W = m[3], c = m[4];
      const int64_t n = int64_t(N) * H * W * c;
      act_t* cat = up_act(need(in, p + "cat"));
      act_t* dcat = up_act(need(in, p + "dcat"));
      float* ta = dalloc<float>(n);
      float* tb = dalloc<float>(n);
      sppf_pool_bwd(cat, dcat, N, H, W, c, ta, tb, st);
      CUDA_CHECK(cudaStreamSynchronize(st));
      out[p + "dcat"] = down_act(dcat, {N, H, W, 4 * c});
    } else if (op == 5) {
      const int B = m[1], S = m[2], G = m[3];
      LossCfg c;
      c.B = B;
      c.imgsz = S;
      c.G = G;
      for (int l = 0; l < 3; l++) c.lvl_h[l] = c.lvl_w[l] = S / c.stride[l];
      c.Hp = c.Wp = S / 4;
      SegLoss L;
      L.init(c);
      HeadIO io{};
      std::vector<int64_t> cshape[3];
      for (int l = 0; l < 3; l++) {
        const std::string k = std::to_string(l);
        const int h = c.lvl_h[l], w = c.lvl_w[l];
        io.box[l] = up_act(need(in, p + "box" + k));
        io.cls[l] = up_act(need(in, p + "cls" + k));
        io.coef[l] = up_act(need(in, p + "coef" + k));
        io.dbox[l] = dalloc<act_t>(int64_t(B) * h * w * 64);
        io.dcls[l] = dalloc<act_t>(int64_t(B) * h * w);
        io.dcoef[l] = dalloc<act_t>(int64_t(B) * h * w * 32);
        cshape[l] = {B, h, w, 32};
      }
      io.proto = up_act(need(in, p + "proto"));
      act_t* dproto = dalloc<act_t>(int64_t(B) * c.Hp * c.Wp * 32);
      io.dproto = dproto;
      GtBatch gt;
      gt.n_gt = up_i32(need(in, p + "n_gt"));
      gt.box = reinterpret_cast<float4*>(up_f32(need(in, p + "gt_box")));
      gt.mask = reinterpret_cast<uint32_t*>(up_i32(need(in, p + "gt_mask")));
      float* scale = up_f32(need(in, p + "scale"));
      L.run(io, gt, scale, st);
      CUDA_CHECK(cudaStreamSynchronize(st));
      out[p + "dproto"] = down_act(dproto, {B, c.Hp, c.Wp, 32});
      for (int l = 0; l < 3; l++) out[p + "dcoef" + std::to_string(l)] = down_act(io.dcoef[l], cshape[l]);
      out[p + "items"] = down_f32(L.items(), 16);
      out[p + "agt"] = down_i32(L.assigned_gt(), {B, c.A()});
      if (m_len > 4 && m[4] > 0) {  // timing: mean device time of SegLoss::run, L2 flushed before each call
        static void* flush5 = nullptr;
        const size_t fb = size_t(256) << 20;
        if (!flush5) {
          flush5 = DevMem::alloc(fb);
          CUDA_CHECK(cudaMemset(flush5, 1, fb));
        }
        const float ms = time_flushed([&] { L.run(io, gt, scale, st); }, m[4], flush5, fb, st);
        out[p + "ms"] = HostTensor::make_f32({1}, &ms);
      }
      out[p + "tsc"] = down_f32(L.target_score(), int64_t(B) * c.A());  // [B·A]; entries of negatives are stale
      for (int l = 0; l < 3; l++) {
        const std::string k = std::to_string(l);
        out[p + "dbox" + k] = down_act(io.dbox[l], {B, c.lvl_h[l], c.lvl_w[l], 64});
        out[p + "dcls" + k] = down_act(io.dcls[l], {B, c.lvl_h[l], c.lvl_w[l], 1});
      }
    } else if (op == 6) {
      const int B = m[1], S = m[2], G = m[3], Hp = m[4], Wp = m[5], with_ignore = m[6], iters = m[7];
      const HostTensor& blob = need(in, p + "blob");
      const HostTensor& img = need(in, p + "img");
      const HostTensor& mask = need(in, p + "mask");
      BatchBuf db;
      db.hdr = static_cast<BatchHeader*>(DevMem::alloc(blob.numel()));
      CUDA_CHECK(cudaMemcpy(db.hdr, blob.u8(), blob.numel(), cudaMemcpyHostToDevice));
      db.smp = reinterpret_cast<SampleInfo*>(db.hdr + 1);
      db.src = reinterpret_cast<SrcInfo*>(db.smp + B);
      db.inst = reinterpret_cast<InstInfo*>(db.src + 4 * B);
      db.img = dalloc<uint8_t>(img.numel());
      CUDA_CHECK(cudaMemcpy(db.img, img.u8(), img.numel(), cudaMemcpyHostToDevice));
      db.mask = reinterpret_cast<uint32_t*>(up_i32(mask));
      const int words = Hp * Wp / 32;
      AugOut o;
      o.G = G; o.Hp = Hp; o.Wp = Wp;
      o.img = dalloc<act_t>(int64_t(B) * S * S * 3);
      o.gt.n_gt = dalloc<int>(B);
      o.gt.box = dalloc<float4>(int64_t(B) * G);
      o.gt.mask = dalloc<uint32_t>(int64_t(B) * G * words);
      o.gt.ignore = with_ignore ? dalloc<uint32_t>(int64_t(B) * words) : nullptr;
      o.gt_inst = dalloc<int>(int64_t(B) * G);
      augment(db, B, S, o, st);
      CUDA_CHECK(cudaStreamSynchronize(st));
      out[p + "img"] = down_act(o.img, {B, S, S, 3});
      out[p + "n_gt"] = down_i32(o.gt.n_gt, {B});
      out[p + "box"] = down_f32(reinterpret_cast<const float*>(o.gt.box), int64_t(B) * G * 4);
      out[p + "gt_inst"] = down_i32(o.gt_inst, {B, G});
      out[p + "mask"] = down_i32(reinterpret_cast<const int32_t*>(o.gt.mask), {B, G, words});
      if (with_ignore) out[p + "ignore"] = down_i32(reinterpret_cast<const int32_t*>(o.gt.ignore), {B, words});
      if (iters > 0) {
        static void* flush6 = nullptr;
        const size_t fb = size_t(256) << 20;
        if (!flush6) {
          flush6 = DevMem::alloc(fb);
          CUDA_CHECK(cudaMemset(flush6, 1, fb));
        }
        const float ms = time_flushed([&] { augment(db, B, S, o, st); }, iters, flush6, fb, st);
        out[p + "ms"] = HostTensor::make_f32({1}, &ms);
      }
    } else if (op == 10 || op == 13) {
      static void* flush = nullptr;
      const size_t flush_bytes = size_t(256) << 20;
      if (!flush) {
        flush = DevMem::alloc(flush_bytes);
        CUDA_CHECK(cudaMemset(flush, 1, flush_bytes));
      }
      std::vector<float> ms;
      if (op == 10) {
        const int N = m[1], H = m[2], W = m[3], C = m[4], iters = m[5];
        BnShape s{N, H, W, C};
        const int64_t M = s.M();
        act_t* z = rand_act(M * C, 1, -2.f, 3.f);
        float *gamma = const_f32(C, 1.f), *beta = const_f32(C, 0.f), *rm = const_f32(C, 0.f), *rv = const_f32(C, 1.f);
        float *mean = dalloc<float>(C), *istd = dalloc<float>(C), *scale = dalloc<float>(C), *shift = dalloc<float>(C);
        float *sums = dalloc<float>(2 * C), *gwg = dalloc<float>(C), *gwb = dalloc<float>(C);
        DestList dl;
        Dest& d = dl.d[dl.n++];
        d.p = dalloc<act_t>(M * C);
        d.g = rand_act(M * C, 2, -0.1f, 0.1f);
        d.ctot = C; d.choff = 0; d.c0 = 0; d.c1 = C; d.up = 1;
        act_t* dz = dalloc<act_t>(M * C);
        ms.push_back(time_flushed([&] { bn_forward_stats(z, s, gamma, beta, rm, rv, 0.f, 1e-3f, mean, istd, scale,
                                                          shift, st); }, iters, flush, flush_bytes, st));
        ms.push_back(time_flushed([&] { bn_forward_apply(z, s, scale, shift, nullptr, dl, true, st); }, iters, flush,
                                  flush_bytes, st));
        ms.push_back(time_flushed([&] { bn_backward(z, s, gamma, mean, istd, scale, shift, dl, true, sums, dz, gwg, gwb,
                                                     false, nullptr, false, st); }, iters, flush, flush_bytes, st));
        ms.push_back(time_flushed([&] {
          bn_forward_stats(z, s, gamma, beta, rm, rv, 0.f, 1e-3f, mean, istd, scale, shift, st);
          bn_forward_apply(z, s, scale, shift, nullptr, dl, true, st);
        }, iters, flush, flush_bytes, st));
      } else {
        const int N = m[1], H = m[2], W = m[3], iters = m[4];
        const int P = (H + 1) / 2, Q = (W + 1) / 2;
        act_t* x = rand_act(int64_t(N) * H * W * 3, 3, 0.f, 1.f);
        act_t* dzz = rand_act(int64_t(N) * P * Q * 32, 4, -1.f, 1.f);
        float* tmp = dalloc<float>(32 * 27);
        act_t* dw = dalloc<act_t>(32 * 27);
        bool ran = true;
        ms.push_back(time_flushed([&] { ran = wgrad_rgb_s2(x, dzz, N, H, W, 32, tmp, dw, st); }, iters, flush,
                                  flush_bytes, st));
        if (!ran) ms[0] = -1.f;
      }
      out[p + "ms"] = HostTensor::make_f32({int64_t(ms.size())}, ms.data());
    } else {
      FSO_ASSERT(false, "unknown op %d", op);
    }
  }
  fsow_save(argv[2], out);
  return 0;
}
