// Test infrastructure: drives the reference's own training pass (Model::forward(true) + Model::backward,
// src/model.cpp:383-474, built from its sources by oracle/Makefile into oracle/_ref/ref_train) so that this
// build's training pass can be compared with it on identical weights, images and head gradients, and timed
// beside it on the same B200.
//
//   ref_train <weights.fsow> <in.fsow | -> <out.fsow | -> [iters] [batch imgsz]
//
// in.fsow: "images" (N, S, S, 3) float32 in [0,1] and the head gradients "grad.out.box<l>", "grad.out.cls<l>",
// "grad.out.coef<l>", "grad.out.proto" (NHWC float32); "-" makes seeded pseudo-random ones of batch×imgsz².
// out.fsow: every parameter gradient as "grad.<name>" (Params::save with grads, PyTorch layouts), the running
// statistics after the pass as "<name>" (running_mean / running_var) and the heads as "out.*".
// iters > 0: forward(true) + backward(false) timed with CUDA events (eager, after 3 warm-up passes) — one JSON
// line.  BN momentum 0.03, eps 1e-3 (ModelCfg defaults).
#include <chrono>
#include <cstdio>
#include <random>
#include <string>
#include <vector>

#include "fsow.h"
#include "model.h"

namespace {
std::vector<float> to_host(const act_t* p, size_t n) {
  std::vector<act_t> t(n);
  CUDA_CHECK(cudaMemcpy(t.data(), p, n * sizeof(act_t), cudaMemcpyDeviceToHost));
  std::vector<float> o(n);
  for (size_t i = 0; i < n; i++) o[i] = to_f(t[i]);
  return o;
}
void upload(act_t* dst, const float* src, size_t n) {
  std::vector<act_t> h(n);
  for (size_t i = 0; i < n; i++) h[i] = from_f<act_t>(src[i]);
  CUDA_CHECK(cudaMemcpy(dst, h.data(), n * sizeof(act_t), cudaMemcpyHostToDevice));
}
}  // namespace

int main(int argc, char** argv) {
  FSO_ASSERT(argc >= 4, "usage: ref_train <weights.fsow> <in.fsow|-> <out.fsow|-> [iters] [batch imgsz]");
  const std::string wpath = argv[1], ipath = argv[2], opath = argv[3];
  const int iters = argc > 4 ? atoi(argv[4]) : 0;
  int B = argc > 5 ? atoi(argv[5]) : 2, S = argc > 6 ? atoi(argv[6]) : 256;
  TensorMap in;
  if (ipath != "-") {
    in = fsow_load(ipath);
    const HostTensor& t = in.at("images");
    B = int(t.shape[0]);
    S = int(t.shape[1]);
  }
  cudaStream_t st;
  CUDA_CHECK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  cudnnHandle_t h;
  CUDNN_CHECK(cudnnCreate(&h));
  CUDNN_CHECK(cudnnSetStream(h, st));
  TensorMap W = fsow_load(wpath);
  Model m;
  ModelCfg cfg;
  cfg.batch = B;
  cfg.imgsz = S;
  cfg.reg_max = reg_max_of(W);
  m.build(cfg, h, st);
  m.params.load(W);
  m.sync_weights();

  std::mt19937 rng(777);
  std::uniform_real_distribution<float> U(0.f, 1.f);
  std::normal_distribution<float> Nd(0.f, 0.05f);
  {
    const size_t n = size_t(B) * S * S * kInC;
    std::vector<float> img(n);
    if (ipath != "-") {
      const float* s = in.at("images").f32();
      img.assign(s, s + n);
    } else {
      for (auto& v : img) v = U(rng);
    }
    upload(m.input()->p, img.data(), n);
  }
  auto set_grad = [&](Act* a, const std::string& name) {
    const size_t n = size_t(B) * a->H * a->W * a->C;
    std::vector<float> g(n);
    if (ipath != "-") {
      const float* s = in.at("grad." + name).f32();
      g.assign(s, s + n);
    } else {
      for (auto& v : g) v = Nd(rng);
    }
    upload(a->g, g.data(), n);
  };
  const char* kinds[3] = {"box", "cls", "coef"};
  m.forward(true);
  for (int k = 0; k < 3; k++)
    for (int l = 0; l < 3; l++) set_grad(m.head(k, l), "out." + std::string(kinds[k]) + std::to_string(l));
  set_grad(m.proto(), "out.proto");
  m.backward(false);
  CUDA_CHECK(cudaStreamSynchronize(st));

  if (opath != "-") {
    TensorMap out = m.params.save("grad.", true);
    TensorMap vals = m.params.save("", false);
    for (auto& kv : vals)
      if (kv.first.find("running_") != std::string::npos) out[kv.first] = kv.second;
    for (int k = 0; k < 3; k++)
      for (int l = 0; l < 3; l++) {
        Act* a = m.head(k, l);
        out["out." + std::string(kinds[k]) + std::to_string(l)] =
            HostTensor::make_f32({B, a->H, a->W, a->C}, to_host(a->p, size_t(B) * a->H * a->W * a->C).data());
      }
    fsow_save(opath, out);
  }
  if (iters > 0) {
    cudaEvent_t e0, e1;
    CUDA_CHECK(cudaEventCreate(&e0));
    CUDA_CHECK(cudaEventCreate(&e1));
    for (int i = 0; i < 3; i++) {
      m.forward(true);
      m.backward(false);
    }
    CUDA_CHECK(cudaEventRecord(e0, st));
    for (int i = 0; i < iters; i++) {
      m.forward(true);
      m.backward(false);
    }
    CUDA_CHECK(cudaEventRecord(e1, st));
    CUDA_CHECK(cudaEventSynchronize(e1));
    float ms = 0.f;
    CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
    printf("{\"impl\": \"reference-cudnn\", \"pass\": \"forward(train) + backward\", \"batch\": %d, \"imgsz\": %d, "
           "\"iters\": %d, \"ms\": %.4f, \"img_per_s\": %.2f}\n",
           B, S, iters, ms / iters, B / (ms / iters / 1e3));
  }
  return 0;
}
