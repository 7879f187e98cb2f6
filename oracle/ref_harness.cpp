// Test infrastructure: drives the reference's own Model (built from its sources by oracle/Makefile into
// oracle/_ref/) so that its cuDNN path can be (a) compared with this build's kernels on identical weights
// and inputs, and (b) timed on the same B200 as the reference baseline.
//
//   ref_forward <weights.fsow> <images.fsow | -> <out.fsow | -> [iters] [batch imgsz]
//
// images.fsow holds "images" (N, S, S, 3) float32 in [0,1]; "-" makes a seeded U[0,1] batch of
// `batch`×imgsz² instead.  The weights use the reference's FSOW names (src/fsow.h).  The forward is the
// reference's Model::build + Params::load + sync_weights + forward(false) (src/model.cpp:168-414);
// out.fsow receives the raw heads and proto as NHWC float32 ("out.box0" … "out.proto").  With iters > 0
// the forward is timed with CUDA events, eagerly and as a captured CUDA graph (the reference captures its
// training step the same way, src/train.cpp:209-222), and one JSON line is printed.
#include <chrono>
#include <cstdio>
#include <random>
#include <string>
#include <vector>

#include "model.h"

namespace {
std::vector<float> to_host(const Act* a, int N) {
  const size_t n = size_t(N) * a->H * a->W * a->C;
  std::vector<act_t> t(n);
  CUDA_CHECK(cudaMemcpy(t.data(), a->p, n * sizeof(act_t), cudaMemcpyDeviceToHost));
  std::vector<float> o(n);
  for (size_t i = 0; i < n; i++) o[i] = to_f(t[i]);
  return o;
}
}  // namespace

int main(int argc, char** argv) {
  FSO_ASSERT(argc >= 4, "usage: ref_forward <weights.fsow> <images.fsow|-> <out.fsow|-> [iters] [batch imgsz]");
  const std::string wpath = argv[1], ipath = argv[2], opath = argv[3];
  const int iters = argc > 4 ? atoi(argv[4]) : 0;
  int B = argc > 5 ? atoi(argv[5]) : 1, S = argc > 6 ? atoi(argv[6]) : 640;
  TensorMap images;
  if (ipath != "-") {
    images = fsow_load(ipath);
    const HostTensor& t = images.at("images");
    FSO_ASSERT(t.shape.size() == 4 && t.shape[3] == 3, "images must be (N,S,S,3)");
    B = int(t.shape[0]);
    S = int(t.shape[1]);
  }
  cudaStream_t st;
  CUDA_CHECK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  cudnnHandle_t h;
  CUDNN_CHECK(cudnnCreate(&h));
  CUDNN_CHECK(cudnnSetStream(h, st));
  const auto t0 = std::chrono::steady_clock::now();
  TensorMap W = fsow_load(wpath);
  Model m;
  m.build(ModelCfg{B, S, reg_max_of(W)}, h, st);
  m.params.load(W);
  m.sync_weights();
  const double build_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();

  // input (NHWC, C = kInC = 3)
  {
    const size_t n = size_t(B) * S * S * kInC;
    std::vector<act_t> img(n);
    if (ipath != "-") {
      const float* src = images.at("images").f32();
      for (size_t i = 0; i < n; i++) img[i] = from_f<act_t>(src[i]);
    } else {
      std::mt19937 rng(12345);
      std::uniform_real_distribution<float> U(0.f, 1.f);
      for (size_t i = 0; i < n; i++) img[i] = from_f<act_t>(U(rng));
    }
    CUDA_CHECK(cudaMemcpy(m.input()->p, img.data(), n * sizeof(act_t), cudaMemcpyHostToDevice));
  }
  m.forward(false);
  CUDA_CHECK(cudaStreamSynchronize(st));

  if (opath != "-") {
    TensorMap out;
    const char* kinds[3] = {"box", "cls", "coef"};
    for (int k = 0; k < 3; k++)
      for (int l = 0; l < 3; l++) {
        const Act* a = m.head(k, l);
        out["out." + std::string(kinds[k]) + std::to_string(l)] =
            HostTensor::make_f32({B, a->H, a->W, a->C}, to_host(a, B).data());
      }
    const Act* p = m.proto();
    out["out.proto"] = HostTensor::make_f32({B, p->H, p->W, p->C}, to_host(p, B).data());
    fsow_save(opath, out);
  }

  if (getenv("OSAM_REF_PRINT_CONVS")) m.print_convs();  // the reference's per-conv tuned timings (to stdout)
  if (iters > 0) {
    cudaEvent_t e0, e1;
    CUDA_CHECK(cudaEventCreate(&e0));
    CUDA_CHECK(cudaEventCreate(&e1));
    for (int i = 0; i < 3; i++) m.forward(false);
    CUDA_CHECK(cudaEventRecord(e0, st));
    for (int i = 0; i < iters; i++) m.forward(false);
    CUDA_CHECK(cudaEventRecord(e1, st));
    CUDA_CHECK(cudaEventSynchronize(e1));
    float eager_ms = 0.f;
    CUDA_CHECK(cudaEventElapsedTime(&eager_ms, e0, e1));
    // the same forward replayed as a CUDA graph
    cudaGraph_t g;
    cudaGraphExec_t ge;
    CUDA_CHECK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    m.forward(false);
    CUDA_CHECK(cudaStreamEndCapture(st, &g));
    CUDA_CHECK(cudaGraphInstantiate(&ge, g, 0));
    for (int i = 0; i < 3; i++) CUDA_CHECK(cudaGraphLaunch(ge, st));
    CUDA_CHECK(cudaEventRecord(e0, st));
    for (int i = 0; i < iters; i++) CUDA_CHECK(cudaGraphLaunch(ge, st));
    CUDA_CHECK(cudaEventRecord(e1, st));
    CUDA_CHECK(cudaEventSynchronize(e1));
    float graph_ms = 0.f;
    CUDA_CHECK(cudaEventElapsedTime(&graph_ms, e0, e1));
    const float best = std::min(eager_ms, graph_ms) / iters;
    printf("{\"impl\": \"reference-cudnn\", \"batch\": %d, \"imgsz\": %d, \"iters\": %d, \"eager_ms\": %.4f, "
           "\"graph_ms\": %.4f, \"img_per_s\": %.2f, \"build_s\": %.1f, \"precision\": \"%s\"}\n",
           B, S, iters, eager_ms / iters, graph_ms / iters, B / (best / 1e3), build_s,
           sizeof(act_t) == 2 ? "fp16" : "fp32");
    CUDA_CHECK(cudaGraphExecDestroy(ge));
    CUDA_CHECK(cudaGraphDestroy(g));
  }
  return 0;
}
