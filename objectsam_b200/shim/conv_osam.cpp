// ConvOp on the B200 kernels: a drop-in replacement for the reference's src/conv.cpp.
//
// Compiled against the reference's own, unmodified src/conv.h, so its callers — src/model.cpp
// (Model::build / forward / backward), tests/bench_train.cpp, tests/parity.cpp, teacher/tnet.cpp — build
// and run unchanged; link this file and libosam.so in place of src/conv.cpp (oracle/Makefile, targets
// shim_*).  Every member goes through the C ABI of include/osam.h:
//   init       → the plan of (geometry, transposed).  Plans are immutable host objects that depend on the
//                geometry alone, so ConvOps of the same geometry share one, from a process-wide cache;
//                nothing is stored in ConvOp's cuDNN members (descriptors, algorithms, backend plans),
//                which stay at their defaults.
//   tune       → the plan's workspace size (osam_conv_workspace_size), checked against ws_limit; like
//                cuDNN's find, each direction runs on the caller's buffers and is timed once with CUDA
//                events (tuned_ms: forward, input gradient, weight gradient — for the transposed conv in
//                the layer's own sense).  A direction the kernels do not implement for the geometry (the
//                input gradient of the 3-channel stem, which the model never asks for) is timed as 0.
//   tune_fwd   → the same for the forward alone.
//   fwd / fwd_v / dgrad / wgrad → osam_conv_fwd / osam_conv_dgrad / osam_conv_wgrad with the same beta,
//                on the stream of the cuDNN handle (cudnnGetStream, as the reference's calls use it: the
//                model switches that stream around its weight gradients).
// Data types: the kernels take fp16 activations and weights (the reference's default build,
// act_t = __half).  init with any other cudnnDataType_t (the fp32 parity build, -DFSO_FP32) aborts with a
// message: that build needs the reference's own cuDNN path.
// Errors abort like the reference's CUDNN_CHECK / FSO_ASSERT.  Launches are asynchronous, so a kernel
// whose bounded wait ran out (it returns early and records OSAM_ERR_TIMEOUT) is caught at the next
// ConvOp call, which polls the library's host-mapped error word (osam_device_error_peek, no
// synchronisation), and at tune, which synchronises anyway (osam_device_error).
#include <array>
#include <map>
#include <mutex>

#include "conv.h"
#include "osam.h"

namespace {

osam_conv_plan* plan_for(const ConvGeom& g, bool transposed) {
  static std::mutex mu;
  static std::map<std::array<int, 10>, osam_conv_plan*> cache;  // lives until the process exits
  const std::array<int, 10> key = {g.N, g.H, g.W, g.C, g.K, g.R, g.S, g.stride, g.pad, transposed ? 1 : 0};
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  const osam_conv_geom og{g.N, g.H, g.W, g.C, g.K, g.R, g.S, g.stride, g.pad};
  osam_conv_plan* p = nullptr;
  const int rc = osam_conv_plan_create(&og, transposed ? 1 : 0, &p);
  FSO_ASSERT(rc == OSAM_OK, "osam_conv_plan_create(N=%d H=%d W=%d C=%d K=%d R=%d S=%d stride=%d pad=%d%s): %s", g.N,
             g.H, g.W, g.C, g.K, g.R, g.S, g.stride, g.pad, transposed ? " transposed" : "", osam_last_error());
  cache.emplace(key, p);
  return p;
}

cudaStream_t stream_of(cudnnHandle_t h) {
  cudaStream_t s = nullptr;
  CUDNN_CHECK(cudnnGetStream(h, &s));
  return s;
}

osam_stream_t as_osam(cudaStream_t s) { return reinterpret_cast<osam_stream_t>(s); }

// Before a launch: a kernel that already finished with a timed-out wait stops the program here.
void poll_device_error() {
  const int v = osam_device_error_peek();
  FSO_ASSERT(v == 0, "a conv kernel reported device error %d (a bounded wait ran out): %s", v, osam_last_error());
}

void check(int rc, const char* what, const ConvGeom& g) {
  FSO_ASSERT(rc == OSAM_OK, "%s (N=%d H=%d W=%d C=%d K=%d R=%d stride=%d): %s", what, g.N, g.H, g.W, g.C, g.K, g.R,
             g.stride, osam_last_error());
}

// Mean time of `reps` runs of `op` on stream s after one untimed run; op returns an osam status.
template <class F>
float time_op(cudaStream_t s, F op, int* status) {
  *status = op();
  if (*status != OSAM_OK) return 0.f;
  cudaEvent_t e0, e1;
  CUDA_CHECK(cudaEventCreate(&e0));
  CUDA_CHECK(cudaEventCreate(&e1));
  const int reps = 3;
  CUDA_CHECK(cudaEventRecord(e0, s));
  for (int i = 0; i < reps && *status == OSAM_OK; i++) *status = op();
  CUDA_CHECK(cudaEventRecord(e1, s));
  CUDA_CHECK(cudaEventSynchronize(e1));
  float ms = 0.f;
  CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
  CUDA_CHECK(cudaEventDestroy(e0));
  CUDA_CHECK(cudaEventDestroy(e1));
  return ms / reps;
}

}  // namespace

void ConvOp::init(cudnnHandle_t h, const ConvGeom& g, bool transposed, cudnnDataType_t dt) {
  FSO_ASSERT(dt == CUDNN_DATA_HALF,
             "ConvOp on the B200 kernels takes fp16 activations and weights; data type %d needs the cuDNN path",
             (int)dt);
  if (transposed)
    FSO_ASSERT(g.R == g.stride && g.S == g.stride && g.pad == 0, "transposed conv: kernel = stride, pad 0");
  h_ = h;
  g_ = g;
  tr_ = transposed;
  dt_ = dt;
  plan_for(g_, tr_);  // the plan exists from init on: never created inside a (possibly captured) launch
}

int64_t ConvOp::out_elems() const { return osam_conv_out_elems(plan_for(g_, tr_)); }

size_t ConvOp::tune(act_t* x, act_t* w, act_t* y, act_t* dx, act_t* dw, act_t* dy, void* ws, size_t ws_limit,
                    float dgrad_beta) {
  const osam_conv_plan* p = plan_for(g_, tr_);
  const size_t need = osam_conv_workspace_size(p);
  FSO_ASSERT(need <= ws_limit, "conv workspace %zu B exceeds the tuning limit %zu B", need, ws_limit);
  const cudaStream_t s = stream_of(h_);
  int st = OSAM_OK;
  tuned_ms[0] = time_op(s, [&] { return osam_conv_fwd(p, x, w, y, 0.f, ws, ws_limit, as_osam(s)); }, &st);
  check(st, "ConvOp::tune forward", g_);
  tuned_ms[1] = time_op(s, [&] { return osam_conv_dgrad(p, dy, w, dx, dgrad_beta, ws, ws_limit, as_osam(s)); }, &st);
  if (st == OSAM_ERR_UNSUPPORTED) tuned_ms[1] = 0.f;  // not needed by the model for this layer (the stem)
  else check(st, "ConvOp::tune input gradient", g_);
  tuned_ms[2] = time_op(s, [&] { return osam_conv_wgrad(p, x, dy, dw, 0.f, ws, ws_limit, as_osam(s)); }, &st);
  if (st == OSAM_ERR_UNSUPPORTED) tuned_ms[2] = 0.f;
  else check(st, "ConvOp::tune weight gradient", g_);
  const int v = osam_device_error();  // tune synchronises anyway: read and clear the error word
  FSO_ASSERT(v == 0, "a conv kernel reported device error %d while tuning", v);
  return need;
}

size_t ConvOp::tune_fwd(void* x, void* w, void* y, void* ws, size_t ws_limit) {
  FSO_ASSERT(!tr_, "tune_fwd: forward-only tuning is for ordinary convs");
  const osam_conv_plan* p = plan_for(g_, tr_);
  const size_t need = osam_conv_workspace_size(p);
  FSO_ASSERT(need <= ws_limit, "conv workspace %zu B exceeds the tuning limit %zu B", need, ws_limit);
  const cudaStream_t s = stream_of(h_);
  int st = OSAM_OK;
  tuned_ms[0] = time_op(s, [&] { return osam_conv_fwd(p, x, w, y, 0.f, ws, ws_limit, as_osam(s)); }, &st);
  check(st, "ConvOp::tune_fwd", g_);
  const int v = osam_device_error();
  FSO_ASSERT(v == 0, "a conv kernel reported device error %d while tuning", v);
  return need;
}

void ConvOp::fwd_v(const void* x, const void* w, void* y, void* ws, size_t wsz) const {
  poll_device_error();
  check(osam_conv_fwd(plan_for(g_, tr_), x, w, y, 0.f, ws, wsz, as_osam(stream_of(h_))), "ConvOp::fwd_v", g_);
}

void ConvOp::fwd(const act_t* x, const act_t* w, act_t* y, void* ws, size_t wsz, float beta) const {
  poll_device_error();
  check(osam_conv_fwd(plan_for(g_, tr_), x, w, y, beta, ws, wsz, as_osam(stream_of(h_))), "ConvOp::fwd", g_);
}

void ConvOp::dgrad(const act_t* dy, const act_t* w, act_t* dx, void* ws, size_t wsz, float beta) const {
  poll_device_error();
  check(osam_conv_dgrad(plan_for(g_, tr_), dy, w, dx, beta, ws, wsz, as_osam(stream_of(h_))), "ConvOp::dgrad", g_);
}

void ConvOp::wgrad(const act_t* x, const act_t* dy, act_t* dw, void* ws, size_t wsz, float beta) const {
  poll_device_error();
  check(osam_conv_wgrad(plan_for(g_, tr_), x, dy, dw, beta, ws, wsz, as_osam(stream_of(h_))), "ConvOp::wgrad", g_);
}
