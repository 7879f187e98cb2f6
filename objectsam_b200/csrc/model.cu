// YOLOv8s-seg (nc = 1) inference graph on the fused conv kernels (C ABI: osam_model_*).
//
// Same topology, parameter names and activation routing as the reference's Model (src/model.cpp:168-275):
// concat is implicit — each producer's epilogue writes straight into its slices of the concat buffers
// (with the 2× nearest upsample for the neck), C2f's cv1 writes both the concat buffer and the first
// bottleneck input, and the three first convs of each head level share one K = 64+128+32 conv.
// Differences by design: eval-mode BN is folded into each conv's epilogue (no z buffer, no apply pass),
// head/upsample biases are applied in the epilogue, SPPF's three pools are one kernel, and the whole
// forward can be replayed as one CUDA graph.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "conv_internal.h"

namespace osam {
int model_fail(int code, const char* fmt, ...);
}

namespace {
using namespace osam;

struct MAct {
  std::string name;
  int C = 0, H = 0, W = 0;
  __half* p = nullptr;
  size_t off = 0;     // byte offset in the activation arena
  __half* g = nullptr;  // training: gradient buffer (same shape), none for the input image
};

struct MDest {
  MAct* a;
  int choff, c0, c1, up;
};

enum NodeKind { N_CONVBN = 0, N_HEAD = 1, N_CONVT = 2, N_POOL = 3 };

struct MNode {
  NodeKind kind;
  std::string name;
  MAct* in = nullptr;
  int K = 0, k = 1, s = 1;
  std::vector<std::string> pre;  // parameter prefixes (three for a fused head conv)
  std::vector<int> ks;           // output channels per prefix
  std::vector<MDest> dests;
  MAct* res = nullptr;
  MAct* out = nullptr;
  MAct* cat = nullptr;
  int pc = 0;
  osam_conv_plan plan{};
  ConvLaunch L{};
  size_t w_off = 0;  // fp16 weight arena offset (elements)
  size_t f_off = 0;  // fp32 arena offset: scale[K] + shift[K] (CONVBN) or bias[K]
  // training
  __half* z = nullptr;       // CONVBN: conv output before BN (fp16, as the reference stores it)
  size_t t_off = 0;          // CONVBN: fp32 train arena: γ, β, running μ, running σ², mean, istd, scale, shift
  size_t g_off = 0, g_w = 0;  // fp32 parameter-gradient arena: weights (g_w elements) then γ, β or the bias
  __half* pre_w = nullptr;     // this node's re-laid-out dgrad weights (nullptr: none needed)
  bool res_accum = false, dgrad_accum = false;
};

struct PInfo {
  std::vector<int64_t> shape;
  std::vector<float> host;
  bool set = false;
};

__global__ void k_f32_to_f16(const float* __restrict__ s, __half* __restrict__ d, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    d[i] = __float2half_rn(s[i]);
}
// Eval-mode BN fold, same formula as the reference's k_eval_scale (src/bn.cu:277-284).
__global__ void k_bn_fold(const float* __restrict__ gbmv, int C, float eps, float* __restrict__ scale,
                          float* __restrict__ shift) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const float g = gbmv[c], b = gbmv[C + c], rm = gbmv[2 * C + c], rv = gbmv[3 * C + c];
  const float sc = g * rsqrtf(rv + eps);
  scale[c] = sc;
  shift[c] = b - rm * sc;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

struct osam_model {
  int N = 0, S = 0, reg_max = 16;
  float bn_eps = 1e-3f;
  std::map<std::string, std::unique_ptr<MAct>> acts;
  std::vector<std::unique_ptr<MNode>> nodes;
  std::map<std::string, PInfo> params;
  std::vector<std::string> porder;
  MAct* in = nullptr;
  MAct* head[3][3] = {};
  MAct* proto = nullptr;
  uint8_t* arena = nullptr;
  size_t arena_bytes = 0;
  __half* w16 = nullptr;
  size_t w16_n = 0;
  float* f32 = nullptr;
  size_t f32_n = 0;
  bool synced = false;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaStream_t cap = nullptr;  // private stream the graph is recorded on (the legacy stream cannot capture)
  // training (osam_model_train_init)
  bool train = false;
  uint8_t* garena = nullptr;   // activation gradients
  __half* zarena = nullptr;    // z of every CONVBN node
  float* tarena = nullptr;     // BN parameters and batch statistics
  float* grad32 = nullptr;     // parameter gradients, nodes in reverse order (contiguous DP buckets)
  size_t grad32_n = 0;
  __half* dz = nullptr;        // one node's dz (fp16), reused
  __half* gw16 = nullptr;      // one node's fp16 weight gradient, reused
  __half* wconvt = nullptr;    // transposed conv weights in the reference's (C_in, R, S, C_out) layout
  void* ws = nullptr;          // conv workspace (max over nodes)
  size_t ws_bytes = 0;
  void* bnws = nullptr;        // zero-filled BN / channel-sum accumulators
  size_t bnws_bytes = 0;
  // backward: weight gradients run on a side stream, overlapping the next node's BN backward and input
  // gradient on the caller's stream (the reference's wgrad_side, src/model.cpp:416-428); two dz buffers
  // alternate so a node's BN backward never overwrites the dz a pending weight gradient still reads
  __half* dz2 = nullptr;
  void* ws_side = nullptr;
  // the input-gradient convs' re-laid-out weights, all nodes, refreshed by one batched launch per step
  __half* prelaid = nullptr;
  DgradJob* jobs = nullptr;
  int njobs = 0;
  cudaStream_t side = nullptr;
  cudaEvent_t ev_dz[2] = {}, ev_wg[2] = {}, ev_fork = nullptr, ev_join = nullptr;
  // forward on several streams: nodes that do not depend on each other (the neck's PAN path, the three
  // head levels and their branches, the proto chain) overlap, so small layers fill the SMs that a big one
  // leaves idle in its last wave.  Stream 0 is the caller's; the schedule is fixed at the first forward.
  static constexpr int kFwdStreams = 3;
  cudaStream_t fwd_st[kFwdStreams - 1] = {};
  std::vector<int> node_order;               // launch order: topological, longest remaining path first
  std::vector<int> node_stream;              // per node: 0 … kFwdStreams − 1
  std::vector<std::vector<int>> node_waits;  // per node: producers on other streams (latest per stream)
  std::vector<cudaEvent_t> node_ev;          // per node: recorded after it when another stream waits on it
  cudaEvent_t ev_fwd_start = nullptr, ev_fwd_end[kFwdStreams - 1] = {};

  // ------------------------------------------------------------------ graph construction
  MAct* act(const std::string& n, int C, int H, int W) {
    auto a = std::make_unique<MAct>();
    a->name = n;
    a->C = C;
    a->H = H;
    a->W = W;
    MAct* p = a.get();
    acts[n] = std::move(a);
    return p;
  }
  void add_param(const std::string& name, std::vector<int64_t> shape) {
    params[name].shape = std::move(shape);
    porder.push_back(name);
  }
  void convbn(const std::string& name, MAct* in_, int K, int k, int s, std::vector<MDest> dests, MAct* res = nullptr,
              std::vector<std::string> fused = {}, std::vector<int> fused_k = {}) {
    auto nd = std::make_unique<MNode>();
    nd->kind = N_CONVBN;
    nd->name = name;
    nd->in = in_;
    nd->K = K;
    nd->k = k;
    nd->s = s;
    nd->pre = fused.empty() ? std::vector<std::string>{name} : fused;
    nd->ks = fused.empty() ? std::vector<int>{K} : fused_k;
    for (size_t i = 0; i < nd->pre.size(); i++) {
      const std::string& p = nd->pre[i];
      add_param(p + ".conv.weight", {nd->ks[i], in_->C, k, k});
      for (const char* b : {".bn.weight", ".bn.bias", ".bn.running_mean", ".bn.running_var"})
        add_param(p + b, {nd->ks[i]});
    }
    for (auto& d : dests)
      if (d.c1 == 0) d.c1 = K;
    nd->dests = dests;
    nd->res = res;
    nodes.push_back(std::move(nd));
  }
  MAct* c2f(const std::string& name, MAct* x, int c2, int n, bool shortcut, std::vector<MDest> out) {
    const int c = c2 / 2, H = x->H, W = x->W;
    MAct* cat = act(name + ".cat", (2 + n) * c, H, W);
    MAct* bin = act(name + ".m0.in", c, H, W);
    convbn(name + ".cv1", x, 2 * c, 1, 1, {{cat, 0, 0, 2 * c, 1}, {bin, 0, c, 2 * c, 1}});
    for (int j = 0; j < n; j++) {
      const std::string mj = name + ".m." + std::to_string(j);
      MAct* t = act(mj + ".t", c, H, W);
      convbn(mj + ".cv1", bin, c, 3, 1, {{t, 0, 0, c, 1}});
      std::vector<MDest> d = {{cat, (2 + j) * c, 0, c, 1}};
      MAct* next = nullptr;
      if (j + 1 < n) {
        next = act(name + ".m" + std::to_string(j + 1) + ".in", c, H, W);
        d.push_back({next, 0, 0, c, 1});
      }
      convbn(mj + ".cv2", t, c, 3, 1, d, shortcut ? bin : nullptr);
      bin = next;
    }
    convbn(name + ".cv2", cat, c2, 1, 1, out);
    return cat;
  }
  void head_conv(const std::string& name, MAct* x, int K, MAct* out) {
    auto nd = std::make_unique<MNode>();
    nd->kind = N_HEAD;
    nd->name = name;
    nd->in = x;
    nd->K = K;
    nd->out = out;
    add_param(name + ".weight", {K, x->C, 1, 1});
    add_param(name + ".bias", {K});
    nodes.push_back(std::move(nd));
  }

  void build() {
    auto M = [](int i) { return "model." + std::to_string(i); };
    in = act("in", 3, S, S);
    MAct* a0 = act("a0", 32, S / 2, S / 2);
    convbn(M(0), in, 32, 3, 2, {{a0, 0, 0, 0, 1}});
    MAct* a1 = act("a1", 64, S / 4, S / 4);
    convbn(M(1), a0, 64, 3, 2, {{a1, 0, 0, 0, 1}});
    MAct* a2 = act("a2", 64, S / 4, S / 4);
    c2f(M(2), a1, 64, 1, true, {{a2, 0, 0, 0, 1}});
    MAct* a3 = act("a3", 128, S / 8, S / 8);
    convbn(M(3), a2, 128, 3, 2, {{a3, 0, 0, 0, 1}});
    MAct* cat11 = act("cat11", 768, S / 16, S / 16);
    MAct* cat14 = act("cat14", 384, S / 8, S / 8);
    MAct* cat17 = act("cat17", 384, S / 16, S / 16);
    MAct* cat20 = act("cat20", 768, S / 32, S / 32);
    MAct* a4 = act("a4", 128, S / 8, S / 8);
    c2f(M(4), a3, 128, 2, true, {{a4, 0, 0, 0, 1}, {cat14, 256, 0, 0, 1}});
    MAct* a5 = act("a5", 256, S / 16, S / 16);
    convbn(M(5), a4, 256, 3, 2, {{a5, 0, 0, 0, 1}});
    MAct* a6 = act("a6", 256, S / 16, S / 16);
    c2f(M(6), a5, 256, 2, true, {{a6, 0, 0, 0, 1}, {cat11, 512, 0, 0, 1}});
    MAct* a7 = act("a7", 512, S / 32, S / 32);
    convbn(M(7), a6, 512, 3, 2, {{a7, 0, 0, 0, 1}});
    MAct* a8 = act("a8", 512, S / 32, S / 32);
    c2f(M(8), a7, 512, 1, true, {{a8, 0, 0, 0, 1}});
    MAct* sp = act(M(9) + ".cat", 1024, S / 32, S / 32);
    convbn(M(9) + ".cv1", a8, 256, 1, 1, {{sp, 0, 0, 0, 1}});
    {
      auto nd = std::make_unique<MNode>();
      nd->kind = N_POOL;
      nd->name = M(9) + ".m";
      nd->cat = sp;
      nd->pc = 256;
      nodes.push_back(std::move(nd));
    }
    convbn(M(9) + ".cv2", sp, 512, 1, 1, {{cat11, 0, 0, 0, 2}, {cat20, 256, 0, 0, 1}});
    c2f(M(12), cat11, 256, 1, false, {{cat14, 0, 0, 0, 2}, {cat17, 128, 0, 0, 1}});
    MAct* p3 = act("p3", 128, S / 8, S / 8);
    c2f(M(15), cat14, 128, 1, false, {{p3, 0, 0, 0, 1}});
    convbn(M(16), p3, 128, 3, 2, {{cat17, 0, 0, 0, 1}});
    MAct* p4 = act("p4", 256, S / 16, S / 16);
    c2f(M(18), cat17, 256, 1, false, {{p4, 0, 0, 0, 1}});
    convbn(M(19), p4, 256, 3, 2, {{cat20, 0, 0, 0, 1}});
    MAct* p5 = act("p5", 512, S / 32, S / 32);
    c2f(M(21), cat20, 512, 1, false, {{p5, 0, 0, 0, 1}});
    // Segment head: per level one fused 3×3 conv (box c2 | cls 128 | coef 32), then the three branches.
    const int R4 = 4 * reg_max;
    const int c2 = std::max(16, std::max(128 / 4, R4));
    const int KH = c2 + 128 + 32;
    MAct* P[3] = {p3, p4, p5};
    const std::string hd = M(22);
    for (int l = 0; l < 3; l++) {
      const std::string L = std::to_string(l);
      const int H = P[l]->H, W = P[l]->W;
      MAct* hb = act("h" + L + ".b1", c2, H, W);
      MAct* hc = act("h" + L + ".c1", 128, H, W);
      MAct* hm = act("h" + L + ".m1", 32, H, W);
      convbn(hd + ".h" + L + ".0", P[l], KH, 3, 1,
             {{hb, 0, 0, c2, 1}, {hc, 0, c2, c2 + 128, 1}, {hm, 0, c2 + 128, KH, 1}}, nullptr,
             {hd + ".cv2." + L + ".0", hd + ".cv3." + L + ".0", hd + ".cv4." + L + ".0"}, {c2, 128, 32});
      MAct* hb2 = act("h" + L + ".b2", c2, H, W);
      MAct* hc2 = act("h" + L + ".c2", 128, H, W);
      MAct* hm2 = act("h" + L + ".m2", 32, H, W);
      convbn(hd + ".cv2." + L + ".1", hb, c2, 3, 1, {{hb2, 0, 0, 0, 1}});
      convbn(hd + ".cv3." + L + ".1", hc, 128, 3, 1, {{hc2, 0, 0, 0, 1}});
      convbn(hd + ".cv4." + L + ".1", hm, 32, 3, 1, {{hm2, 0, 0, 0, 1}});
      head[0][l] = act("out.box" + L, R4, H, W);
      head[1][l] = act("out.cls" + L, 1, H, W);
      head[2][l] = act("out.coef" + L, 32, H, W);
      head_conv(hd + ".cv2." + L + ".2", hb2, R4, head[0][l]);
      head_conv(hd + ".cv3." + L + ".2", hc2, 1, head[1][l]);
      head_conv(hd + ".cv4." + L + ".2", hm2, 32, head[2][l]);
    }
    MAct* pr1 = act("proto.1", 128, S / 8, S / 8);
    convbn(hd + ".proto.cv1", p3, 128, 3, 1, {{pr1, 0, 0, 0, 1}});
    MAct* pru = act("proto.up", 128, S / 4, S / 4);
    {
      auto nd = std::make_unique<MNode>();
      nd->kind = N_CONVT;
      nd->name = hd + ".proto.upsample";
      nd->in = pr1;
      nd->out = pru;
      nd->K = 128;
      add_param(nd->name + ".weight", {128, 128, 2, 2});
      add_param(nd->name + ".bias", {128});
      nodes.push_back(std::move(nd));
    }
    MAct* pr2 = act("proto.2", 128, S / 4, S / 4);
    convbn(hd + ".proto.cv2", pru, 128, 3, 1, {{pr2, 0, 0, 0, 1}});
    proto = act("out.proto", 32, S / 4, S / 4);
    convbn(hd + ".proto.cv3", pr2, 32, 1, 1, {{proto, 0, 0, 0, 1}});
  }

  int allocate() {
    size_t off = 0;
    for (auto& kv : acts) {
      MAct* a = kv.second.get();
      a->off = off;
      off = align_up(off + (size_t)N * a->H * a->W * a->C * sizeof(__half), 1024);
    }
    arena_bytes = off;
    cudaError_t e = cudaMalloc(&arena, arena_bytes);
    if (e != cudaSuccess) return model_fail(OSAM_ERR_NOMEM, "activation arena (%zu B): %s", arena_bytes, cudaGetErrorString(e));
    cudaMemset(arena, 0, arena_bytes);
    for (auto& kv : acts) kv.second->p = reinterpret_cast<__half*>(arena + kv.second->off);
    // weight / fp32 arenas
    size_t w = 0, f = 0;
    for (auto& nd : nodes) {
      if (nd->kind == N_POOL) continue;
      const int C = nd->in->C;
      nd->w_off = w;
      const size_t wn = nd->kind == N_CONVT ? (size_t)C * 4 * nd->K : (size_t)nd->K * nd->k * nd->k * C;
      w = align_up(w + wn, 64);
      nd->f_off = f;
      f = align_up(f + (nd->kind == N_CONVBN ? 2 * (size_t)nd->K : (size_t)nd->K), 32);
    }
    w16_n = w;
    f32_n = f;
    if ((e = cudaMalloc(&w16, w16_n * sizeof(__half))) != cudaSuccess) return model_fail(OSAM_ERR_NOMEM, "weights");
    if ((e = cudaMalloc(&f32, f32_n * sizeof(float))) != cudaSuccess) return model_fail(OSAM_ERR_NOMEM, "bn arena");
    return OSAM_OK;
  }

  static void free_subplans(osam_conv_plan& p) {
    for (int i = 0; i < 4; i++) {
      delete p.dg[i];
      p.dg[i] = nullptr;
    }
  }

  void release() {
    // the instantiated graph refers to the forward's streams' events: destroy it first
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    exec = nullptr;
    graph = nullptr;
    for (auto& nd : nodes) free_subplans(nd->plan);
    cudaFree(garena);
    cudaFree(zarena);
    cudaFree(tarena);
    cudaFree(grad32);
    cudaFree(dz);
    cudaFree(gw16);
    cudaFree(wconvt);
    cudaFree(ws);
    cudaFree(bnws);
    cudaFree(dz2);
    cudaFree(ws_side);
    cudaFree(prelaid);
    cudaFree(jobs);
    prelaid = nullptr;
    jobs = nullptr;
    njobs = 0;
    for (int i = 0; i < 2; i++) {
      if (ev_dz[i]) cudaEventDestroy(ev_dz[i]);
      if (ev_wg[i]) cudaEventDestroy(ev_wg[i]);
      ev_dz[i] = ev_wg[i] = nullptr;
    }
    if (ev_fork) cudaEventDestroy(ev_fork);
    if (ev_join) cudaEventDestroy(ev_join);
    if (side) cudaStreamDestroy(side);
    for (cudaEvent_t ev : node_ev)
      if (ev) cudaEventDestroy(ev);
    node_ev.clear();
    node_order.clear();
    node_stream.clear();
    node_waits.clear();
    for (int k = 0; k < kFwdStreams - 1; k++) {
      if (fwd_st[k]) cudaStreamDestroy(fwd_st[k]);
      if (ev_fwd_end[k]) cudaEventDestroy(ev_fwd_end[k]);
      fwd_st[k] = nullptr;
      ev_fwd_end[k] = nullptr;
    }
    if (ev_fwd_start) cudaEventDestroy(ev_fwd_start);
    ev_fwd_start = nullptr;
    ev_fork = ev_join = nullptr;
    side = nullptr;
    dz2 = nullptr;
    ws_side = nullptr;
    garena = nullptr;
    zarena = nullptr;
    tarena = nullptr;
    grad32 = nullptr;
    dz = gw16 = wconvt = nullptr;
    ws = bnws = nullptr;
    train = false;
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (cap) cudaStreamDestroy(cap);
    exec = nullptr;
    graph = nullptr;
    cap = nullptr;
    cudaFree(arena);
    cudaFree(w16);
    cudaFree(f32);
    arena = nullptr;
    w16 = nullptr;
    f32 = nullptr;
  }

  // ------------------------------------------------------------------ weights
  int sync(cudaStream_t st) {
    for (auto& n : porder)
      if (!params[n].set) return model_fail(OSAM_ERR_INVALID, "parameter %s was not set", n.c_str());
    std::vector<float> wst(w16_n, 0.f);  // fp32 staging of the fp16 weight arena
    std::vector<float> bnst;             // [γ|β|μ|σ²] per CONVBN node, concatenated
    std::vector<size_t> bn_at(nodes.size(), 0);
    std::vector<float> fst(f32_n, 0.f);  // biases go straight into the fp32 arena
    for (size_t ni = 0; ni < nodes.size(); ni++) {
      MNode& nd = *nodes[ni];
      if (nd.kind == N_POOL) continue;
      const int C = nd.in->C, k = nd.k;
      if (nd.kind == N_CONVBN) {
        // KRSC: the fused head concatenates its prefixes along K
        int k0 = 0;
        bn_at[ni] = bnst.size();
        bnst.resize(bnst.size() + 4 * (size_t)nd.K);
        for (size_t pi = 0; pi < nd.pre.size(); pi++) {
          const PInfo& W = params[nd.pre[pi] + ".conv.weight"];
          const int Kp = nd.ks[pi];
          for (int kk = 0; kk < Kp; kk++)
            for (int r = 0; r < k; r++)
              for (int s = 0; s < k; s++)
                for (int c = 0; c < C; c++)
                  wst[nd.w_off + (((size_t)(k0 + kk) * k + r) * k + s) * C + c] =
                      W.host[(((size_t)kk * C + c) * k + r) * k + s];
          const char* bnn[4] = {".bn.weight", ".bn.bias", ".bn.running_mean", ".bn.running_var"};
          for (int q = 0; q < 4; q++) {
            const PInfo& B = params[nd.pre[pi] + bnn[q]];
            for (int kk = 0; kk < Kp; kk++) bnst[bn_at[ni] + (size_t)q * nd.K + k0 + kk] = B.host[kk];
          }
          k0 += Kp;
        }
      } else if (nd.kind == N_HEAD) {
        const PInfo& W = params[nd.name + ".weight"];
        for (int kk = 0; kk < nd.K; kk++)
          for (int c = 0; c < C; c++) wst[nd.w_off + (size_t)kk * C + c] = W.host[(size_t)kk * C + c];
        const PInfo& B = params[nd.name + ".bias"];
        for (int kk = 0; kk < nd.K; kk++) fst[nd.f_off + kk] = B.host[kk];
      } else {  // N_CONVT: PyTorch (C_in, C_out, 2, 2) → GEMM B rows ((dy·2+dx)·K + k), K-major over C_in
        const PInfo& W = params[nd.name + ".weight"];
        for (int c = 0; c < C; c++)
          for (int kk = 0; kk < nd.K; kk++)
            for (int dy = 0; dy < 2; dy++)
              for (int dx = 0; dx < 2; dx++)
                wst[nd.w_off + ((size_t)(dy * 2 + dx) * nd.K + kk) * C + c] =
                    W.host[(((size_t)c * nd.K + kk) * 2 + dy) * 2 + dx];
        const PInfo& B = params[nd.name + ".bias"];
        for (int kk = 0; kk < nd.K; kk++) fst[nd.f_off + kk] = B.host[kk];
      }
    }
    float* dw = nullptr;
    float* dbn = nullptr;
    cudaError_t e;
    if ((e = cudaMalloc(&dw, wst.size() * sizeof(float))) != cudaSuccess) return model_fail(OSAM_ERR_NOMEM, "staging");
    if ((e = cudaMalloc(&dbn, std::max<size_t>(bnst.size(), 1) * sizeof(float))) != cudaSuccess) {
      cudaFree(dw);
      return model_fail(OSAM_ERR_NOMEM, "staging");
    }
    cudaMemcpyAsync(dw, wst.data(), wst.size() * sizeof(float), cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(dbn, bnst.data(), bnst.size() * sizeof(float), cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(f32, fst.data(), fst.size() * sizeof(float), cudaMemcpyHostToDevice, st);
    k_f32_to_f16<<<1024, 256, 0, st>>>(dw, w16, (long long)w16_n);
    for (size_t ni = 0; ni < nodes.size(); ni++) {
      MNode& nd = *nodes[ni];
      if (nd.kind != N_CONVBN) continue;
      k_bn_fold<<<(nd.K + 127) / 128, 128, 0, st>>>(dbn + bn_at[ni], nd.K, bn_eps, f32 + nd.f_off,
                                                    f32 + nd.f_off + nd.K);
    }
    e = cudaStreamSynchronize(st);
    cudaFree(dw);
    cudaFree(dbn);
    if (e != cudaSuccess) return model_fail(OSAM_ERR_CUDA, "weight upload: %s", cudaGetErrorString(e));
    int rc = prepare_launches();
    if (rc) return rc;
    synced = true;
    if (exec) {  // weights changed: the graph's kernel arguments are unchanged (same buffers), keep it
    }
    return OSAM_OK;
  }

  int prepare_launches() {
    for (auto& ndp : nodes) {
      MNode& nd = *ndp;
      if (nd.kind == N_POOL) {
        if (sppf_prime() != cudaSuccess) return model_fail(OSAM_ERR_CUDA, "sppf setup");
        continue;
      }
      osam_conv_geom g{N, nd.in->H, nd.in->W, nd.in->C, nd.K, nd.k, nd.k, nd.s, nd.k / 2};
      if (nd.kind == N_HEAD) g = osam_conv_geom{N, nd.in->H, nd.in->W, nd.in->C, nd.K, 1, 1, 1, 0};
      if (nd.kind == N_CONVT) g = osam_conv_geom{N, nd.in->H, nd.in->W, nd.in->C, nd.K, 2, 2, 2, 0};
      osam_conv_plan* plan = nullptr;
      int rc = osam_conv_plan_create(&g, nd.kind == N_CONVT, &plan);
      if (rc) return model_fail(rc, "%s: %s", nd.name.c_str(), osam_last_error());
      free_subplans(nd.plan);
      nd.plan = *plan;  // the node owns the plan's gradient sub-plans from here on
      for (int i = 0; i < 4; i++) plan->dg[i] = nullptr;
      osam_conv_plan_destroy(plan);
      osam_epilogue ep{};
      ep.round_z = 0;  // keep z in fp32 into BN/SiLU (the reference rounds it to fp16 first: ≤ 1 ulp apart)
      if (nd.kind == N_CONVBN) {
        ep.kind = OSAM_EPI_BN_ACT;
        ep.scale = f32 + nd.f_off;
        ep.shift = f32 + nd.f_off + nd.K;
        ep.act = 1;
        ep.res = nd.res ? nd.res->p : nullptr;
        ep.n_dest = (int)nd.dests.size();
        for (size_t i = 0; i < nd.dests.size(); i++) {
          const MDest& d = nd.dests[i];
          ep.dest[i] = osam_dest{d.a->p, d.a->C, d.choff, d.c0, d.c1, d.up};
        }
      } else {
        ep.kind = OSAM_EPI_BIAS;
        ep.bias = f32 + nd.f_off;
        ep.n_dest = 1;
        ep.dest[0] = osam_dest{nd.out->p, nd.out->C, 0, 0, nd.K, 1};
      }
      rc = conv_prepare(&nd.plan, nd.in->p, w16 + nd.w_off, &ep, 0.f, nullptr, nullptr, 0, &nd.L, true);
      if (rc) return model_fail(rc, "%s: %s", nd.name.c_str(), osam_last_error());
      if (conv_prime(nd.L) != cudaSuccess) return model_fail(OSAM_ERR_CUDA, "%s: kernel setup", nd.name.c_str());
    }
    return OSAM_OK;
  }

  // Dependency DAG of the forward (a node depends on every earlier writer of an activation it reads;
  // concat buffers are written by several nodes into disjoint channel slices).  Nodes are launched in a
  // topological order that puts the longest remaining chain (by FLOPs) first — so the proto branch starts
  // as soon as its input exists — and assigned greedily to kFwdStreams streams: a node continues the
  // stream whose last node is its latest producer, else takes the stream idle longest.
  cudaError_t plan_streams() {
    if (!node_stream.empty()) return cudaSuccess;
    const int n = (int)nodes.size();
    std::map<const MAct*, std::vector<int>> writers;
    std::vector<std::vector<const MAct*>> rd(n);
    for (int i = 0; i < n; i++) {
      const MNode& nd = *nodes[i];
      if (nd.kind == N_POOL) {
        rd[i].push_back(nd.cat);
        writers[nd.cat].push_back(i);
        continue;
      }
      rd[i].push_back(nd.in);
      if (nd.res) rd[i].push_back(nd.res);
      if (nd.kind == N_CONVBN)
        for (const MDest& d : nd.dests) writers[d.a].push_back(i);
      else
        writers[nd.out].push_back(i);
    }
    std::vector<std::vector<int>> dep(n), succ(n);
    for (int i = 0; i < n; i++) {
      for (const MAct* a : rd[i]) {
        auto it = writers.find(a);
        if (it == writers.end()) continue;
        for (int w : it->second)
          if (w < i) dep[i].push_back(w);
      }
      std::sort(dep[i].begin(), dep[i].end());
      dep[i].erase(std::unique(dep[i].begin(), dep[i].end()), dep[i].end());
      for (int w : dep[i]) succ[w].push_back(i);
    }
    std::vector<double> bottom(n, 0.0);  // FLOPs of the longest chain from a node to the end
    for (int i = n - 1; i >= 0; i--) {
      const MNode& nd = *nodes[i];
      double c = 1.0;
      if (nd.kind != N_POOL)
        c = 2.0 * (double)nd.plan.M * nd.plan.gemm_n * nd.plan.g.R * nd.plan.g.S * nd.plan.g.C;
      double m = 0.0;
      for (int sx : succ[i]) m = std::max(m, bottom[sx]);
      bottom[i] = c + m;
    }
    node_order.clear();
    std::vector<int> pending(n);
    std::vector<char> ready(n, 0);
    for (int i = 0; i < n; i++) {
      pending[i] = (int)dep[i].size();
      ready[i] = pending[i] == 0;
    }
    for (int step = 0; step < n; step++) {
      int pick = -1;
      for (int i = 0; i < n; i++)
        if (ready[i] == 1 && (pick < 0 || bottom[i] > bottom[pick])) pick = i;
      ready[pick] = 2;
      node_order.push_back(pick);
      for (int sx : succ[pick])
        if (--pending[sx] == 0) ready[sx] = 1;
    }
    node_stream.assign(n, 0);
    node_waits.assign(n, {});
    std::vector<char> signal(n, 0);
    int tail[kFwdStreams];
    for (int k = 0; k < kFwdStreams; k++) tail[k] = -1;
    std::vector<int> pos(n);
    for (int q = 0; q < n; q++) pos[node_order[q]] = q;
    for (int q = 0; q < n; q++) {
      const int i = node_order[q];
      const std::vector<int>& deps = dep[i];  // launched earlier, all of them
      int st = -1;
      int best = -1;  // the latest-launched producer that is still the tail of its stream
      for (int w : deps)
        if (tail[node_stream[w]] == pos[w] && (best < 0 || pos[w] > pos[best])) best = w;
      if (best >= 0) st = node_stream[best];
      if (st < 0) {
        st = 0;
        for (int k = 1; k < kFwdStreams; k++)
          if (tail[k] < tail[st]) st = k;
      }
      node_stream[i] = st;
      int latest[kFwdStreams];  // per other stream, the producer launched last there
      for (int k = 0; k < kFwdStreams; k++) latest[k] = -1;
      for (int w : deps) {
        const int ks = node_stream[w];
        if (ks != st && (latest[ks] < 0 || pos[w] > pos[latest[ks]])) latest[ks] = w;
      }
      for (int k = 0; k < kFwdStreams; k++)
        if (latest[k] >= 0) {
          node_waits[i].push_back(latest[k]);
          signal[latest[k]] = 1;
        }
      tail[st] = q;
    }
    cudaError_t e;
    node_ev.assign(n, nullptr);
    for (int i = 0; i < n; i++)
      if (signal[i] && (e = cudaEventCreateWithFlags(&node_ev[i], cudaEventDisableTiming)) != cudaSuccess) return e;
    for (int k = 0; k < kFwdStreams - 1; k++) {
      if ((e = cudaStreamCreateWithFlags(&fwd_st[k], cudaStreamNonBlocking)) != cudaSuccess) return e;
      if ((e = cudaEventCreateWithFlags(&ev_fwd_end[k], cudaEventDisableTiming)) != cudaSuccess) return e;
    }
    return cudaEventCreateWithFlags(&ev_fwd_start, cudaEventDisableTiming);
  }

  cudaError_t run(cudaStream_t st) {
    cudaError_t e = plan_streams();
    if (e != cudaSuccess) return e;
    cudaStream_t ss[kFwdStreams] = {st};
    for (int k = 1; k < kFwdStreams; k++) ss[k] = fwd_st[k - 1];
    // fork: the internal streams start after the caller's stream has reached this point
    if ((e = cudaEventRecord(ev_fwd_start, st)) != cudaSuccess) return e;
    for (int k = 1; k < kFwdStreams; k++)
      if ((e = cudaStreamWaitEvent(ss[k], ev_fwd_start, 0)) != cudaSuccess) return e;
    for (int i : node_order) {
      MNode& nd = *nodes[i];
      cudaStream_t s = ss[node_stream[i]];
      for (int w : node_waits[i])
        if ((e = cudaStreamWaitEvent(s, node_ev[w], 0)) != cudaSuccess) return e;
      e = nd.kind == N_POOL ? launch_sppf(nd.cat->p, N, nd.cat->H, nd.cat->W, nd.pc, s) : conv_launch(nd.L, s);
      if (e != cudaSuccess) return e;
      if (node_ev[i] && (e = cudaEventRecord(node_ev[i], s)) != cudaSuccess) return e;
    }
    // join: the caller's stream continues after every node
    for (int k = 1; k < kFwdStreams; k++) {
      if ((e = cudaEventRecord(ev_fwd_end[k - 1], ss[k])) != cudaSuccess) return e;
      if ((e = cudaStreamWaitEvent(st, ev_fwd_end[k - 1], 0)) != cudaSuccess) return e;
    }
    return cudaSuccess;
  }

  // ------------------------------------------------------------------ training (reference Model::forward(true)
  // and Model::backward, src/model.cpp:383-470): conv → z, batch statistics, apply; then in reverse order BN
  // backward, weight gradient, input gradient (accumulating where an activation has several consumers).
  int train_init(cudaStream_t st) {
    if (!synced) return model_fail(OSAM_ERR_INVALID, "train_init before osam_model_sync_weights");
    if (train) return OSAM_OK;
    cudaError_t e;
    // activation gradients (all but the input image)
    size_t goff = 0;
    std::vector<std::pair<MAct*, size_t>> gat;
    for (auto& kv : acts) {
      MAct* a = kv.second.get();
      if (a == in) continue;
      gat.push_back({a, goff});
      goff = align_up(goff + (size_t)N * a->H * a->W * a->C * sizeof(__half), 1024);
    }
    if ((e = cudaMalloc(&garena, goff)) != cudaSuccess) return model_fail(OSAM_ERR_NOMEM, "gradient arena");
    cudaMemsetAsync(garena, 0, goff, st);
    for (auto& ga : gat) ga.first->g = reinterpret_cast<__half*>(garena + ga.second);
    // z buffers, BN state, parameter gradients (reverse node order), scratch sizes
    size_t zn = 0, tn = 0, dzn = 0, gwn = 0, wsb = 256, bnb = 256;
    for (auto& nd : nodes)
      if (nd->kind == N_CONVBN) {
        const size_t n = (size_t)N * nd->plan.P * nd->plan.Q * nd->K;
        nd->t_off = tn;
        tn = align_up(tn + 8 * (size_t)nd->K, 32);
        dzn = std::max(dzn, n);
        zn = align_up(zn + n, 512);
      }
    size_t gn = 0;
    for (int i = (int)nodes.size() - 1; i >= 0; i--) {
      MNode& nd = *nodes[i];
      if (nd.kind == N_POOL) continue;
      const int C = nd.in->C;
      nd.g_w = nd.kind == N_CONVT ? (size_t)C * 4 * nd.K : (size_t)nd.K * nd.k * nd.k * C;
      nd.g_off = gn;
      gn = align_up(gn + nd.g_w + (nd.kind == N_CONVBN ? 2 * (size_t)nd.K : (size_t)nd.K), 64);
      gwn = std::max(gwn, nd.g_w);
      wsb = std::max(wsb, osam_conv_workspace_size(&nd.plan));
      bnb = std::max(bnb, std::max(osam_bn_workspace_size(nd.K), osam_chan_sum_workspace_size(nd.K)));
    }
    grad32_n = gn;
    if ((e = cudaMalloc(&zarena, std::max<size_t>(zn, 1) * sizeof(__half))) != cudaSuccess ||
        (e = cudaMalloc(&tarena, std::max<size_t>(tn, 1) * sizeof(float))) != cudaSuccess ||
        (e = cudaMalloc(&grad32, std::max<size_t>(gn, 1) * sizeof(float))) != cudaSuccess ||
        (e = cudaMalloc(&dz, std::max<size_t>(dzn, 1) * sizeof(__half))) != cudaSuccess ||
        (e = cudaMalloc(&gw16, std::max<size_t>(gwn, 1) * sizeof(__half))) != cudaSuccess ||
        (e = cudaMalloc(&ws, wsb)) != cudaSuccess || (e = cudaMalloc(&bnws, bnb)) != cudaSuccess ||
        (e = cudaMalloc(&dz2, std::max<size_t>(dzn, 1) * sizeof(__half))) != cudaSuccess ||
        (e = cudaMalloc(&ws_side, wsb)) != cudaSuccess)
      return model_fail(OSAM_ERR_NOMEM, "training buffers: %s", cudaGetErrorString(e));
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    if ((e = cudaStreamCreateWithPriority(&side, cudaStreamNonBlocking, lo)) != cudaSuccess)
      return model_fail(OSAM_ERR_CUDA, "side stream: %s", cudaGetErrorString(e));
    for (int i = 0; i < 2; i++) {
      cudaEventCreateWithFlags(&ev_dz[i], cudaEventDisableTiming);
      cudaEventCreateWithFlags(&ev_wg[i], cudaEventDisableTiming);
    }
    cudaEventCreateWithFlags(&ev_fork, cudaEventDisableTiming);
    cudaEventCreateWithFlags(&ev_join, cudaEventDisableTiming);
    {
      size_t pb = 0;
      std::vector<size_t> poff(nodes.size(), 0);
      for (size_t i = 0; i < nodes.size(); i++) {
        MNode& nd = *nodes[i];
        if (nd.kind == N_POOL || nd.kind == N_CONVT) continue;
        const size_t b = dgrad_prelaid_bytes(&nd.plan);
        poff[i] = pb;
        pb += b;
      }
      if (pb && (e = cudaMalloc(&prelaid, pb)) != cudaSuccess)
        return model_fail(OSAM_ERR_NOMEM, "dgrad weights: %s", cudaGetErrorString(e));
      std::vector<DgradJob> jh;
      for (size_t i = 0; i < nodes.size(); i++) {
        MNode& nd = *nodes[i];
        if (nd.kind == N_POOL || nd.kind == N_CONVT || !dgrad_prelaid_bytes(&nd.plan)) continue;
        nd.pre_w = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(prelaid) + poff[i]);
        DgradJob j[4];
        const int nj = dgrad_jobs(&nd.plan, w16 + nd.w_off, nd.pre_w, j);
        for (int q = 0; q < nj; q++) jh.push_back(j[q]);
      }
      njobs = (int)jh.size();
      if (njobs) {
        if ((e = cudaMalloc(&jobs, jh.size() * sizeof(DgradJob))) != cudaSuccess)
          return model_fail(OSAM_ERR_NOMEM, "dgrad jobs");
        cudaMemcpy(jobs, jh.data(), jh.size() * sizeof(DgradJob), cudaMemcpyHostToDevice);
      }
    }
    ws_bytes = wsb;
    bnws_bytes = bnb;
    cudaMemsetAsync(bnws, 0, bnb, st);
    cudaMemsetAsync(grad32, 0, std::max<size_t>(gn, 1) * sizeof(float), st);
    size_t zo = 0;
    std::vector<float> th(std::max<size_t>(tn, 1), 0.f);
    for (auto& ndp : nodes) {
      MNode& nd = *ndp;
      if (nd.kind != N_CONVBN) continue;
      nd.z = zarena + zo;
      zo = align_up(zo + (size_t)N * nd.plan.P * nd.plan.Q * nd.K, 512);
      int k0 = 0;
      const char* bnn[4] = {".bn.weight", ".bn.bias", ".bn.running_mean", ".bn.running_var"};
      for (size_t pi = 0; pi < nd.pre.size(); pi++) {
        for (int q = 0; q < 4; q++) {
          const PInfo& B = params[nd.pre[pi] + bnn[q]];
          for (int kk = 0; kk < nd.ks[pi]; kk++) th[nd.t_off + (size_t)q * nd.K + k0 + kk] = B.host[kk];
        }
        k0 += nd.ks[pi];
      }
    }
    cudaMemcpyAsync(tarena, th.data(), th.size() * sizeof(float), cudaMemcpyHostToDevice, st);
    // the transposed conv's weights in the reference's (C_in, R, S, C_out) layout for its gradients
    for (auto& ndp : nodes)
      if (ndp->kind == N_CONVT) {
        MNode& nd = *ndp;
        const int C = nd.in->C;
        std::vector<__half> h((size_t)C * 4 * nd.K);
        const PInfo& W = params[nd.name + ".weight"];  // PyTorch (C_in, C_out, 2, 2)
        for (int c = 0; c < C; c++)
          for (int dy = 0; dy < 2; dy++)
            for (int dx = 0; dx < 2; dx++)
              for (int kk = 0; kk < nd.K; kk++)
                h[(((size_t)c * 2 + dy) * 2 + dx) * nd.K + kk] =
                    __float2half_rn(W.host[(((size_t)c * nd.K + kk) * 2 + dy) * 2 + dx]);
        if ((e = cudaMalloc(&wconvt, h.size() * sizeof(__half))) != cudaSuccess)
          return model_fail(OSAM_ERR_NOMEM, "transposed-conv weights");
        cudaMemcpy(wconvt, h.data(), h.size() * sizeof(__half), cudaMemcpyHostToDevice);
      }
    // which gradient writes overwrite and which accumulate (reference src/model.cpp:352-366)
    std::map<const MAct*, bool> written;
    for (int l = 0; l < 3; l++)
      for (int k = 0; k < 3; k++) written[head[k][l]] = true;
    written[proto] = true;
    for (int i = (int)nodes.size() - 1; i >= 0; i--) {
      MNode& nd = *nodes[i];
      if (nd.kind == N_POOL) continue;
      if (nd.kind == N_CONVBN) {
        for (auto& d : nd.dests)
          if (!written.count(d.a)) return model_fail(OSAM_ERR_INVALID, "%s: gradient of %s not ready", nd.name.c_str(),
                                                     d.a->name.c_str());
        if (nd.res) {
          nd.res_accum = written.count(nd.res) > 0;
          written[nd.res] = true;
        }
      } else if (!written.count(nd.out)) {
        return model_fail(OSAM_ERR_INVALID, "%s: output gradient not ready", nd.name.c_str());
      }
      if (nd.in != in) {
        nd.dgrad_accum = written.count(nd.in) > 0;
        written[nd.in] = true;
      }
    }
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return model_fail(OSAM_ERR_CUDA, "train_init: %s", cudaGetErrorString(e));
    train = true;
    return OSAM_OK;
  }

  int forward_train(float momentum, cudaStream_t st) {
    if (!train) return model_fail(OSAM_ERR_INVALID, "forward_train before osam_model_train_init");
    for (auto& ndp : nodes) {
      MNode& nd = *ndp;
      int rc = OSAM_OK;
      if (nd.kind == N_CONVBN) {
        const int P = nd.plan.P, Q = nd.plan.Q, K = nd.K;
        float* T = tarena + nd.t_off;
        rc = osam_conv_fwd(&nd.plan, nd.in->p, w16 + nd.w_off, nd.z, 0.f, ws, ws_bytes, st);
        if (!rc)
          rc = osam_bn_forward_stats(nd.z, N, P, Q, K, T, T + K, T + 2 * K, T + 3 * K, momentum, bn_eps, T + 4 * K,
                                     T + 5 * K, T + 6 * K, T + 7 * K, bnws, bnws_bytes, st);
        osam_dest d[OSAM_MAX_DEST];
        for (size_t i = 0; i < nd.dests.size(); i++)
          d[i] = osam_dest{nd.dests[i].a->p, nd.dests[i].a->C, nd.dests[i].choff, nd.dests[i].c0, nd.dests[i].c1,
                           nd.dests[i].up};
        if (!rc)
          rc = osam_bn_forward_apply(nd.z, N, P, Q, K, T + 6 * K, T + 7 * K, nd.res ? nd.res->p : nullptr, d,
                                     (int)nd.dests.size(), 1, st);
      } else if (nd.kind == N_POOL) {
        if (launch_sppf(nd.cat->p, N, nd.cat->H, nd.cat->W, nd.pc, st) != cudaSuccess) rc = OSAM_ERR_CUDA;
      } else {
        if (conv_launch(nd.L, st) != cudaSuccess) rc = OSAM_ERR_CUDA;
      }
      if (rc) return model_fail(rc, "%s (train forward): %s", nd.name.c_str(), osam_last_error());
    }
    // this step's weights, re-laid out once for every input-gradient conv of the coming backward
    if (launch_dgrad_weights_batched(jobs, njobs, st) != cudaSuccess)
      return model_fail(OSAM_ERR_CUDA, "dgrad weight re-layout");
    return OSAM_OK;
  }

  int backward_nodes(int first, int count, cudaStream_t st) {
    if (!train) return model_fail(OSAM_ERR_INVALID, "backward before osam_model_train_init");
    // the weight gradients of the range are accumulated straight into the arena: zero it first
    {
      size_t lo = grad32_n, hi = 0;
      for (int i = first; i < first + count; i++) {
        const MNode& nd = *nodes[i];
        if (nd.kind == N_POOL) continue;
        lo = std::min(lo, nd.g_off);
        hi = std::max(hi, nd.g_off + nd.g_w);
      }
      if (hi > lo) cudaMemsetAsync(grad32 + lo, 0, (hi - lo) * sizeof(float), st);
    }
    // the side stream starts after everything issued so far on the caller's stream
    cudaEventRecord(ev_fork, st);
    cudaStreamWaitEvent(side, ev_fork, 0);
    bool busy[2] = {false, false};
    int buf = 0;
    for (int i = first + count - 1; i >= first; i--) {
      MNode& nd = *nodes[i];
      int rc = OSAM_OK;
      if (nd.kind == N_CONVBN) {
        const int P = nd.plan.P, Q = nd.plan.Q, K = nd.K;
        float* T = tarena + nd.t_off;
        __half* d = buf ? dz2 : dz;
        if (busy[buf]) cudaStreamWaitEvent(st, ev_wg[buf], 0);  // its last weight gradient has read it
        osam_dest gd[OSAM_MAX_DEST];
        for (size_t k = 0; k < nd.dests.size(); k++)
          gd[k] = osam_dest{nd.dests[k].a->g, nd.dests[k].a->C, nd.dests[k].choff, nd.dests[k].c0, nd.dests[k].c1,
                            nd.dests[k].up};
        float* gg = grad32 + nd.g_off + nd.g_w;
        rc = osam_bn_backward(nd.z, N, P, Q, K, T + 4 * K, T + 5 * K, T + 6 * K, T + 7 * K, gd, (int)nd.dests.size(), 1,
                              d, gg, gg + K, 0, nd.res ? nd.res->g : nullptr, nd.res_accum ? 1 : 0, bnws, bnws_bytes,
                              st);
        if (!rc) {
          cudaEventRecord(ev_dz[buf], st);
          cudaStreamWaitEvent(side, ev_dz[buf], 0);
          rc = conv_wgrad_f32(&nd.plan, nd.in->p, d, grad32 + nd.g_off, 0.f, ws_side, ws_bytes, side, true);
          cudaEventRecord(ev_wg[buf], side);
          busy[buf] = true;
        }
        if (!rc && nd.in != in)
          rc = conv_dgrad_ex(&nd.plan, d, w16 + nd.w_off, nd.in->g, nd.dgrad_accum ? 1.f : 0.f, ws, ws_bytes, st,
                             nd.pre_w);
        buf ^= 1;
      } else if (nd.kind == N_POOL) {
        rc = osam_sppf_bwd(nd.cat->p, nd.cat->g, N, nd.cat->H, nd.cat->W, nd.pc, st);
      } else {
        // the head gradients are set by the caller before the backward and never change during it
        const long long M = (long long)N * nd.out->H * nd.out->W;
        cudaEventRecord(ev_fork, st);
        cudaStreamWaitEvent(side, ev_fork, 0);
        rc = conv_wgrad_f32(&nd.plan, nd.in->p, nd.out->g, grad32 + nd.g_off, 0.f, ws_side, ws_bytes, side, true);
        if (!rc) rc = osam_chan_sum(nd.out->g, M, nd.K, grad32 + nd.g_off + nd.g_w, 0, bnws, bnws_bytes, st);
        const __half* w = nd.kind == N_CONVT ? wconvt : w16 + nd.w_off;
        if (!rc && nd.in != in)
          rc = conv_dgrad_ex(&nd.plan, nd.out->g, w, nd.in->g, nd.dgrad_accum ? 1.f : 0.f, ws, ws_bytes, st, nd.pre_w);
      }
      if (rc) {
        cudaEventRecord(ev_join, side);
        cudaStreamWaitEvent(st, ev_join, 0);
        return model_fail(rc, "%s (backward): %s", nd.name.c_str(), osam_last_error());
      }
    }
    // every weight gradient of the range is complete when the caller's stream passes this point
    cudaEventRecord(ev_join, side);
    cudaStreamWaitEvent(st, ev_join, 0);
    return OSAM_OK;
  }

  // Gradient of one parameter in its PyTorch name and layout (host fp32), read back after a backward.
  int get_grad(const std::string& name, float* out, size_t n) {
    if (!train) return model_fail(OSAM_ERR_INVALID, "no gradients before osam_model_train_init");
    auto it = params.find(name);
    if (it == params.end()) return model_fail(OSAM_ERR_INVALID, "no parameter %s", name.c_str());
    size_t cnt = 1;
    for (auto v : it->second.shape) cnt *= (size_t)v;
    if (n < cnt) return model_fail(OSAM_ERR_INVALID, "%s: %zu values needed", name.c_str(), cnt);
    for (auto& ndp : nodes) {
      MNode& nd = *ndp;
      if (nd.kind == N_POOL) continue;
      const int C = nd.in->C, k = nd.k;
      std::vector<float> g(nd.g_w + (nd.kind == N_CONVBN ? 2 * (size_t)nd.K : (size_t)nd.K));
      auto fetch = [&]() {
        cudaMemcpy(g.data(), grad32 + nd.g_off, g.size() * sizeof(float), cudaMemcpyDeviceToHost);
      };
      if (nd.kind == N_CONVBN) {
        int k0 = 0;
        for (size_t pi = 0; pi < nd.pre.size(); pi++) {
          const std::string& pf = nd.pre[pi];
          const int Kp = nd.ks[pi];
          if (name == pf + ".conv.weight") {
            fetch();
            for (int kk = 0; kk < Kp; kk++)
              for (int c = 0; c < C; c++)
                for (int r = 0; r < k; r++)
                  for (int s2 = 0; s2 < k; s2++)
                    out[(((size_t)kk * C + c) * k + r) * k + s2] = g[(((size_t)(k0 + kk) * k + r) * k + s2) * C + c];
            return OSAM_OK;
          }
          if (name == pf + ".bn.weight" || name == pf + ".bn.bias") {
            fetch();
            const size_t base = nd.g_w + (name == pf + ".bn.bias" ? (size_t)nd.K : 0);
            for (int kk = 0; kk < Kp; kk++) out[kk] = g[base + k0 + kk];
            return OSAM_OK;
          }
          k0 += Kp;
        }
      } else if (name == nd.name + ".weight") {
        fetch();
        if (nd.kind == N_HEAD) {
          for (size_t q = 0; q < nd.g_w; q++) out[q] = g[q];  // (K, 1, 1, C) = (K, C, 1, 1)
        } else {  // (C_in, 2, 2, C_out) → PyTorch (C_in, C_out, 2, 2)
          for (int c = 0; c < C; c++)
            for (int dy = 0; dy < 2; dy++)
              for (int dx = 0; dx < 2; dx++)
                for (int kk = 0; kk < nd.K; kk++)
                  out[(((size_t)c * nd.K + kk) * 2 + dy) * 2 + dx] = g[(((size_t)c * 2 + dy) * 2 + dx) * nd.K + kk];
        }
        return OSAM_OK;
      } else if (name == nd.name + ".bias") {
        fetch();
        for (int kk = 0; kk < nd.K; kk++) out[kk] = g[nd.g_w + kk];
        return OSAM_OK;
      }
    }
    return model_fail(OSAM_ERR_INVALID, "%s has no gradient (running statistics are not trained)", name.c_str());
  }

  int forward(int use_graph, cudaStream_t st) {
    if (!synced) return model_fail(OSAM_ERR_INVALID, "forward before osam_model_sync_weights");
    cudaError_t e;
    if (!use_graph) {
      e = run(st);
      return e == cudaSuccess ? OSAM_OK : model_fail(OSAM_ERR_CUDA, "forward: %s", cudaGetErrorString(e));
    }
    if ((e = plan_streams()) != cudaSuccess)  // streams and events exist before any capture begins
      return model_fail(OSAM_ERR_CUDA, "forward streams: %s", cudaGetErrorString(e));
    if (!exec) {
      // Record on the model's own stream; recording does not execute, so no ordering with `st` is needed.
      if (!cap && (e = cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking)) != cudaSuccess)
        return model_fail(OSAM_ERR_CUDA, "capture stream: %s", cudaGetErrorString(e));
      if ((e = cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal)) != cudaSuccess)
        return model_fail(OSAM_ERR_CUDA, "begin capture: %s", cudaGetErrorString(e));
      cudaError_t er = run(cap);
      e = cudaStreamEndCapture(cap, &graph);
      if (er != cudaSuccess || e != cudaSuccess)
        return model_fail(OSAM_ERR_CUDA, "capture: %s", cudaGetErrorString(er != cudaSuccess ? er : e));
      if ((e = cudaGraphInstantiate(&exec, graph, 0)) != cudaSuccess)
        return model_fail(OSAM_ERR_CUDA, "instantiate: %s", cudaGetErrorString(e));
    }
    e = cudaGraphLaunch(exec, st);
    return e == cudaSuccess ? OSAM_OK : model_fail(OSAM_ERR_CUDA, "graph launch: %s", cudaGetErrorString(e));
  }
};

namespace osam {
int model_fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  char buf[512];
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_last_error("%s", buf);
  return code;
}
}  // namespace osam

namespace {
int fill_tensor(const osam_model* m, const MAct* a, osam_tensor* t) {
  if (!a || !t) return model_fail(OSAM_ERR_INVALID, "no such tensor");
  t->p = a->p;
  t->n = m->N;
  t->h = a->H;
  t->w = a->W;
  t->c = a->C;
  return OSAM_OK;
}
}  // namespace

extern "C" {

int osam_model_create(int batch, int imgsz, int reg_max, osam_model** out) {
  if (!out || batch < 1 || imgsz < 32 || imgsz % 32 || reg_max < 1 || reg_max > 64)
    return model_fail(OSAM_ERR_INVALID, "osam_model_create(batch=%d, imgsz=%d, reg_max=%d)", batch, imgsz, reg_max);
  *out = nullptr;
  auto m = std::make_unique<osam_model>();
  m->N = batch;
  m->S = imgsz;
  m->reg_max = reg_max;
  m->build();
  int rc = m->allocate();
  if (rc) {
    m->release();
    return rc;
  }
  if (!device_error_word()) {
    m->release();
    return model_fail(OSAM_ERR_CUDA, "device error word");
  }
  *out = m.release();
  return OSAM_OK;
}

int osam_model_destroy(osam_model* m) {
  if (m) {
    m->release();
    delete m;
  }
  return OSAM_OK;
}

int osam_model_set_param(osam_model* m, const char* name, const float* data, const int64_t* shape, int ndim) {
  if (!m || !name || !data || (ndim && !shape)) return model_fail(OSAM_ERR_INVALID, "NULL argument");
  auto it = m->params.find(name);
  if (it == m->params.end()) return OSAM_OK;  // not a parameter of this graph (e.g. the DFL conv)
  PInfo& p = it->second;
  if ((int)p.shape.size() != ndim) return model_fail(OSAM_ERR_INVALID, "%s: rank %d, expected %zu", name, ndim, p.shape.size());
  size_t n = 1;
  for (int i = 0; i < ndim; i++) {
    if (shape[i] != p.shape[i]) return model_fail(OSAM_ERR_INVALID, "%s: shape mismatch at dim %d", name, i);
    n *= (size_t)shape[i];
  }
  p.host.assign(data, data + n);
  p.set = true;
  m->synced = false;
  return OSAM_OK;
}

int osam_model_load_fsow(osam_model* m, const char* path) {
  if (!m || !path) return model_fail(OSAM_ERR_INVALID, "NULL argument");
  std::ifstream f(path, std::ios::binary);
  if (!f.good()) return model_fail(OSAM_ERR_INVALID, "cannot open %s", path);
  char magic[8];
  f.read(magic, 8);
  if (!f.good() || std::memcmp(magic, "FSOW0001", 8)) return model_fail(OSAM_ERR_INVALID, "%s: not an FSOW file", path);
  uint32_t n = 0;
  f.read(reinterpret_cast<char*>(&n), 4);
  static const int isz[3] = {4, 4, 1};
  for (uint32_t i = 0; i < n && f.good(); i++) {
    uint16_t ln = 0;
    f.read(reinterpret_cast<char*>(&ln), 2);
    std::string name(ln, '\0');
    f.read(&name[0], ln);
    uint8_t nd = 0;
    f.read(reinterpret_cast<char*>(&nd), 1);
    std::vector<int64_t> shape(nd);
    f.read(reinterpret_cast<char*>(shape.data()), 8 * nd);
    uint8_t dt = 0;
    f.read(reinterpret_cast<char*>(&dt), 1);
    if (dt > 2) return model_fail(OSAM_ERR_INVALID, "%s: bad dtype", path);
    size_t cnt = 1;
    for (auto s : shape) cnt *= (size_t)s;
    std::vector<char> buf(cnt * isz[dt]);
    f.read(buf.data(), buf.size());
    if (!f.good()) return model_fail(OSAM_ERR_INVALID, "%s: truncated", path);
    if (dt != 0) continue;
    int rc = osam_model_set_param(m, name.c_str(), reinterpret_cast<const float*>(buf.data()), shape.data(), nd);
    if (rc) return rc;
  }
  return OSAM_OK;
}

int osam_model_sync_weights(osam_model* m, osam_stream_t stream) {
  if (!m) return model_fail(OSAM_ERR_INVALID, "NULL model");
  return m->sync(reinterpret_cast<cudaStream_t>(stream));
}

int osam_model_input(const osam_model* m, osam_tensor* t) { return m ? fill_tensor(m, m->in, t) : OSAM_ERR_INVALID; }

int osam_model_head(const osam_model* m, int kind, int level, osam_tensor* t) {
  if (!m || kind < 0 || kind > 2 || level < 0 || level > 2) return model_fail(OSAM_ERR_INVALID, "head(%d,%d)", kind, level);
  return fill_tensor(m, m->head[kind][level], t);
}

int osam_model_proto(const osam_model* m, osam_tensor* t) { return m ? fill_tensor(m, m->proto, t) : OSAM_ERR_INVALID; }

int osam_model_act(const osam_model* m, const char* name, osam_tensor* t) {
  if (!m || !name) return model_fail(OSAM_ERR_INVALID, "NULL argument");
  auto it = m->acts.find(name);
  if (it == m->acts.end()) return model_fail(OSAM_ERR_INVALID, "no activation %s", name);
  return fill_tensor(m, it->second.get(), t);
}

int osam_model_forward(osam_model* m, int use_graph, osam_stream_t stream) {
  if (!m) return model_fail(OSAM_ERR_INVALID, "NULL model");
  return m->forward(use_graph, reinterpret_cast<cudaStream_t>(stream));
}

int osam_model_num_launches(const osam_model* m) { return m ? (int)m->nodes.size() : 0; }

int osam_model_forward_nodes(osam_model* m, int first, int count, osam_stream_t stream) {
  if (!m || first < 0 || count < 0 || first + count > (int)m->nodes.size())
    return model_fail(OSAM_ERR_INVALID, "forward_nodes range");
  if (!m->synced) return model_fail(OSAM_ERR_INVALID, "forward before osam_model_sync_weights");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  for (int i = first; i < first + count; i++) {
    MNode& nd = *m->nodes[i];
    cudaError_t e = nd.kind == N_POOL ? launch_sppf(nd.cat->p, m->N, nd.cat->H, nd.cat->W, nd.pc, st)
                                      : conv_launch(nd.L, st);
    if (e != cudaSuccess) return model_fail(OSAM_ERR_CUDA, "%s: %s", nd.name.c_str(), cudaGetErrorString(e));
  }
  return OSAM_OK;
}

int osam_model_train_init(osam_model* m, osam_stream_t stream) {
  if (!m) return model_fail(OSAM_ERR_INVALID, "NULL model");
  return m->train_init(reinterpret_cast<cudaStream_t>(stream));
}

int osam_model_forward_train(osam_model* m, float momentum, osam_stream_t stream) {
  if (!m) return model_fail(OSAM_ERR_INVALID, "NULL model");
  return m->forward_train(momentum, reinterpret_cast<cudaStream_t>(stream));
}

int osam_model_backward_nodes(osam_model* m, int first, int count, osam_stream_t stream) {
  if (!m || first < 0 || count < 0 || first + count > (int)m->nodes.size())
    return model_fail(OSAM_ERR_INVALID, "backward_nodes range");
  return m->backward_nodes(first, count, reinterpret_cast<cudaStream_t>(stream));
}

int osam_model_act_grad(const osam_model* m, const char* name, osam_tensor* t) {
  if (!m || !name || !t) return model_fail(OSAM_ERR_INVALID, "NULL argument");
  if (!m->train) return model_fail(OSAM_ERR_INVALID, "no gradients before osam_model_train_init");
  auto it = m->acts.find(name);
  if (it == m->acts.end() || !it->second->g) return model_fail(OSAM_ERR_INVALID, "no gradient for %s", name);
  int rc = fill_tensor(m, it->second.get(), t);
  t->p = it->second->g;
  return rc;
}

int osam_model_grad_arena(const osam_model* m, float** p, int64_t* n) {
  if (!m || !p || !n) return model_fail(OSAM_ERR_INVALID, "NULL argument");
  if (!m->train) return model_fail(OSAM_ERR_INVALID, "no gradients before osam_model_train_init");
  *p = m->grad32;
  *n = (int64_t)m->grad32_n;
  return OSAM_OK;
}

int osam_model_node_grad_range(const osam_model* m, int i, int64_t* off, int64_t* n) {
  if (!m || i < 0 || i >= (int)m->nodes.size() || !off || !n) return model_fail(OSAM_ERR_INVALID, "node index %d", i);
  const MNode& nd = *m->nodes[i];
  *off = (int64_t)nd.g_off;
  *n = nd.kind == N_POOL ? 0 : (int64_t)(nd.g_w + (nd.kind == N_CONVBN ? 2 * (size_t)nd.K : (size_t)nd.K));
  return OSAM_OK;
}

int osam_model_get_grad(osam_model* m, const char* name, float* out, int64_t n) {
  if (!m || !name || !out || n < 0) return model_fail(OSAM_ERR_INVALID, "NULL argument");
  return m->get_grad(name, out, (size_t)n);
}

int osam_model_node_info(const osam_model* m, int i, char* name, int name_len, int* kind, osam_conv_geom* g) {
  if (!m || i < 0 || i >= (int)m->nodes.size()) return model_fail(OSAM_ERR_INVALID, "node index %d", i);
  const MNode& nd = *m->nodes[i];
  if (name && name_len > 0) {
    std::strncpy(name, nd.name.c_str(), name_len - 1);
    name[name_len - 1] = 0;
  }
  if (kind) *kind = (int)nd.kind;
  if (g) {
    if (nd.kind == N_POOL) *g = osam_conv_geom{m->N, nd.cat->H, nd.cat->W, nd.pc, nd.pc, 5, 5, 1, 2};
    else *g = nd.plan.g;
  }
  return OSAM_OK;
}

}  // extern "C"
