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
  cudaStream_t cap = nullptr;  // private stream the step graphs are recorded on (the legacy stream cannot capture)
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
  // gradient on the caller's stream (the reference's wgrad_side, src/model.cpp:416-428); kDzBufs dz buffers
  // rotate so a node's BN backward never overwrites the dz a pending weight gradient still reads, and the
  // caller's stream runs up to kDzBufs − 1 nodes ahead of the side stream
  static constexpr int kDzBufs = 4;
  __half* dzx[kDzBufs - 1] = {};  // buffers 1.. (buffer 0 is dz)
  void* ws_side = nullptr;
  // the input-gradient convs' re-laid-out weights, all nodes, refreshed by one batched launch per step
  __half* prelaid = nullptr;
  DgradJob* jobs = nullptr;
  int njobs = 0;
  cudaStream_t side = nullptr;
  cudaEvent_t ev_dz[kDzBufs] = {}, ev_wg[kDzBufs] = {}, ev_fork = nullptr, ev_join = nullptr;
  // forward on several streams: nodes that do not depend on each other (the neck's PAN path, the three
  // head levels and their branches, the proto chain) overlap, so small layers fill the SMs that a big one
  // leaves idle in its last wave.  Stream 0 is the caller's; the schedule is fixed at the first forward.
  static constexpr int kFwdStreams = 3;
  cudaStream_t fwd_st[kFwdStreams - 1] = {};
  cudaEvent_t ev_fwd_start = nullptr, ev_fwd_end[kFwdStreams - 1] = {};
  // A task of a scheduled step: a model node (its kernel) or a post-process launch of the detect step.
  enum TaskKind { T_NODE = 0, T_DECODE = 1, T_NMS = 2, T_MASK = 3 };
  struct Task {
    TaskKind kind;
    int node;  // T_NODE: index into nodes
    std::vector<const MAct*> reads, writes;
    double cost;  // FLOPs (the longest-remaining-chain priority)
  };
  struct Schedule {
    std::vector<Task> tasks;
    std::vector<int> order;               // launch order: topological, longest remaining path first
    std::vector<int> stream;              // per task: 0 … kFwdStreams − 1
    std::vector<std::vector<int>> waits;  // per task: producers on other streams (latest per stream)
    std::vector<cudaEvent_t> ev;          // per task: recorded after it when another stream waits on it
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
  };
  Schedule fwd_sched, det_sched;  // the forward; the forward with decode / NMS / masks

  // ---- the detect step (osam_model_detect_*): post-process outputs owned by the model
  bool det_on = false;
  float det_conf = 0.25f, det_iou = 0.7f;
  int det_max = 300, det_forced = 0, det_packed = 1;
  float* det_xyxy = nullptr;   // [N][A][4]
  float* det_confs = nullptr;  // [N][A]
  int* det_n = nullptr;        // [N]
  int* det_keep = nullptr;     // [N][max_det]
  float* det_box = nullptr;    // [N][max_det][4]
  float* det_score = nullptr;  // [N][max_det]
  __half* det_coef = nullptr;  // [N][ceil128(max_det)][32]
  void* det_masks = nullptr;   // [N][max_det][words or Hp·Wp]
  MAct det_decoded, det_kept, det_maskt;  // stand-ins for the DAG (read/written by the post-process tasks)

  // ------------------------------------------------------------------ graph construction
  // The network is data (kLayers below, one row per model.<i> module) lowered in two steps:
  //   1. expand(): each module becomes primitive tensors (Prim) — convs, channel slices, 2× upsamples,
  //      concats, the SPPF pool chain — with explicit producers;
  //   2. lower(): concats, slices and upsamples vanish.  A compute primitive's output is routed to every
  //      place that reads it: its own buffer only when some primitive reads it directly, and otherwise (or
  //      besides) the channel range of each concat that contains it, 2× upsampled on the way when an
  //      upsample sits in between — the epilogue's destination list (osam_dest).
  // Every compute primitive becomes one node (one kernel launch), in primitive order.

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

  enum PrimOp { P_INPUT, P_CONV, P_HEAD, P_CONVT, P_POOLCAT, P_SLICE, P_UP2, P_CAT };
  struct Prim {
    PrimOp op;
    std::string name;              // tensor name when it is given a buffer of its own
    std::vector<int> src;          // producers (P_CAT: in channel order)
    int C = 0, H = 0, W = 0;       // output shape
    int k = 1, s = 1, res = -1;    // P_CONV: kernel, stride, residual primitive (added after the SiLU)
    int c0 = 0;                    // P_SLICE: first channel taken from its producer
    std::string param;             // P_CONV / P_HEAD / P_CONVT: parameter prefix
    std::vector<std::string> branch;  // P_CONV: prefixes of convs fused along K (one per branch)
    std::vector<int> branch_k;
    bool output = false;           // a model output (head or proto): always has its own buffer
    MAct* buf = nullptr;
  };
  std::vector<Prim> prims;

  int prim(Prim p) {
    prims.push_back(std::move(p));
    return (int)prims.size() - 1;
  }
  int conv(const std::string& pre, int x, int K, int k, int s, int res = -1) {
    Prim p{P_CONV, pre, {x}};
    p.C = K;
    p.H = (prims[x].H + 2 * (k / 2) - k) / s + 1;
    p.W = (prims[x].W + 2 * (k / 2) - k) / s + 1;
    p.k = k;
    p.s = s;
    p.res = res;
    p.param = pre;
    return prim(p);
  }
  int slice(int x, int c0, int c1, const std::string& name) {
    Prim p{P_SLICE, name, {x}};
    p.C = c1 - c0;
    p.H = prims[x].H;
    p.W = prims[x].W;
    p.c0 = c0;
    return prim(p);
  }
  int concat(const std::vector<int>& xs, const std::string& name) {
    Prim p{P_CAT, name, xs};
    for (int x : xs) p.C += prims[x].C;
    p.H = prims[xs[0]].H;
    p.W = prims[xs[0]].W;
    return prim(p);
  }
  int up2(int x) {
    Prim p{P_UP2, prims[x].name + ".up", {x}};
    p.C = prims[x].C;
    p.H = 2 * prims[x].H;
    p.W = 2 * prims[x].W;
    return prim(p);
  }

  // YOLOv8-seg: the rows of Ultralytics' yolov8-seg model description at full width and depth; the "s"
  // variant scales channels by 0.5 (at most 1024 before scaling, multiples of 8) and repeats by 1/3.
  enum Mod { M_CONV, M_C2F, M_SPPF, M_UP, M_CAT, M_SEGMENT };
  struct Row {
    Mod m;
    int from[3];  // producer rows, -1 = the row before; unused entries 0
    int nfrom;
    int repeats, ch, k, s;
    bool shortcut;
  };
  static constexpr Row kLayers[23] = {
      {M_CONV, {-1}, 1, 1, 64, 3, 2, false},       // 0   P1/2
      {M_CONV, {-1}, 1, 1, 128, 3, 2, false},      // 1   P2/4
      {M_C2F, {-1}, 1, 3, 128, 0, 0, true},        // 2
      {M_CONV, {-1}, 1, 1, 256, 3, 2, false},      // 3   P3/8
      {M_C2F, {-1}, 1, 6, 256, 0, 0, true},        // 4
      {M_CONV, {-1}, 1, 1, 512, 3, 2, false},      // 5   P4/16
      {M_C2F, {-1}, 1, 6, 512, 0, 0, true},        // 6
      {M_CONV, {-1}, 1, 1, 1024, 3, 2, false},     // 7   P5/32
      {M_C2F, {-1}, 1, 3, 1024, 0, 0, true},       // 8
      {M_SPPF, {-1}, 1, 1, 1024, 5, 1, false},     // 9
      {M_UP, {-1}, 1, 1, 0, 0, 0, false},          // 10
      {M_CAT, {-1, 6}, 2, 1, 0, 0, 0, false},      // 11
      {M_C2F, {-1}, 1, 3, 512, 0, 0, false},       // 12
      {M_UP, {-1}, 1, 1, 0, 0, 0, false},          // 13
      {M_CAT, {-1, 4}, 2, 1, 0, 0, 0, false},      // 14
      {M_C2F, {-1}, 1, 3, 256, 0, 0, false},       // 15  P3 out
      {M_CONV, {-1}, 1, 1, 256, 3, 2, false},      // 16
      {M_CAT, {-1, 12}, 2, 1, 0, 0, 0, false},     // 17
      {M_C2F, {-1}, 1, 3, 512, 0, 0, false},       // 18  P4 out
      {M_CONV, {-1}, 1, 1, 512, 3, 2, false},      // 19
      {M_CAT, {-1, 9}, 2, 1, 0, 0, 0, false},      // 20
      {M_C2F, {-1}, 1, 3, 1024, 0, 0, false},      // 21  P5 out
      {M_SEGMENT, {15, 18, 21}, 3, 1, 256, 0, 0, false},  // 22  Segment(nc = 1, nm = 32, npr = 256)
  };
  static int width(int c) { return (std::min(c, 1024) / 2 + 7) / 8 * 8; }
  static int depth(int n) { return std::max((int)std::lround(n * 0.33), 1); }

  // C2f: cv1 (1×1, 2c) split in halves; n bottlenecks (3×3, 3×3, + input if shortcut) chained from the
  // second half; cv2 (1×1) over the concat of both halves and every bottleneck output.
  int expand_c2f(const std::string& pre, const std::string& tn, int x, int c2, int n, bool shortcut) {
    const int c = c2 / 2;
    const int y = conv(pre + ".cv1", x, 2 * c, 1, 1);
    std::vector<int> parts = {y};
    int b = slice(y, c, 2 * c, tn + ".b0");
    for (int j = 0; j < n; j++) {
      const std::string mj = pre + ".m." + std::to_string(j);
      const int t = conv(mj + ".cv1", b, c, 3, 1);
      prims[t].name = tn + ".t" + std::to_string(j);
      b = conv(mj + ".cv2", t, c, 3, 1, shortcut ? b : -1);
      prims[b].name = tn + ".b" + std::to_string(j + 1);
      parts.push_back(b);
    }
    return conv(pre + ".cv2", concat(parts, tn + ".cat"), c2, 1, 1);
  }
  // SPPF: cv1 (1×1, c/2) → three chained 5×5 max-pools, concatenated with cv1's output → cv2 (1×1).  The
  // pool chain is one kernel that reads channels [0, c/2) of the concat and writes the other three slices.
  int expand_sppf(const std::string& pre, const std::string& tn, int x, int c2) {
    const int ch = prims[x].C / 2;
    const int a = conv(pre + ".cv1", x, ch, 1, 1);
    Prim p{P_POOLCAT, tn + ".cat", {a}};
    p.C = 4 * ch;
    p.H = prims[a].H;
    p.W = prims[a].W;
    p.param = pre + ".m";
    return conv(pre + ".cv2", prim(p), c2, 1, 1);
  }
  // Segment head: per level three branches (box 4·reg_max, class nc, mask coefficients nm), each
  // Conv3×3 → Conv3×3 → Conv2d 1×1 + bias; the three branch stems read the same input with the same
  // geometry, so they run as ONE conv whose output channels are the branches side by side.  Proto:
  // Conv3×3 → ConvTranspose 2×2/s2 + bias → Conv3×3 → Conv1×1 (nm channels) on P3.
  void expand_segment(const std::string& pre, const int lv[3], int npr) {
    const int nm = 32, ch0 = prims[lv[0]].C;
    // Ultralytics' branch widths: box max(16, ch0/4, 4·reg_max), class max(ch0, min(nc, 100)) with nc = 1,
    // mask coefficients max(ch0/4, nm)
    const int cb = std::max({16, ch0 / 4, 4 * reg_max}), cc = std::max(ch0, 1), cm = std::max(ch0 / 4, nm);
    const int widths[3] = {cb, cc, cm}, outs[3] = {4 * reg_max, 1, nm};
    const char* branch[3] = {".cv2.", ".cv3.", ".cv4."};
    const char* kind[3] = {"box", "cls", "coef"};
    for (int l = 0; l < 3; l++) {
      const std::string L = std::to_string(l);
      const int stem = conv(pre + ".h" + L + ".0", lv[l], cb + cc + cm, 3, 1);
      prims[stem].name = "h" + L + ".stem";
      int c0 = 0;
      for (int b = 0; b < 3; b++) {
        prims[stem].branch.push_back(pre + branch[b] + L + ".0");
        prims[stem].branch_k.push_back(widths[b]);
        const int sb = slice(stem, c0, c0 + widths[b], "h" + L + "." + kind[b] + ".1");
        c0 += widths[b];
        const int mid = conv(pre + branch[b] + L + ".1", sb, widths[b], 3, 1);
        prims[mid].name = "h" + L + "." + kind[b] + ".2";
        Prim h{P_HEAD, std::string("out.") + kind[b] + L, {mid}};
        h.C = outs[b];
        h.H = prims[mid].H;
        h.W = prims[mid].W;
        h.param = pre + branch[b] + L + ".2";
        h.output = true;
        head_prim[b][l] = prim(h);
      }
    }
    const int p1 = conv(pre + ".proto.cv1", lv[0], npr, 3, 1);
    prims[p1].name = "proto.1";
    Prim u{P_CONVT, "proto.up", {p1}};
    u.C = npr;
    u.H = 2 * prims[p1].H;
    u.W = 2 * prims[p1].W;
    u.param = pre + ".proto.upsample";
    const int pu = prim(u);
    const int p2 = conv(pre + ".proto.cv2", pu, npr, 3, 1);
    prims[p2].name = "proto.2";
    proto_prim = conv(pre + ".proto.cv3", p2, nm, 1, 1);
    prims[proto_prim].name = "out.proto";
    prims[proto_prim].output = true;
  }
  int head_prim[3][3] = {}, proto_prim = -1;

  void expand() {
    Prim x{P_INPUT, "in"};
    x.C = 3;
    x.H = x.W = S;
    int row_out[23];
    row_out[0] = -1;
    int cur = prim(x);
    for (int i = 0; i < 23; i++) {
      const Row& r = kLayers[i];
      int src[3];
      for (int j = 0; j < r.nfrom; j++) src[j] = r.from[j] < 0 ? (i == 0 ? cur : row_out[i - 1]) : row_out[r.from[j]];
      const std::string pre = "model." + std::to_string(i), tn = "L" + std::to_string(i);
      int out = -1;
      switch (r.m) {
        case M_CONV: out = conv(pre, src[0], width(r.ch), r.k, r.s); break;
        case M_C2F: out = expand_c2f(pre, tn, src[0], width(r.ch), depth(r.repeats), r.shortcut); break;
        case M_SPPF: out = expand_sppf(pre, tn, src[0], width(r.ch)); break;
        case M_UP: out = up2(src[0]); break;
        case M_CAT: out = concat(std::vector<int>(src, src + r.nfrom), tn); break;
        case M_SEGMENT: expand_segment(pre, src, width(r.ch)); break;
      }
      if (out >= 0 && prims[out].op != P_CAT && prims[out].op != P_UP2) prims[out].name = tn;
      row_out[i] = out;
    }
  }

  // Destinations of a producer's channels: they sit at channels [c0, c1) of primitive p, starting at the
  // producer's channel pc; followed through the slices, upsamples and concats that read p.
  void route(int p, int c0, int c1, int pc, int up, std::vector<MDest>& out) {
    for (int q = 0; q < (int)prims.size(); q++) {
      const Prim& Q = prims[q];
      for (size_t j = 0; j < Q.src.size(); j++) {
        if (Q.src[j] != p) continue;
        if (Q.op == P_CAT) {
          int off = 0;
          for (size_t t = 0; t < j; t++) off += prims[Q.src[t]].C;
          route(q, off + c0, off + c1, pc, up, out);
        } else if (Q.op == P_POOLCAT) {
          route(q, c0, c1, pc, up, out);
        } else if (Q.op == P_UP2) {
          route(q, c0, c1, pc, up * 2, out);
        } else if (Q.op == P_SLICE) {
          const int a = std::max(c0, Q.c0), b = std::min(c1, Q.c0 + Q.C);
          if (a < b) route(q, a - Q.c0, b - Q.c0, pc + (a - c0), up, out);
        }
      }
    }
    if (prims[p].buf) out.push_back(MDest{prims[p].buf, c0, pc, pc + (c1 - c0), up});
  }

  void build() {
    prims.clear();
    expand();
    // buffers: the input, every concat (and the SPPF pool concat), the model outputs, and every other
    // primitive that a compute primitive reads as its input or residual
    std::vector<char> read_direct(prims.size(), 0);
    for (const Prim& p : prims) {
      if (p.op == P_CONV || p.op == P_HEAD || p.op == P_CONVT) read_direct[p.src[0]] = 1;
      if (p.res >= 0) read_direct[p.res] = 1;
    }
    for (int i = 0; i < (int)prims.size(); i++) {
      Prim& p = prims[i];
      if (p.op == P_INPUT || p.op == P_CAT || p.op == P_POOLCAT || p.output || read_direct[i])
        p.buf = act(p.name, p.C, p.H, p.W);
    }
    in = prims[0].buf;
    for (int b = 0; b < 3; b++)
      for (int l = 0; l < 3; l++) head[b][l] = prims[head_prim[b][l]].buf;
    proto = prims[proto_prim].buf;
    // nodes, in primitive order
    for (int i = 0; i < (int)prims.size(); i++) {
      const Prim& p = prims[i];
      auto nd = std::make_unique<MNode>();
      nd->name = p.param;
      if (p.op == P_CONV) {
        nd->kind = N_CONVBN;
        nd->in = prims[p.src[0]].buf;
        nd->K = p.C;
        nd->k = p.k;
        nd->s = p.s;
        nd->pre = p.branch.empty() ? std::vector<std::string>{p.param} : p.branch;
        nd->ks = p.branch.empty() ? std::vector<int>{p.C} : p.branch_k;
        for (size_t b = 0; b < nd->pre.size(); b++) {
          add_param(nd->pre[b] + ".conv.weight", {nd->ks[b], nd->in->C, p.k, p.k});
          for (const char* t : {".bn.weight", ".bn.bias", ".bn.running_mean", ".bn.running_var"})
            add_param(nd->pre[b] + t, {nd->ks[b]});
        }
        route(i, 0, p.C, 0, 1, nd->dests);
        nd->res = p.res >= 0 ? prims[p.res].buf : nullptr;
      } else if (p.op == P_HEAD || p.op == P_CONVT) {
        nd->kind = p.op == P_HEAD ? N_HEAD : N_CONVT;
        nd->in = prims[p.src[0]].buf;
        nd->out = p.buf;
        nd->K = p.C;
        if (p.op == P_HEAD) add_param(p.param + ".weight", {p.C, nd->in->C, 1, 1});
        else add_param(p.param + ".weight", {nd->in->C, p.C, 2, 2});
        add_param(p.param + ".bias", {p.C});
      } else if (p.op == P_POOLCAT) {
        nd->kind = N_POOL;
        nd->cat = p.buf;
        nd->pc = prims[p.src[0]].C;
      } else {
        continue;
      }
      nodes.push_back(std::move(nd));
    }
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
    // the instantiated step graphs refer to the forward's streams' events: destroy them first
    for (Schedule* sc : {&fwd_sched, &det_sched}) {
      if (sc->exec) cudaGraphExecDestroy(sc->exec);
      if (sc->graph) cudaGraphDestroy(sc->graph);
      for (cudaEvent_t ev : sc->ev)
        if (ev) cudaEventDestroy(ev);
      *sc = Schedule{};
    }
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
    for (auto& p : dzx) {
      cudaFree(p);
      p = nullptr;
    }
    cudaFree(ws_side);
    cudaFree(prelaid);
    cudaFree(jobs);
    prelaid = nullptr;
    jobs = nullptr;
    njobs = 0;
    for (int i = 0; i < kDzBufs; i++) {
      if (ev_dz[i]) cudaEventDestroy(ev_dz[i]);
      if (ev_wg[i]) cudaEventDestroy(ev_wg[i]);
      ev_dz[i] = ev_wg[i] = nullptr;
    }
    if (ev_fork) cudaEventDestroy(ev_fork);
    if (ev_join) cudaEventDestroy(ev_join);
    if (side) cudaStreamDestroy(side);
    for (void* p : {(void*)det_xyxy, (void*)det_confs, (void*)det_n, (void*)det_keep, (void*)det_box,
                    (void*)det_score, (void*)det_coef, det_masks})
      cudaFree(p);
    det_xyxy = det_confs = det_box = det_score = nullptr;
    det_n = det_keep = nullptr;
    det_coef = nullptr;
    det_masks = nullptr;
    det_on = false;
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
    ws_side = nullptr;
    garena = nullptr;
    zarena = nullptr;
    tarena = nullptr;
    grad32 = nullptr;
    dz = gw16 = wconvt = nullptr;
    ws = bnws = nullptr;
    train = false;
    if (cap) cudaStreamDestroy(cap);
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
    synced = true;  // the step graphs stay valid: new weights, same buffers and kernel arguments
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

  // The tasks of a step: every node of the forward (what it reads and writes), and with `detect` the
  // post-process — decode (the box and class heads), NMS (decoded boxes, the coefficient heads) and the
  // masks (NMS results, proto) — so that decode and NMS run while the proto branch still computes.
  std::vector<Task> step_tasks(bool detect) {
    std::vector<Task> t;
    for (int i = 0; i < (int)nodes.size(); i++) {
      const MNode& nd = *nodes[i];
      Task k{T_NODE, i, {}, {}, 1.0};
      if (nd.kind == N_POOL) {
        k.reads = {nd.cat};
        k.writes = {nd.cat};
      } else {
        k.reads.push_back(nd.in);
        if (nd.res) k.reads.push_back(nd.res);
        if (nd.kind == N_CONVBN)
          for (const MDest& d : nd.dests) k.writes.push_back(d.a);
        else
          k.writes.push_back(nd.out);
        k.cost = 2.0 * (double)nd.plan.M * nd.plan.gemm_n * nd.plan.g.R * nd.plan.g.S * nd.plan.g.C;
      }
      t.push_back(std::move(k));
    }
    if (detect) {
      // Priorities of the post-process (FLOP-equivalents).  k_nms runs one latency-bound CTA per image for
      // ≈ 0.2 ms whatever the batch; it needs only the detection heads, so it should start as soon as they
      // are done and overlap the prototype branch, which only the mask assembly needs.  Weighting it at half
      // the step's conv FLOPs puts the head → decode → NMS chain ahead of the prototype chain (measured at
      // batch 64: detect step 4.19–4.21 → 4.08–4.10 ms; with the NMS at its time-equivalent weight, or
      // weightless, the prototype chain went first and the NMS ran after it).  Decode and mask assembly
      // count at their time-equivalents at the forward's rate of ≈ 0.67 PFLOP/s (≈ 0.15 µs and ≈ 3 µs per image).
      double conv_flops = 0.0;
      for (const Task& k : t) conv_flops += k.cost;
      const double cd = 1.0e8 * N, cn = 0.5 * conv_flops, cm = 2.0e9 * N;
      t.push_back(Task{T_DECODE, -1, {head[0][0], head[0][1], head[0][2], head[1][0], head[1][1], head[1][2]},
                       {&det_decoded}, cd});
      t.push_back(Task{T_NMS, -1, {&det_decoded, head[2][0], head[2][1], head[2][2]}, {&det_kept}, cn});
      t.push_back(Task{T_MASK, -1, {&det_kept, proto}, {&det_maskt}, cm});
    }
    return t;
  }

  // Dependency DAG of a step (a task depends on every earlier writer of a tensor it reads; concat buffers
  // are written by several nodes into disjoint channel slices).  Tasks are launched in a topological order
  // that puts the longest remaining chain (by FLOPs; the post-process by the weights above) first — so the
  // detection heads and the NMS go ahead of the proto branch, which then overlaps the NMS — and assigned
  // greedily to kFwdStreams streams: a task continues the stream whose last task is its latest producer,
  // else takes the stream idle longest.
  cudaError_t plan(Schedule& sc, bool detect) {
    if (!sc.stream.empty()) return cudaSuccess;
    sc.tasks = step_tasks(detect);
    const int n = (int)sc.tasks.size();
    std::map<const MAct*, std::vector<int>> writers;
    for (int i = 0; i < n; i++)
      for (const MAct* a : sc.tasks[i].writes) writers[a].push_back(i);
    std::vector<std::vector<int>> dep(n), succ(n);
    for (int i = 0; i < n; i++) {
      for (const MAct* a : sc.tasks[i].reads) {
        auto it = writers.find(a);
        if (it == writers.end()) continue;
        for (int w : it->second)
          if (w < i) dep[i].push_back(w);
      }
      std::sort(dep[i].begin(), dep[i].end());
      dep[i].erase(std::unique(dep[i].begin(), dep[i].end()), dep[i].end());
      for (int w : dep[i]) succ[w].push_back(i);
    }
    std::vector<double> bottom(n, 0.0);  // FLOPs of the longest chain from a task to the end
    for (int i = n - 1; i >= 0; i--) {
      double m = 0.0;
      for (int sx : succ[i]) m = std::max(m, bottom[sx]);
      bottom[i] = sc.tasks[i].cost + m;
    }
    sc.order.clear();
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
      sc.order.push_back(pick);
      for (int sx : succ[pick])
        if (--pending[sx] == 0) ready[sx] = 1;
    }
    sc.stream.assign(n, 0);
    sc.waits.assign(n, {});
    std::vector<char> signal(n, 0);
    int tail[kFwdStreams];
    for (int k = 0; k < kFwdStreams; k++) tail[k] = -1;
    std::vector<int> pos(n);
    for (int q = 0; q < n; q++) pos[sc.order[q]] = q;
    for (int q = 0; q < n; q++) {
      const int i = sc.order[q];
      int st = -1, best = -1;  // the latest-launched producer that is still the tail of its stream
      for (int w : dep[i])
        if (tail[sc.stream[w]] == pos[w] && (best < 0 || pos[w] > pos[best])) best = w;
      if (best >= 0) st = sc.stream[best];
      if (st < 0) {
        st = 0;
        for (int k = 1; k < kFwdStreams; k++)
          if (tail[k] < tail[st]) st = k;
      }
      sc.stream[i] = st;
      int latest[kFwdStreams];  // per other stream, the producer launched last there
      for (int k = 0; k < kFwdStreams; k++) latest[k] = -1;
      for (int w : dep[i]) {
        const int ks = sc.stream[w];
        if (ks != st && (latest[ks] < 0 || pos[w] > pos[latest[ks]])) latest[ks] = w;
      }
      for (int k = 0; k < kFwdStreams; k++)
        if (latest[k] >= 0) {
          sc.waits[i].push_back(latest[k]);
          signal[latest[k]] = 1;
        }
      tail[st] = q;
    }
    cudaError_t e;
    sc.ev.assign(n, nullptr);
    for (int i = 0; i < n; i++)
      if (signal[i] && (e = cudaEventCreateWithFlags(&sc.ev[i], cudaEventDisableTiming)) != cudaSuccess) return e;
    if (!ev_fwd_start) {
      for (int k = 0; k < kFwdStreams - 1; k++) {
        if ((e = cudaStreamCreateWithFlags(&fwd_st[k], cudaStreamNonBlocking)) != cudaSuccess) return e;
        if ((e = cudaEventCreateWithFlags(&ev_fwd_end[k], cudaEventDisableTiming)) != cudaSuccess) return e;
      }
      if ((e = cudaEventCreateWithFlags(&ev_fwd_start, cudaEventDisableTiming)) != cudaSuccess) return e;
    }
    return cudaSuccess;
  }

  cudaError_t launch_task(const Task& t, cudaStream_t s) {
    if (t.kind == T_NODE) {
      MNode& nd = *nodes[t.node];
      return nd.kind == N_POOL ? launch_sppf(nd.cat->p, N, nd.cat->H, nd.cat->W, nd.pc, s) : conv_launch(nd.L, s);
    }
    const int hw[6] = {head[0][0]->H, head[0][0]->W, head[0][1]->H, head[0][1]->W, head[0][2]->H, head[0][2]->W};
    const int A = hw[0] * hw[1] + hw[2] * hw[3] + hw[4] * hw[5];
    const osam_stream_t os = reinterpret_cast<osam_stream_t>(s);
    int rc = OSAM_OK;
    if (t.kind == T_DECODE) {
      const void* box[3] = {head[0][0]->p, head[0][1]->p, head[0][2]->p};
      const void* cls[3] = {head[1][0]->p, head[1][1]->p, head[1][2]->p};
      rc = osam_decode(box, cls, hw, N, S, reg_max, det_xyxy, det_confs, os);
    } else if (t.kind == T_NMS) {
      const void* coef[3] = {head[2][0]->p, head[2][1]->p, head[2][2]->p};
      rc = osam_nms(det_xyxy, det_confs, N, A, det_conf, det_iou, det_max, det_forced, coef, hw, det_n, det_keep,
                    det_box, det_score, det_coef, os);
    } else {
      rc = osam_mask_assemble(det_coef, proto->p, det_box, det_n, N, proto->H, proto->W, S, det_max, det_packed,
                              det_masks, os);
    }
    return rc == OSAM_OK ? cudaSuccess : cudaErrorLaunchFailure;
  }

  cudaError_t run(Schedule& sc, cudaStream_t st) {
    cudaStream_t ss[kFwdStreams] = {st};
    for (int k = 1; k < kFwdStreams; k++) ss[k] = fwd_st[k - 1];
    cudaError_t e;
    // fork: the internal streams start after the caller's stream has reached this point
    if ((e = cudaEventRecord(ev_fwd_start, st)) != cudaSuccess) return e;
    for (int k = 1; k < kFwdStreams; k++)
      if ((e = cudaStreamWaitEvent(ss[k], ev_fwd_start, 0)) != cudaSuccess) return e;
    for (int i : sc.order) {
      cudaStream_t s = ss[sc.stream[i]];
      for (int w : sc.waits[i])
        if ((e = cudaStreamWaitEvent(s, sc.ev[w], 0)) != cudaSuccess) return e;
      if ((e = launch_task(sc.tasks[i], s)) != cudaSuccess) return e;
      if (sc.ev[i] && (e = cudaEventRecord(sc.ev[i], s)) != cudaSuccess) return e;
    }
    // join: the caller's stream continues after every task
    for (int k = 1; k < kFwdStreams; k++) {
      if ((e = cudaEventRecord(ev_fwd_end[k - 1], ss[k])) != cudaSuccess) return e;
      if ((e = cudaStreamWaitEvent(st, ev_fwd_end[k - 1], 0)) != cudaSuccess) return e;
    }
    return cudaSuccess;
  }

  // One step (the forward, or the forward with the post-process), eagerly or as this schedule's captured
  // CUDA graph (recorded at the first call, on the model's own stream, replayed on the caller's).
  int step(Schedule& sc, bool detect, int use_graph, cudaStream_t st) {
    cudaError_t e;
    if ((e = plan(sc, detect)) != cudaSuccess)  // streams and events exist before any capture begins
      return model_fail(OSAM_ERR_CUDA, "step schedule: %s", cudaGetErrorString(e));
    if (!use_graph) {
      e = run(sc, st);
      return e == cudaSuccess ? OSAM_OK : model_fail(OSAM_ERR_CUDA, "step: %s", cudaGetErrorString(e));
    }
    if (!sc.exec) {
      if (!cap && (e = cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking)) != cudaSuccess)
        return model_fail(OSAM_ERR_CUDA, "capture stream: %s", cudaGetErrorString(e));
      if ((e = cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal)) != cudaSuccess)
        return model_fail(OSAM_ERR_CUDA, "begin capture: %s", cudaGetErrorString(e));
      cudaError_t er = run(sc, cap);
      e = cudaStreamEndCapture(cap, &sc.graph);
      if (er != cudaSuccess || e != cudaSuccess)
        return model_fail(OSAM_ERR_CUDA, "capture: %s", cudaGetErrorString(er != cudaSuccess ? er : e));
      if ((e = cudaGraphInstantiate(&sc.exec, sc.graph, 0)) != cudaSuccess)
        return model_fail(OSAM_ERR_CUDA, "instantiate: %s", cudaGetErrorString(e));
    }
    e = cudaGraphLaunch(sc.exec, st);
    return e == cudaSuccess ? OSAM_OK : model_fail(OSAM_ERR_CUDA, "graph launch: %s", cudaGetErrorString(e));
  }

  int detect_init(float conf_th, float iou_th, int max_det, int forced, int packed) {
    if (!synced) return model_fail(OSAM_ERR_INVALID, "detect_init before osam_model_sync_weights");
    if (max_det < 1 || max_det > 1024) return model_fail(OSAM_ERR_INVALID, "max_det must be in [1, 1024]");
    // settings change the captured launches: drop the detect step's graph (its buffers stay if sizes match)
    if (det_sched.exec) cudaGraphExecDestroy(det_sched.exec);
    if (det_sched.graph) cudaGraphDestroy(det_sched.graph);
    det_sched.exec = nullptr;
    det_sched.graph = nullptr;
    const size_t A = (size_t)head[0][0]->H * head[0][0]->W + (size_t)head[0][1]->H * head[0][1]->W +
                     (size_t)head[0][2]->H * head[0][2]->W;
    const size_t pad = ((size_t)max_det + 127) / 128 * 128, hw = (size_t)proto->H * proto->W;
    const size_t mask_bytes = packed ? 4 * ((hw + 31) / 32) : hw;
    if (!det_on || max_det != det_max || packed != det_packed) {
      for (void* q : {(void*)det_xyxy, (void*)det_confs, (void*)det_n, (void*)det_keep, (void*)det_box,
                      (void*)det_score, (void*)det_coef, det_masks})
        cudaFree(q);
      cudaError_t e;
      if ((e = cudaMalloc(&det_xyxy, (size_t)N * A * 4 * sizeof(float))) != cudaSuccess ||
          (e = cudaMalloc(&det_confs, (size_t)N * A * sizeof(float))) != cudaSuccess ||
          (e = cudaMalloc(&det_n, (size_t)N * sizeof(int))) != cudaSuccess ||
          (e = cudaMalloc(&det_keep, (size_t)N * max_det * sizeof(int))) != cudaSuccess ||
          (e = cudaMalloc(&det_box, (size_t)N * max_det * 4 * sizeof(float))) != cudaSuccess ||
          (e = cudaMalloc(&det_score, (size_t)N * max_det * sizeof(float))) != cudaSuccess ||
          (e = cudaMalloc(&det_coef, (size_t)N * pad * 32 * sizeof(__half))) != cudaSuccess ||
          (e = cudaMalloc(&det_masks, (size_t)N * max_det * mask_bytes)) != cudaSuccess) {
        det_on = false;
        return model_fail(OSAM_ERR_NOMEM, "detection buffers: %s", cudaGetErrorString(e));
      }
    }
    det_conf = conf_th;
    det_iou = iou_th;
    det_max = max_det;
    det_forced = forced ? 1 : 0;
    det_packed = packed ? 1 : 0;
    det_on = true;
    return OSAM_OK;
  }

  int plan_gradient_modes() {
    // Gradient write modes.  An activation read by several nodes (as input or as residual) receives one
    // gradient contribution per read.  The backward visits nodes last to first, so the read in the LAST
    // reading node writes (beta 0) and every earlier read accumulates (beta 1); inside one node the
    // residual's gradient is written before the input gradient.  Every buffer a node writes must receive a
    // gradient: from a later reader, or from the caller (the heads and proto).
    std::map<const MAct*, int> last_reader;
    for (int i = 0; i < (int)nodes.size(); i++) {
      const MNode& nd = *nodes[i];
      if (nd.kind == N_POOL) continue;
      last_reader[nd.in] = i;
      if (nd.res) last_reader[nd.res] = i;
    }
    auto gets_grad = [&](const MAct* a, int i) {
      if (a == proto) return true;
      for (int l = 0; l < 3; l++)
        for (int k = 0; k < 3; k++)
          if (a == head[k][l]) return true;
      auto it = last_reader.find(a);
      return it != last_reader.end() && it->second > i;
    };
    for (int i = 0; i < (int)nodes.size(); i++) {
      MNode& nd = *nodes[i];
      if (nd.kind == N_POOL) continue;
      if (nd.kind == N_CONVBN) {
        for (auto& d : nd.dests)
          if (!gets_grad(d.a, i))
            return model_fail(OSAM_ERR_INVALID, "%s: nothing reads %s", nd.name.c_str(), d.a->name.c_str());
      } else if (!gets_grad(nd.out, i)) {
        return model_fail(OSAM_ERR_INVALID, "%s: nothing reads its output", nd.name.c_str());
      }
      if (nd.res) nd.res_accum = last_reader[nd.res] != i;
      if (nd.in != in) nd.dgrad_accum = last_reader[nd.in] != i || nd.res == nd.in;
    }
    return OSAM_OK;
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
        (e = cudaMalloc(&ws_side, wsb)) != cudaSuccess)
      return model_fail(OSAM_ERR_NOMEM, "training buffers: %s", cudaGetErrorString(e));
    for (auto& p : dzx)
      if ((e = cudaMalloc(&p, std::max<size_t>(dzn, 1) * sizeof(__half))) != cudaSuccess)
        return model_fail(OSAM_ERR_NOMEM, "dz buffers: %s", cudaGetErrorString(e));
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    if ((e = cudaStreamCreateWithPriority(&side, cudaStreamNonBlocking, lo)) != cudaSuccess)
      return model_fail(OSAM_ERR_CUDA, "side stream: %s", cudaGetErrorString(e));
    for (int i = 0; i < kDzBufs; i++) {
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
    if (int rc = plan_gradient_modes()) return rc;
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
        osam_dest d[OSAM_MAX_DEST];
        for (size_t i = 0; i < nd.dests.size(); i++)
          d[i] = osam_dest{nd.dests[i].a->p, nd.dests[i].a->C, nd.dests[i].choff, nd.dests[i].c0, nd.dests[i].c1,
                           nd.dests[i].up};
        // batch statistics and the normalised, activated output in one kernel
        if (!rc)
          rc = osam_bn_forward_train(nd.z, N, P, Q, K, T, T + K, T + 2 * K, T + 3 * K, momentum, bn_eps, T + 4 * K,
                                     T + 5 * K, T + 6 * K, T + 7 * K, nd.res ? nd.res->p : nullptr, d,
                                     (int)nd.dests.size(), 1, bnws, bnws_bytes, st);
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
    bool busy[kDzBufs] = {};
    int buf = 0;
    for (int i = first + count - 1; i >= first; i--) {
      MNode& nd = *nodes[i];
      int rc = OSAM_OK;
      if (nd.kind == N_CONVBN) {
        const int P = nd.plan.P, Q = nd.plan.Q, K = nd.K;
        float* T = tarena + nd.t_off;
        __half* d = buf ? dzx[buf - 1] : dz;
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
        buf = (buf + 1) % kDzBufs;
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
    return step(fwd_sched, false, use_graph, st);
  }

  int forward_detect(int use_graph, cudaStream_t st) {
    if (!synced) return model_fail(OSAM_ERR_INVALID, "forward before osam_model_sync_weights");
    if (!det_on) return model_fail(OSAM_ERR_INVALID, "forward_detect before osam_model_detect_init");
    return step(det_sched, true, use_graph, st);
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
  if ((rc = error_word_init()) != OSAM_OK || !device_error_word()) {
    m->release();
    return rc ? rc : model_fail(OSAM_ERR_CUDA, "device error word");
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

int osam_model_detect_init(osam_model* m, float conf_th, float iou_th, int max_det, int forced, int packed) {
  if (!m) return model_fail(OSAM_ERR_INVALID, "NULL model");
  return m->detect_init(conf_th, iou_th, max_det, forced, packed);
}

int osam_model_forward_detect(osam_model* m, int use_graph, osam_stream_t stream) {
  if (!m) return model_fail(OSAM_ERR_INVALID, "NULL model");
  return m->forward_detect(use_graph, reinterpret_cast<cudaStream_t>(stream));
}

int osam_model_detections(const osam_model* m, osam_detections* d) {
  if (!m || !d) return model_fail(OSAM_ERR_INVALID, "NULL argument");
  if (!m->det_on) return model_fail(OSAM_ERR_INVALID, "no detections before osam_model_detect_init");
  d->batch = m->N;
  d->anchors = m->head[0][0]->H * m->head[0][0]->W + m->head[0][1]->H * m->head[0][1]->W +
               m->head[0][2]->H * m->head[0][2]->W;
  d->max_det = m->det_max;
  d->packed = m->det_packed;
  d->proto_h = m->proto->H;
  d->proto_w = m->proto->W;
  d->xyxy = m->det_xyxy;
  d->conf = m->det_confs;
  d->n_det = m->det_n;
  d->keep = m->det_keep;
  d->box = m->det_box;
  d->score = m->det_score;
  d->coef_g = m->det_coef;
  d->masks = m->det_masks;
  return OSAM_OK;
}

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
