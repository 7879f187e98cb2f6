// Internal (C++) interface between the C ABI / model runner and the conv kernels.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/osam.h"

namespace osam {

// How the A (activation) tile of one K-step is fetched by TMA.
enum AMode : int {
  A_GEMM = 0,  // 1×1/s1/p0 conv or transposed conv: A is the [N·H·W, C] matrix itself (2-D map)
  A_S1 = 1,    // stride-1 R×S conv: 4-D map (C, W, H, N); one shifted box per tap, halo = TMA zero fill
  A_S2 = 2,    // stride-2 conv: 5-D map (2C, W/2, 2, H/2, N) — the parity-split view of NHWC — so a
               // stride-2 gather becomes a dense box per tap
  A_STEM = 3,  // R·S·C ≤ 32 (RGB stem): per-thread im2col gather into shared memory, no TMA
  A_WIN = 4,   // 3×3/s1/p1 with C, K ∈ {32, 64} (conv_win.cu): one shared input window per 128-position tile
  A_W3 = 5,    // 3×3/s1/p1 (conv_fprop.cu): 128-pixel tiles (rows × images × columns); per channel chunk three
               // column-shifted input windows, each serving its column's three taps
  A_W3R = 6,   // A_W3 with all nine weight taps resident in shared memory (C = BK, one N tile, BN ≤ 64)
  A_W3S2 = 7,  // 3×3/s2/p1 window form: three column windows of the parity view per chunk (16 × 8 tiles)
  A_W3S2R = 8  // A_W3S2 with the weight taps resident
};
constexpr bool mode_window(int m) { return m == A_W3 || m == A_W3R || m == A_W3S2 || m == A_W3S2R; }
constexpr bool mode_resident(int m) { return m == A_W3R || m == A_W3S2R; }
constexpr bool mode_s2_window(int m) { return m == A_W3S2 || m == A_W3S2R; }

// Dynamic shared memory a window-conv CTA may use (the sm_100 opt-in limit per block).
constexpr size_t kWinSmemLimit = 227 * 1024;

struct DestDev {
  __half* p;
  int ctot, choff, c0, c1, up;
  int vec;  // 16-byte vector stores allowed
};

struct EpiDev {
  int kind;  // OSAM_EPI_*
  const float* scale;
  const float* shift;
  const float* bias;
  const __half* res;
  int act, round_z;
  float beta;  // OSAM_EPI_STORE: y = conv + beta·y
  int ndest;
  DestDev dest[OSAM_MAX_DEST];
  int shuffle;  // transposed conv: GEMM column j = (dy·2+dx)·kout + k → pixel (2p+dy, 2q+dx)
  int kout;     // channels per (dy,dx) block for shuffle
  int par;      // 1..4: every column goes to pixel (2p + (par−1)/2, 2q + (par−1)%2) of a 2P × 2Q grid (the
                // output-parity classes of a stride-2 dgrad); 0: none
  int coop;     // warp-cooperative coalesced epilogue allowed (see epilogue.cuh)
  int tstore;   // warp rows leave through TMA tensor stores (StoreMaps); implies coop
  int wtw, wth, wtn;  // a warp's 32 rows as a (wtn images × wth rows × wtw cols) box of the tile
};

// Division by a divisor fixed at launch preparation without the integer-division instruction sequence:
// q = (umulhi(n, m) + n) >> s for 0 ≤ n < 2³¹, with s = ⌈log₂ d⌉ and m = ⌊2³²·(2ˢ − d)/d⌋ + 1 (the
// round-up method of Granlund & Montgomery, "Division by invariant integers using multiplication", 1994).
// A power of two gives m = 1: a shift.  The kernels' per-tile and per-row index math (tile → image, row,
// column) uses it; with the generic sequence that math cost about as many instructions as the
// epilogue's arithmetic on the narrow layers.
struct FastDiv {
  int d = 1, s = 0;
  uint32_t m = 1;
  void set(int dv) {
    d = dv < 1 ? 1 : dv;
    s = 0;
    while ((1LL << s) < d) s++;
    m = (uint32_t)(((1ULL << 32) * ((1ULL << s) - (unsigned long long)d)) / (unsigned long long)d + 1);
  }
#ifdef __CUDACC__
  __device__ __forceinline__ int quo(int n) const {
    return (int)((__umulhi((uint32_t)n, m) + (uint32_t)n) >> s);
  }
  __device__ __forceinline__ int rem(int n, int q) const { return n - q * d; }
#endif
};

struct ConvDev {
  int N, H, W, C, K, P, Q, R, S, stride, pad;
  int gemm_n;                 // GEMM N (= K, or 4·K for the transposed conv)
  int tn, th, tw;             // spatial tile (tn images × th rows × tw cols = 128 pixels)
  int tiles_q, tiles_p;       // spatial tiles along Q and P
  long long M;                // N·P·Q (GEMM M) — for the transposed conv N·H·W
  int ntn;                    // tiles along GEMM N
  int tiles_m;                // tiles along GEMM M
  int nkc;                    // channel chunks per tap
  int nk;                     // K iterations = taps · nkc
  int win_wp, win_lw;         // A_WIN: row pitch W + 2 of the flattened space, window length (positions)
  int win_slab, win_wbytes;   // A_WIN: bytes of one 8-channel slab of a window, of one window buffer
  int win_tpi;                // A_WIN: 128-position tiles per image
  int win_nwb;                // A_WIN: window buffers (2 or 3)
  unsigned win_mul;           // A_WIN: ⌈2³²/pitch⌉ — u / pitch = umulhi(u, win_mul) for the sizes planned
  int* err;                   // device error word
  // the divisions of the conv kernels' index math (FastDiv): GEMM-N tiles, spatial tiles along Q and P,
  // tile columns, images × columns of a window-form tile row, rows × columns of a tile, channel chunks, S
  FastDiv f_ntn, f_tq, f_tp, f_tw, f_nw, f_thw, f_nkc, f_S;
  EpiDev ep;
};

// Output tensor maps of the TMA-store epilogue: index 4·dest + view; view 0 for plain destinations, views
// (dy·2+dx) for 2×-upsampled destinations and for the transposed conv's pixel shuffle.
constexpr int kMaxStoreMaps = 4 * OSAM_MAX_DEST;
struct StoreMaps {
  CUtensorMap m[kMaxStoreMaps];
};

struct ConvLaunch {
  int BK, BN, mode;
  int pair;  // conv_fprop: CTA pairs with 2-SM UMMAs (the weight map's box is then BN/2 rows)
  int grid;
  CUtensorMap ta, tb;
  StoreMaps sm;
  ConvDev d;
  // transposed conv: weights must be re-laid out (C,R,S,K) → (R·S·K, C) before the GEMM
  const __half* wt_src = nullptr;
  __half* wt_dst = nullptr;
  // A_STEM: raw operand pointers (no tensor maps)
  const __half* x = nullptr;
  const __half* w = nullptr;
  int stem_rgb = 0;  // pipelined RGB stem kernel (window tensor map in ta, TMA-store epilogue)
};

// One weight-gradient launch (conv_wgrad.cu).
struct WgradLaunch {
  CUtensorMap tdz, tx;  // dz (K, Q, P, N) and x (forward A view) boxes of 128 tile pixels
  ConvDev d;            // geometry and the forward plan's spatial tiling
  float* acc;           // fp32 KRSC accumulator (workspace), zeroed by the launch
  __half* dw;           // fp16 KRSC result
  float* dw32;          // or, when non-null, the fp32 result (dw unused)
  bool direct;          // dw32 is zero already: the kernels add into it (acc = dw32, no zeroing, no finish pass)
  long long n_out;      // K·R·S·C
  float beta;
  int AB, BB, BN;       // dz / x box channels (32 or 64), GEMM N block
  int mode;             // A_S1, A_S2, or A_STEM (R·S·C ≤ 32: patch gather, dz as one 2-D map)
  const __half* xp;     // A_STEM: the input itself (gathered by the producer warps, no tensor map)
  int grid, nsplit, tiles_per_split;
  // window form (3×3, pad 1, C = 32·CB ∈ {32, 64}): per tile one dz box and, per column tap, one x window per
  // 32-channel block, the three row taps stacked in the GEMM M dimension (d.th/tw/tn/tiles_* = its tiling)
  int win;              // 0 = per-tap form; 1 = window form
  int CB, NB;           // 32-channel blocks of x; dz channels (GEMM N) per CTA
  int win_bytes;        // bytes of one x window box
};
cudaError_t launch_conv_wgrad(const WgradLaunch& L, cudaStream_t st);
// the (x channel blocks, dz channels per CTA) pairs the window form of the weight gradient is built for
bool wgrad_win_supported(int CB, int NB);
// 1×1 conv with one output channel: dx = dy ⊗ w (+ beta·dx); dw = Σ dy·x (fp32 acc[C] scratch, + beta·dw)
cudaError_t launch_dgrad_k1(const __half* dy, const __half* w, __half* dx, long long npix, int C, float beta,
                            cudaStream_t st);
cudaError_t launch_wgrad_k1(const __half* x, const __half* dy, float* acc, __half* dw, float* dw32, long long npix,
                            int C, float beta, bool direct, cudaStream_t st);
// osam_conv_wgrad with the result in fp32 (dw32, + beta·dw32) instead of fp16: the training path's gradient arena.
// direct = true: dw32 has been zeroed by the caller and the kernels add into it (no workspace, no extra passes).
int conv_wgrad_f32(const osam_conv_plan* plan, const void* x, const void* dz, float* dw32, float beta, void* ws,
                   size_t ws_bytes, cudaStream_t st, bool direct = false);
// osam_conv_dgrad with the sub-convs' re-laid-out weights already in `prelaid` (dgrad_prelaid_bytes(plan) bytes,
// written by launch_dgrad_weights_batched); prelaid = nullptr re-lays them out into ws first.
int conv_dgrad_ex(const osam_conv_plan* plan, const void* dz, const void* w, void* dx, float beta, void* ws,
                  size_t ws_bytes, cudaStream_t st, const __half* prelaid);
size_t dgrad_prelaid_bytes(const osam_conv_plan* plan);
struct DgradJob {
  const __half* w;
  __half* dst;
  int K, R, S, C, Rs, Ss;
  int r[8], s[8];
  long long n;
};
// All of a model's dgrad weight re-layouts (jobs in device memory) in one launch.
cudaError_t launch_dgrad_weights_batched(const DgradJob* jobs, int njobs, cudaStream_t st);
// The jobs that produce `prelaid` for one plan from its KRSC weights (at most 4; returns the count).
int dgrad_jobs(const osam_conv_plan* plan, const __half* w, __half* prelaid, DgradJob* out);

// Fills `L` (tensor maps, tiling, epilogue) for one call.  Returns an OSAM_* code.
// err_word: device word the kernels report timeouts to (nullptr = the library's per-device word).
// y_ctot / y_choff (plain store only): y is a slice [y_choff, y_choff + K) of a tensor with y_ctot channels.
int conv_prepare(const osam_conv_plan* plan, const void* x, const void* w, const osam_epilogue* ep, float beta,
                 void* y, void* ws, size_t ws_bytes, ConvLaunch* L, bool w_gemm_ready = false,
                 int* err_word = nullptr, int par = 0, int y_ctot = 0, int y_choff = 0);
cudaError_t launch_dgrad_weights(const __half* w, __half* dst, int K, int R, int S, int C, int Rs, int Ss,
                                 const int* rmap, const int* smap, cudaStream_t st);
cudaError_t conv_launch(const ConvLaunch& L, cudaStream_t st);
// One-time per-kernel set-up (dynamic shared-memory opt-in) without launching: call before capturing.
cudaError_t conv_prime(const ConvLaunch& L);
cudaError_t sppf_prime();

// kernels living in other translation units
cudaError_t launch_conv_fprop(const ConvLaunch& L, cudaStream_t st, bool prime_only = false);
cudaError_t launch_conv_win(const ConvLaunch& L, cudaStream_t st, bool prime_only = false);
size_t win_fixed_smem_bytes(int C, int K);  // a window-conv CTA's shared memory besides its windows
cudaError_t launch_convt_weight_relayout(const __half* src, __half* dst, int C, int RS, int K, cudaStream_t st);
cudaError_t launch_sppf(__half* cat, int N, int H, int W, int c, cudaStream_t st);
cudaError_t launch_sppf_bwd(const __half* cat, __half* dcat, int N, int H, int W, int c, cudaStream_t st);
size_t sppf_bwd_smem_bytes(int H, int W);
cudaError_t launch_conv_stem(const __half* x, const __half* w, const ConvDev& d, int BN, cudaStream_t st);
cudaError_t launch_conv_stem_rgb(const ConvLaunch& L, cudaStream_t st);

int* device_error_word();       // the error word kernels report to (host-mapped after error_word_init)
int error_word_init();           // allocates the host-mapped error word once per process (plan/model creation)
int static_scratch_take_error();  // error recorded by the static-scratch entry point's kernels (and clear it)
void set_last_error(const char* fmt, ...);

}  // namespace osam

struct osam_conv_plan {
  osam_conv_geom g;
  int transposed;
  int P, Q;
  int mode, BK, BN;
  int tn, th, tw, tiles_q, tiles_p;
  long long M;
  int gemm_n, ntn, nkc, nk, tiles_m;
  // dgrad: sub-plans over dz (1 for stride 1, the 4 output-parity classes for stride 2) with their weight
  // re-layouts Wsub[c][r'][s'][k] = W[k][rmap[r']][smap[s']][c] packed in the caller's workspace
  osam_conv_plan* dg[4];
  int n_dg, dg_par[4], dg_R[4], dg_S[4], dg_rmap[4][8], dg_smap[4][8];
  // transposed conv (k = s = 2): dg[0] is the forward conv {N, 2H, 2W, C_out → C_in, 2×2, stride 2} whose
  // KRSC weights are the transposed conv's own (C_in, R, S, C_out) array: dgrad runs it on dy as is, and
  // wgrad is that conv's weight gradient with the operands' roles swapped.
  int dg_direct;
  // stride-1 convs with more than 512 input channels: the dgrad's output channels in dg_n_chunk slices of
  // dg_chunk channels (sub-plan i writes dx channels [dg_chunk·i, dg_chunk·(i+1)) of one re-laid-out set)
  int dg_chunk;
  long long dg_woff[4];
  // window tiling (A_WIN), used when the epilogue allows the coalesced warp stores (decided per call)
  int win, win_wp, win_lw, win_slab, win_wbytes, win_tpi, win_tiles, win_nwb;
  unsigned win_mul;
};
