// C ABI (include/osam.h): conv plans, TMA tensor-map encoding, argument validation and dispatch.
// Replaces the cuDNN descriptor/plan machinery of ConvOp (reference src/conv.cpp:64-366): the tile shape
// of a layer is a static function of its geometry, so "tuning" is a table lookup.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>

#include "conv_internal.h"
#include "sm100.cuh"

namespace osam {

// ------------------------------------------------------------------ errors
static thread_local char g_last_error[512] = "";

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

static int cuda_fail(cudaError_t e, const char* what) {
  return fail(OSAM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// ------------------------------------------------------------------ device error word
// Kernels record a failed bounded wait in an error word.  At the first plan or model creation the word
// becomes one int of pinned, host-mapped memory shared by every device (allocated once per process,
// never inside a launch), so the host can read it at any time without synchronising
// (osam_device_error_peek).  Before that — post-process or BN entry points used without any plan — the
// kernels report to a file-scope device variable, which needs no allocation at all.
static __device__ int g_dev_err_word;
static std::mutex g_err_mu;
static int* g_err_static[64] = {};       // device address of g_dev_err_word, per device
static volatile int* g_err_host = nullptr;  // host view of the mapped word
static int* g_err_mapped = nullptr;         // device view of the mapped word

int error_word_init() {
  std::lock_guard<std::mutex> lk(g_err_mu);
  if (g_err_mapped) return OSAM_OK;
  int* h = nullptr;
  cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&h), 64, cudaHostAllocMapped | cudaHostAllocPortable);
  if (e != cudaSuccess) return fail(OSAM_ERR_CUDA, "error word: cudaHostAlloc: %s", cudaGetErrorString(e));
  *h = 0;
  void* d = nullptr;
  if ((e = cudaHostGetDevicePointer(&d, h, 0)) != cudaSuccess || d != h) {
    cudaFreeHost(h);
    return fail(OSAM_ERR_CUDA, "error word: no unified device address for mapped host memory");
  }
  g_err_host = h;
  g_err_mapped = h;
  return OSAM_OK;
}

int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_err_mu);
  if (g_err_mapped) return g_err_mapped;
  if (!g_err_static[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dev_err_word) != cudaSuccess || !p) return nullptr;
    g_err_static[dev] = static_cast<int*>(p);
  }
  return g_err_static[dev];
}

// Self-test of the bounded wait: one thread waits on an mbarrier that nothing arrives at, with the given
// budget, so the wait runs out, records kDevErrTimeout in the error word and the kernel returns.
__global__ void k_selftest_wait(unsigned long long budget_ns, int* err) {
  __shared__ __align__(8) uint64_t bar;
  mbar_init(&bar, 1);
  fence_barrier_init();
  mbar_wait_for(&bar, 0, err, budget_ns);
}

// ------------------------------------------------------------------ tensor maps
typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled_t encode_fn() {
  static PFN_encodeTiled_t fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled_t>(p);
  });
  return fn;
}

// fp16 tensor map: dims[0] innermost, strides in bytes for dims 1..rank-1.
static int make_map(CUtensorMap* tm, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_b,
                    const uint32_t* box, int row_bytes) {
  PFN_encodeTiled_t fn = encode_fn();
  if (!fn) return fail(OSAM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(base) & 15) return fail(OSAM_ERR_INVALID, "operand not 16-byte aligned");
  cuuint64_t gd[5], gs[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; i++) {
    gd[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i < rank - 1) {
      gs[i] = strides_b[i];
      if (strides_b[i] & 15) return fail(OSAM_ERR_INVALID, "tensor stride %llu not a multiple of 16 B",
                                         (unsigned long long)strides_b[i]);
    }
  }
  const CUtensorMapSwizzle sw = row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                  : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void*>(base), gd, gs, bx, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(OSAM_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return OSAM_OK;
}

// ------------------------------------------------------------------ planning
// GEMM N tile: the narrowest that covers GEMM N (96 and 192: the input gradients of the C2f output convs,
// whose GEMM N is 3·c_; a 128 / 224 tile would not divide it and force the scalar epilogue).
static int choose_bn(int gemm_n) {
  static const int opts[] = {16, 32, 64, 96, 128, 192, 224, 256};
  if (gemm_n <= 256)
    for (int o : opts)
      if (o >= gemm_n) return o;
  if (gemm_n % 256 == 0) return 256;
  return 128;
}

static long long cdivll(long long a, long long b) { return (a + b - 1) / b; }

// 128-pixel spatial tile (tn images × th rows × tw cols) with the least padding; ties → wider rows.
static void choose_tile(int N, int P, int Q, int* tn, int* th, int* tw) {
  long long best = -1;
  for (int lw = 7; lw >= 0; lw--)
    for (int lh = 7 - lw; lh >= 0; lh--) {
      const int w = 1 << lw, h = 1 << lh, n = 128 / (w * h);
      const long long cost = cdivll(Q, w) * cdivll(P, h) * cdivll(N, n);
      if (best < 0 || cost < best) {
        best = cost;
        *tn = n;
        *th = h;
        *tw = w;
      }
    }
}

// Window tiling for a narrow 3×3/s1/p1 conv (conv_win.cu): 128 positions of the row-flattened output
// per tile, pitch = W + 2 rounded up to 32 (so every warp's 32 positions lie in one output row), and a
// window of 128 + 2·pitch + 2 input positions in C/8 slabs of 16-byte rows (an odd row count per slab
// keeps the slabs on different shared-memory banks); two or three windows and all nine weight taps must
// fit in shared memory.
static void plan_win(osam_conv_plan* p) {
  const osam_conv_geom& g = p->g;
  p->win = 0;
  if (p->transposed || g.stride != 1 || g.R != 3 || g.S != 3 || g.pad != 1) return;
  if ((g.C != 32 && g.C != 64) || (g.K != 32 && g.K != 64)) return;
  // measured on B200: the window wins for 32 input channels on grids ≥ 64 wide; at 64 channels, and on
  // small grids (where rounding the pitch to 32 wastes a third of the tile), the TMA path is as fast or faster
  if (g.C != 32 || g.W < 64) return;
  const int wp = (g.W + 2 + 31) / 32 * 32, lw = (128 + 2 * wp + 2) | 1;
  const size_t slab = (size_t)lw * 16, wbytes = (slab * (g.C / 8) + 1023) & ~size_t(1023);
  int nwb = 3;
  if (win_fixed_smem_bytes(g.C, g.K) + 3 * wbytes > kWinSmemLimit) nwb = 2;
  if (win_fixed_smem_bytes(g.C, g.K) + nwb * wbytes > kWinSmemLimit) return;
  const long long tpi = cdivll((long long)p->P * wp, 128), tiles = tpi * g.N;
  if (tiles > 0x7fffffffLL) return;
  // u / pitch by a multiply-high: exact while u · pitch < 2³² (u < (P + 3)·pitch)
  if ((double)(p->P + 3) * wp * wp >= 4294967296.0) return;
  p->win = 1;
  p->win_nwb = nwb;
  p->win_mul = (unsigned)((0x100000000ull + wp - 1) / wp);
  p->win_wp = wp;
  p->win_lw = lw;
  p->win_slab = (int)slab;
  p->win_wbytes = (int)wbytes;
  p->win_tpi = (int)tpi;
  p->win_tiles = (int)tiles;
}

static int plan_init(const osam_conv_geom* g, int transposed, osam_conv_plan* p);

// Re-tile a plan for an output grid of P × Q (a dgrad sub-plan whose last taps read past dz: zero fill).
static void plan_set_output(osam_conv_plan* p, int P, int Q) {
  const osam_conv_geom& g = p->g;
  p->P = P;
  p->Q = Q;
  p->M = (long long)g.N * P * Q;
  if (p->mode == A_S1 || p->mode == A_S2) {
    choose_tile(g.N, P, Q, &p->tn, &p->th, &p->tw);
    p->tiles_q = (int)cdivll(Q, p->tw);
    p->tiles_p = (int)cdivll(P, p->th);
    p->tiles_m = (int)(p->tiles_q * (long long)p->tiles_p * cdivll(g.N, p->tn));
  } else {
    p->tiles_m = (int)cdivll(p->M, 128);
  }
  p->win = 0;
}

// Input gradient as forward convs over dz (ConvOp::dgrad, src/conv.cpp:346-355).
//  stride 1: dx = conv(dz, Wd, pad' = R − 1 − pad) with Wd[c][r'][s'][k] = W[k][R−1−r'][S−1−s'][c];
//  stride 2: output row h = 2i + ph only sees taps r ≡ ph + pad (mod 2), at dz row i + (ph + pad − r)/2 —
//  for each parity class (ph, pw) a stride-1 conv over dz with those taps (ordered by dz offset) whose
//  result lands on pixels (2i + ph, 2j + pw) of dx.
static void plan_dgrad(osam_conv_plan* p) {
  const osam_conv_geom& g = p->g;
  p->n_dg = 0;
  p->dg_direct = 0;
  if (p->transposed) {
    if (g.R != g.stride || g.S != g.stride || g.stride != 2) return;
    osam_conv_geom sg{g.N, 2 * g.H, 2 * g.W, g.K, g.C, 2, 2, 2, 0};
    osam_conv_plan* s = new (std::nothrow) osam_conv_plan;
    if (!s) return;
    if (plan_init(&sg, 0, s) != OSAM_OK || s->mode != A_S2 || s->P != g.H || s->Q != g.W) {
      delete s;
      return;
    }
    p->dg[0] = s;
    p->dg_R[0] = p->dg_S[0] = 2;
    p->dg_woff[0] = 0;
    p->dg_direct = 1;
    p->n_dg = 1;
    return;
  }
  if (g.R != g.S) return;
  auto make = [&](int i, int R2, int S2, int pad2, int P, int Q, int par) -> bool {
    osam_conv_geom sg{g.N, p->P, p->Q, g.K, g.C, R2, S2, 1, pad2};
    osam_conv_plan* s = new (std::nothrow) osam_conv_plan;
    if (!s) return false;
    if (plan_init(&sg, 0, s) != OSAM_OK || s->mode == A_STEM) {
      delete s;
      return false;
    }
    plan_set_output(s, P, Q);
    p->dg[i] = s;
    p->dg_R[i] = R2;
    p->dg_S[i] = S2;
    p->dg_par[i] = par;
    return true;
  };
  bool ok = true;
  int n = 0;
  p->dg_chunk = 0;
  if (g.stride == 1 && g.C > 512) {
    // the sub-conv's GEMM N is C: split it into equal 32-aligned slices of at most 512 channels
    int nc = (g.C + 511) / 512;
    while (nc <= 4 && (g.C % nc || (g.C / nc) % 32)) nc++;
    ok = nc <= 4 && g.R <= 8;
    const int chunk = ok ? g.C / nc : 0;
    for (int i = 0; i < nc && ok; i++) {
      osam_conv_geom sg{g.N, p->P, p->Q, g.K, chunk, g.R, g.S, 1, g.R - 1 - g.pad};
      osam_conv_plan* s = new (std::nothrow) osam_conv_plan;
      if (!s || plan_init(&sg, 0, s) != OSAM_OK || s->mode == A_STEM) {
        delete s;
        ok = false;
        break;
      }
      plan_set_output(s, g.H, g.W);
      p->dg[i] = s;
      p->dg_R[i] = g.R;
      p->dg_S[i] = g.S;
      p->dg_par[i] = 0;
      for (int r = 0; r < g.R; r++) p->dg_rmap[i][r] = g.R - 1 - r;
      for (int s2 = 0; s2 < g.S; s2++) p->dg_smap[i][s2] = g.S - 1 - s2;
    }
    if (ok) {
      p->dg_chunk = chunk;
      for (int i = 0; i < nc; i++) p->dg_woff[i] = 0;  // one re-laid-out set; slice i starts at c = chunk·i
      p->n_dg = nc;
      return;
    }
  } else if (g.stride == 1) {
    ok = g.R <= 8 && make(0, g.R, g.S, g.R - 1 - g.pad, g.H, g.W, 0);
    if (ok) {
      for (int r = 0; r < g.R; r++) p->dg_rmap[0][r] = g.R - 1 - r;
      for (int s = 0; s < g.S; s++) p->dg_smap[0][s] = g.S - 1 - s;
      n = 1;
    }
  } else if (g.stride == 2 && g.H == 2 * p->P && g.W == 2 * p->Q && g.R <= 8) {
    for (int ph = 0; ph < 2 && ok; ph++)
      for (int pw = 0; pw < 2 && ok; pw++) {
        // taps of each parity, in increasing dz offset (decreasing r)
        int rt[8], st[8], nr = 0, ns = 0;
        for (int r = g.R - 1; r >= 0; r--)
          if (((ph + g.pad - r) % 2 + 2) % 2 == 0) rt[nr++] = r;
        for (int s = g.S - 1; s >= 0; s--)
          if (((pw + g.pad - s) % 2 + 2) % 2 == 0) st[ns++] = s;
        if (nr == 0 || ns == 0) {
          ok = false;
          break;
        }
        const int orow = (ph + g.pad - rt[0]) / 2, ocol = (pw + g.pad - st[0]) / 2;
        if (orow > 0 || ocol > 0 || orow != ocol) {
          ok = false;
          break;
        }
        const int i = ph * 2 + pw;
        ok = make(i, nr, ns, -orow, p->P, p->Q, i + 1);
        for (int r = 0; r < nr && ok; r++) p->dg_rmap[i][r] = rt[r];
        for (int s = 0; s < ns && ok; s++) p->dg_smap[i][s] = st[s];
        n += ok;
      }
  } else {
    ok = false;
  }
  if (!ok) {
    for (int i = 0; i < 4; i++) {
      delete p->dg[i];
      p->dg[i] = nullptr;
    }
    return;
  }
  long long off = 0;
  for (int i = 0; i < n; i++) {
    p->dg_woff[i] = off;
    off += ((long long)g.C * p->dg_R[i] * p->dg_S[i] * g.K + 127) / 128 * 128;  // 256-byte aligned blocks
  }
  p->n_dg = n;
}

static int plan_init(const osam_conv_geom* g, int transposed, osam_conv_plan* p) {
  std::memset(p, 0, sizeof(*p));
  p->g = *g;
  p->transposed = transposed;
  if (g->N < 1 || g->H < 1 || g->W < 1 || g->C < 1 || g->K < 1 || g->R < 1 || g->S < 1 || g->stride < 1 || g->pad < 0)
    return fail(OSAM_ERR_INVALID, "invalid conv geometry");
  if (transposed) {
    if (g->R != 2 || g->S != 2 || g->stride != 2 || g->pad != 0)
      return fail(OSAM_ERR_UNSUPPORTED, "transposed conv: only kernel 2, stride 2, pad 0");
    if (g->C % 32 || g->K % 8) return fail(OSAM_ERR_UNSUPPORTED, "transposed conv: C %% 32, K %% 8 required");
    p->P = g->H;  // GEMM grid = input grid; the epilogue scatters to 2H × 2W
    p->Q = g->W;
    p->mode = A_S1;  // one "tap" (R = S = 1 view of the input), spatial tiles
    p->BK = g->C % 64 == 0 ? 64 : 32;
    p->gemm_n = 4 * g->K;
    p->M = (long long)g->N * g->H * g->W;
    p->nkc = g->C / p->BK;
    p->nk = p->nkc;
  } else {
    p->P = (g->H + 2 * g->pad - g->R) / g->stride + 1;
    p->Q = (g->W + 2 * g->pad - g->S) / g->stride + 1;
    if (p->P < 1 || p->Q < 1) return fail(OSAM_ERR_INVALID, "empty conv output");
    p->M = (long long)g->N * p->P * p->Q;
    p->gemm_n = g->K;
    if (g->R * g->S * g->C <= 32 && g->C % 32 != 0) {
      p->mode = A_STEM;
      p->BK = 32;
      p->nkc = 1;
      p->nk = 1;
      if (g->K > 64) return fail(OSAM_ERR_UNSUPPORTED, "small-C conv: K <= 64 required");
    } else {
      if (g->C % 32) return fail(OSAM_ERR_UNSUPPORTED, "conv input channels must be a multiple of 32 (C=%d)", g->C);
      p->BK = g->C % 64 == 0 ? 64 : 32;
      p->nkc = g->C / p->BK;
      p->nk = g->R * g->S * p->nkc;
      if (g->stride == 1)
        p->mode = A_S1;
      else if (g->stride == 2 && g->H % 2 == 0 && g->W % 2 == 0)
        p->mode = A_S2;
      else
        return fail(OSAM_ERR_UNSUPPORTED, "conv stride %d with H=%d W=%d", g->stride, g->H, g->W);
    }
  }
  if (p->gemm_n > 512) return fail(OSAM_ERR_UNSUPPORTED, "more than 512 GEMM output columns (%d)", p->gemm_n);
  p->BN = choose_bn(p->gemm_n);
  if (p->mode == A_STEM && p->BN > 64) return fail(OSAM_ERR_UNSUPPORTED, "small-C conv: K <= 64 required");
  p->ntn = (int)cdivll(p->gemm_n, p->BN);
  if (p->mode == A_STEM) {
    // one image per tile, th × tw = 128 output pixels; the input window must fit 48 KiB of shared memory
    long long best = -1;
    for (int tw = 128; tw >= 16; tw /= 2) {
      const int th = 128 / tw;
      const long long wbytes = (long long)((th - 1) * g->stride + g->R) * ((tw - 1) * g->stride + g->S) * g->C * 2;
      if (wbytes > 48 * 1024) continue;
      const long long cost = cdivll(p->Q, tw) * cdivll(p->P, th);
      if (best < 0 || cost < best) {
        best = cost;
        p->tw = tw;
        p->th = th;
      }
    }
    if (best < 0) return fail(OSAM_ERR_UNSUPPORTED, "small-C conv: input window too large");
    p->tn = 1;
    p->tiles_q = (int)cdivll(p->Q, p->tw);
    p->tiles_p = (int)cdivll(p->P, p->th);
    p->tiles_m = (int)(p->tiles_q * (long long)p->tiles_p * g->N);
  } else if (p->mode == A_S1 || p->mode == A_S2) {
    choose_tile(g->N, p->P, p->Q, &p->tn, &p->th, &p->tw);
    p->tiles_q = (int)cdivll(p->Q, p->tw);
    p->tiles_p = (int)cdivll(p->P, p->th);
    p->tiles_m = (int)(p->tiles_q * (long long)p->tiles_p * cdivll(g->N, p->tn));
  } else {
    p->tiles_m = (int)cdivll(p->M, 128);
  }
  if ((long long)p->tiles_m * p->ntn > 0x7fffffffLL) return fail(OSAM_ERR_UNSUPPORTED, "conv too large");
  plan_win(p);
  return OSAM_OK;
}

static int fill_dest(const osam_dest& s, int kout, DestDev* d, int transposed) {
  if (!s.p) return fail(OSAM_ERR_INVALID, "destination pointer is NULL");
  if (s.c0 < 0 || s.c1 <= s.c0 || s.c1 > kout) return fail(OSAM_ERR_INVALID, "destination channels [%d,%d)", s.c0, s.c1);
  if (s.choff < 0 || s.choff + s.c1 - s.c0 > s.ctot) return fail(OSAM_ERR_INVALID, "destination channel offset");
  if (s.up != 1 && s.up != 2) return fail(OSAM_ERR_INVALID, "destination up must be 1 or 2");
  if (transposed && s.up != 1) return fail(OSAM_ERR_INVALID, "transposed conv: up must be 1");
  d->p = static_cast<__half*>(s.p);
  d->ctot = s.ctot;
  d->choff = s.choff;
  d->c0 = s.c0;
  d->c1 = s.c1;
  d->up = s.up;
  d->vec = (s.ctot % 8 == 0 && s.choff % 8 == 0 && s.c0 % 8 == 0 && s.c1 % 8 == 0 &&
            (reinterpret_cast<uintptr_t>(s.p) & 15) == 0);
  return OSAM_OK;
}

// Planner switches, read at every plan preparation (never in graph replays); the tests force each form.
static int env_switch(const char* name) {
  const char* v = getenv(name);
  return (v && (v[0] == '0' || v[0] == '1')) ? v[0] - '0' : -1;
}

// CTA pairs with 2-SM UMMAs (conv_fprop.cu; OSAM_FPROP_PAIR=0|1 forces it).  Measured on B200 at the
// network's shapes (batch 64): with ≥ 128 output channels and ≥ 600 tiles, 3–4 % faster for the stride-2
// convs and 4–11 % for the window form (proto.cv2 0.417 → 0.372 ms: with the windows, the weight stream
// is most of what the SM loads, and a pair loads half of it); slower for 1×1 convs, 64-wide tiles and
// small grids.  A pair sums every output in the same order as a single CTA (same K sequence), so the
// choice may depend on N.
static int choose_pair(const osam_conv_plan* p, int mode) {
  if (mode != A_GEMM && mode != A_S1 && mode != A_S2 && mode != A_W3 && mode != A_W3S2) return 0;
  if ((p->BN / 2) * p->BK * 2 % 1024 != 0) return 0;  // each CTA's half of B must fill whole 1 KB atoms
  const int f = env_switch("OSAM_FPROP_PAIR");
  if (f >= 0) return f;
  return (mode == A_S2 || mode == A_W3 || mode == A_W3S2) && p->BN >= 128 && (long long)p->tiles_m * p->ntn >= 600;
}

// Column-shifted windows (A_W3) for a 3×3/s1/p1 conv.  Whether a layer takes the window form is decided
// from its grid alone (the window form sums in another order than the per-tap form, so a layer must take
// the same form at every batch size): the best spatial block th × tw (th·tw ∈ {128, 64, 32}, tw ∈
// {4, 8, 16}) pads the image by ≤ 5 %, or by ≤ 25 % when C ≤ 64 or the conv has more than 128 output
// channels (measured on B200).  The tile — th rows × tw columns × ni images, th·tw·ni = 128, tw·ni ∈
// {8, 16} — is then the one with the fewest tiles for this batch.  OSAM_FPROP_W3=0|1 forces the form (1:
// whenever the geometry allows).  Returns false when the window form is not taken.
struct W3Tile {
  int th, tw, ni;
};
static bool choose_w3(const osam_conv_plan* p, W3Tile* out) {
  const osam_conv_geom& g = p->g;
  if (p->transposed || p->mode != A_S1 || g.R != 3 || g.S != 3 || g.pad != 1 || g.stride != 1) return false;
  const int f = env_switch("OSAM_FPROP_W3");
  if (f == 0) return false;
  static const W3Tile opts[] = {{16, 8, 1}, {8, 16, 1}, {8, 8, 2}, {16, 4, 2}, {8, 4, 4}};
  long long best_sp = -1;  // padded pixels of the best spatial block, per image
  for (const W3Tile& o : opts) {
    const long long sp = cdivll(p->Q, o.tw) * o.tw * cdivll(p->P, o.th) * o.th;
    if (best_sp < 0 || sp < best_sp) best_sp = sp;
  }
  const long long area = (long long)p->P * p->Q;
  const bool take = f == 1 || best_sp * 100 <= area * 105 ||
                    (best_sp * 100 <= area * 125 && (g.C <= 64 || p->BN > 128));
  if (!take) return false;
  long long best = -1;
  for (const W3Tile& o : opts) {
    const long long tiles = cdivll(p->Q, o.tw) * cdivll(p->P, o.th) * cdivll(g.N, o.ni);
    if (best < 0 || tiles < best) {
      best = tiles;
      *out = o;
    }
  }
  return true;
}

// Stride-2 window form (A_W3S2) for a 3×3/s2/p1 conv whose output grid tiles into 16 × 8 blocks exactly,
// by default only where the weights can stay resident (one channel chunk, BN ≤ 64: model.1, 0.173 →
// 0.106 ms at batch 64; streamed, the 64 → 128 conv measured 1 % slower than the per-tap form).
// OSAM_FPROP_W3S2=0|1 forces it (1: any grid, ragged tiles zero-filled).
static bool choose_w3s2(const osam_conv_plan* p) {
  const osam_conv_geom& g = p->g;
  if (p->transposed || p->mode != A_S2 || g.R != 3 || g.S != 3 || g.pad != 1 || g.stride != 2) return false;
  if (p->BN != 32 && p->BN != 64 && p->BN != 128) return false;  // the instantiated widths
  const int f = env_switch("OSAM_FPROP_W3S2");
  if (f >= 0) return f == 1;
  return p->P % 16 == 0 && p->Q % 8 == 0 && g.C == p->BK && p->ntn == 1 && p->BN <= 64;
}

static int conv_prepare_launch(const osam_conv_plan* p, const void* x, const void* w, const osam_epilogue* ep,
                               float beta, void* y, void* ws, size_t ws_bytes, ConvLaunch* L, bool w_gemm_ready,
                               int* err_word, int par, int y_ctot, int y_choff);

int conv_prepare(const osam_conv_plan* p, const void* x, const void* w, const osam_epilogue* ep, float beta, void* y,
                 void* ws, size_t ws_bytes, ConvLaunch* L, bool w_gemm_ready, int* err_word, int par, int y_ctot,
                 int y_choff) {
  const int rc = conv_prepare_launch(p, x, w, ep, beta, y, ws, ws_bytes, L, w_gemm_ready, err_word, par, y_ctot,
                                     y_choff);
  if (rc == OSAM_OK) {  // the kernels' divisors, once the tile shape is final
    ConvDev& d = L->d;
    d.f_ntn.set(d.ntn);
    d.f_tq.set(d.tiles_q);
    d.f_tp.set(d.tiles_p);
    d.f_tw.set(d.tw);
    d.f_nw.set(d.tn * d.tw);
    d.f_thw.set(d.th * d.tw);
    d.f_nkc.set(d.nkc);
    d.f_S.set(d.S);
  }
  return rc;
}

static int conv_prepare_launch(const osam_conv_plan* p, const void* x, const void* w, const osam_epilogue* ep,
                               float beta, void* y, void* ws, size_t ws_bytes, ConvLaunch* L, bool w_gemm_ready,
                               int* err_word, int par, int y_ctot, int y_choff) {
  if (!p || !x || !w) return fail(OSAM_ERR_INVALID, "NULL plan or operand");
  const osam_conv_geom& g = p->g;
  *L = ConvLaunch{};
  L->BK = p->BK;
  L->BN = p->BN;
  L->mode = p->mode;
  L->pair = 0;
  L->grid = p->tiles_m * p->ntn;
  ConvDev& d = L->d;
  d.N = g.N; d.H = g.H; d.W = g.W; d.C = g.C; d.K = g.K;
  d.P = p->P; d.Q = p->Q; d.R = g.R; d.S = g.S; d.stride = g.stride; d.pad = g.pad;
  if (p->transposed) {  // a single tap at offset 0 over the input grid
    d.R = 1;
    d.S = 1;
    d.pad = 0;
  }
  d.gemm_n = p->gemm_n;
  d.tn = p->tn; d.th = p->th; d.tw = p->tw; d.tiles_q = p->tiles_q; d.tiles_p = p->tiles_p;
  d.M = p->M;
  d.ntn = p->ntn;
  d.tiles_m = p->tiles_m;
  d.nkc = p->nkc;
  d.nk = p->nk;
  d.err = err_word ? err_word : device_error_word();
  if (!d.err) return fail(OSAM_ERR_CUDA, "cannot allocate the device error word");

  // ---- epilogue
  EpiDev& e = d.ep;
  e.shuffle = p->transposed;
  e.kout = g.K;
  e.par = par;
  if (par && p->mode == A_STEM) return fail(OSAM_ERR_UNSUPPORTED, "parity placement on the small-C path");
  if (!ep) {
    if (!y) return fail(OSAM_ERR_INVALID, "NULL output");
    e.kind = OSAM_EPI_STORE;
    e.beta = beta;
    e.ndest = 1;
    osam_dest o{y, y_ctot > 0 ? y_ctot : g.K, y_ctot > 0 ? y_choff : 0, 0, g.K, 1};
    int rc = fill_dest(o, g.K, &e.dest[0], p->transposed);
    if (rc) return rc;
  } else {
    if (ep->kind < 0 || ep->kind > 2) return fail(OSAM_ERR_INVALID, "epilogue kind %d", ep->kind);
    if (ep->n_dest < 1 || ep->n_dest > OSAM_MAX_DEST) return fail(OSAM_ERR_INVALID, "n_dest %d", ep->n_dest);
    if (ep->kind == OSAM_EPI_BN_ACT && (!ep->scale || !ep->shift)) return fail(OSAM_ERR_INVALID, "BN epilogue needs scale/shift");
    if (ep->kind == OSAM_EPI_BIAS && !ep->bias) return fail(OSAM_ERR_INVALID, "bias epilogue needs bias");
    if (ep->res && p->transposed) return fail(OSAM_ERR_INVALID, "transposed conv: no residual");
    if (ep->res && (reinterpret_cast<uintptr_t>(ep->res) & 15)) return fail(OSAM_ERR_INVALID, "residual not 16-byte aligned");
    e.kind = ep->kind;
    e.scale = ep->scale;
    e.shift = ep->shift;
    e.bias = ep->bias;
    e.res = static_cast<const __half*>(ep->res);
    e.act = ep->act;
    e.round_z = ep->round_z;
    e.beta = 0.f;
    e.ndest = ep->n_dest;
    for (int i = 0; i < ep->n_dest; i++) {
      int rc = fill_dest(ep->dest[i], g.K, &e.dest[i], p->transposed);
      if (rc) return rc;
    }
  }

  // ---- warp-cooperative epilogue: every destination 8-channel aligned, tiles fully inside the GEMM N
  {
    // beta ≠ 0 (an input gradient added to what is there): one plain destination, its old rows read
    // coalesced through the stage like a residual (not with the TMA-store epilogue)
    bool coop = (p->gemm_n % p->BN == 0) && (p->BN % 16 == 0) &&
                (e.beta == 0.f || (e.ndest == 1 && e.dest[0].up == 1 && !e.shuffle));
    for (int i = 0; i < e.ndest; i++) coop = coop && e.dest[i].vec;
    if (e.shuffle) coop = coop && (e.kout % 32 == 0);
    if (e.res) coop = coop && (g.K % 8 == 0);
    if (p->mode == A_STEM) coop = coop && (p->BN == 32 || p->BN == 16 || p->BN == 64);
    if (p->mode != A_STEM && p->mode != A_GEMM) coop = coop && (p->P < 65536 && p->Q < 65536);
    e.coop = coop;
  }
  // ---- narrow 3×3 convs: one shared input window per tile (TMA-store epilogue, one output row per warp)
  // the window form of the tensor-map kernel (A_W3) is faster than conv_win.cu where both apply (measured:
  // 160² 32 → 32 0.117 vs 0.143 ms, 80² 0.033 vs 0.037 ms at batch 64)
  W3Tile w3t{};
  bool win = p->win && e.coop && e.beta == 0.f && !e.shuffle && !e.par && env_switch("OSAM_FPROP_WIN") != 0 &&
             !choose_w3(p, &w3t);
  for (int i = 0; i < e.ndest && win; i++) win = e.dest[i].c0 % 32 == 0 && e.dest[i].c1 % 32 == 0;
  if (win) {
    L->mode = A_WIN;
    d.tn = 1;
    d.th = 1;
    d.tw = 32;
    d.win_nwb = p->win_nwb;
    d.win_mul = p->win_mul;
    L->x = static_cast<const __half*>(x);
    d.win_wp = p->win_wp;
    d.win_lw = p->win_lw;
    d.win_slab = p->win_slab;
    d.win_wbytes = p->win_wbytes;
    d.win_tpi = p->win_tpi;
    d.tiles_m = p->win_tiles;
    d.ntn = 1;
    L->grid = p->win_tiles;
  }
  if (L->mode == A_S1) {
    if (choose_w3(p, &w3t)) {
      L->mode = A_W3;
      d.tn = w3t.ni;
      d.tw = w3t.tw;
      d.th = w3t.th;
      d.tiles_q = (int)cdivll(p->Q, d.tw);
      d.tiles_p = (int)cdivll(p->P, d.th);
      d.tiles_m = (int)((long long)d.tiles_q * d.tiles_p * cdivll(g.N, d.tn));
      L->grid = d.tiles_m * p->ntn;
    }
  } else if (L->mode == A_S2 && choose_w3s2(p)) {
    L->mode = A_W3S2;
    d.tn = 1;
    d.tw = 8;
    d.th = 16;
    d.tiles_q = (int)cdivll(p->Q, 8);
    d.tiles_p = (int)cdivll(p->P, 16);
    d.tiles_m = (int)((long long)d.tiles_q * d.tiles_p * g.N);
    L->grid = d.tiles_m * p->ntn;
  }
  // ---- TMA-store epilogue: spatial tiles, 32-column passes, destinations on 32-column boundaries
  {
    bool ts = e.coop && e.beta == 0.f && (L->mode == A_WIN || p->mode == A_S1 || p->mode == A_S2) && p->BN % 32 == 0;
    for (int i = 0; i < e.ndest && ts; i++) ts = e.dest[i].c0 % 32 == 0 && e.dest[i].c1 % 32 == 0;
    if (e.shuffle) ts = ts && e.ndest == 1 && e.kout % 32 == 0;
    if (e.par) ts = ts && e.ndest == 1;
    e.tstore = 0;
    if (ts) {
      // A_W3: (C, Q, N, P) views (a warp's rows run row, image, column): box {32, tw, ni, 32 / (ni·tw)}
      const bool w3 = mode_window(L->mode);
      e.wtw = d.tw < 32 ? d.tw : 32;
      e.wth = d.th < 32 / e.wtw ? d.th : 32 / e.wtw;
      e.wtn = 32 / (e.wtw * e.wth);
      if (w3) {
        e.wtw = d.tw;
        e.wtn = d.tn;
        e.wth = 32 / (d.tw * d.tn);
      }
      const uint32_t box[4] = {32, (uint32_t)e.wtw, (uint32_t)(w3 ? e.wtn : e.wth), (uint32_t)(w3 ? e.wth : e.wtn)};
      int rc = OSAM_OK;
      for (int t = 0; t < e.ndest && rc == OSAM_OK; t++) {
        const DestDev& ds = e.dest[t];
        const uint64_t c = (uint64_t)ds.ctot;
        const bool four = ds.up == 2 || e.shuffle || e.par;
        const uint64_t OQ2 = 2ull * p->Q, OP2 = 2ull * p->P;
        for (int v = 0; v < (four ? 4 : 1) && rc == OSAM_OK; v++) {
          const int dy = v >> 1, dx = v & 1;
          const __half* b = ds.p + (four ? ((uint64_t)dy * OQ2 + dx) * c : 0);
          uint64_t dims[4] = {c, (uint64_t)p->Q, (uint64_t)p->P, (uint64_t)g.N};
          uint64_t str[3];
          if (four) {
            str[0] = 2 * c * 2;
            str[1] = 2 * OQ2 * c * 2;
            str[2] = OP2 * OQ2 * c * 2;
          } else {
            str[0] = c * 2;
            str[1] = (uint64_t)p->Q * c * 2;
            str[2] = (uint64_t)p->P * p->Q * c * 2;
          }
          if (w3) {  // (C, Q, N, P)
            std::swap(dims[2], dims[3]);
            std::swap(str[1], str[2]);
          }
          rc = make_map(&L->sm.m[4 * t + v], b, 4, dims, str, box, 64);
        }
      }
      if (rc != OSAM_OK) return rc;
      e.tstore = 1;
    }
  }

  // ---- operands
  const int row_bytes = p->BK * 2;
  if (p->mode == A_STEM) {
    L->x = static_cast<const __half*>(x);
    L->w = static_cast<const __half*>(w);
    // Pipelined RGB stem: 3×3/s2/p1, C = 3, K = 32, 2 × 64-pixel tiles, all destinations TMA-storable.
    bool rgb = g.R == 3 && g.S == 3 && g.C == 3 && g.stride == 2 && g.pad == 1 && g.K == 32 && p->Q % 64 == 0 &&
               p->P % 2 == 0 && e.coop && !e.res && !e.shuffle && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
               ((size_t)g.W * 3 * 2) % 16 == 0;
    for (int i = 0; i < e.ndest && rgb; i++) rgb = e.dest[i].c0 % 16 == 0 && e.dest[i].c1 % 16 == 0;
    if (rgb) {
      d.th = 2;
      d.tw = 64;
      d.tn = 1;
      d.tiles_q = p->Q / 64;
      d.tiles_p = p->P / 2;
      d.tiles_m = d.tiles_q * d.tiles_p * g.N;
      const uint64_t dims[3] = {(uint64_t)g.W * 3, (uint64_t)g.H, (uint64_t)g.N};
      const uint64_t str[2] = {(uint64_t)g.W * 3 * 2, (uint64_t)g.H * g.W * 3 * 2};
      const uint32_t box[3] = {208, 5, 1};
      int rc = make_map(&L->ta, x, 3, dims, str, box, 0);
      if (rc) return rc;
      const uint32_t sbox[4] = {16, 32, 1, 1};  // one epilogue warp: 16 channels × 32 pixels, unswizzled
      for (int t = 0; t < e.ndest && rc == OSAM_OK; t++) {
        const DestDev& ds = e.dest[t];
        const uint64_t c = (uint64_t)ds.ctot;
        const bool four = ds.up == 2;
        const uint64_t OQ2 = 2ull * p->Q, OP2 = 2ull * p->P;
        for (int v = 0; v < (four ? 4 : 1) && rc == OSAM_OK; v++) {
          const __half* b = ds.p + (four ? ((uint64_t)(v >> 1) * OQ2 + (v & 1)) * c : 0);
          const uint64_t sd[4] = {c, (uint64_t)p->Q, (uint64_t)p->P, (uint64_t)g.N};
          uint64_t ss[3];
          if (four) {
            ss[0] = 2 * c * 2;
            ss[1] = 2 * OQ2 * c * 2;
            ss[2] = OP2 * OQ2 * c * 2;
          } else {
            ss[0] = c * 2;
            ss[1] = (uint64_t)p->Q * c * 2;
            ss[2] = (uint64_t)p->P * p->Q * c * 2;
          }
          rc = make_map(&L->sm.m[4 * t + v], b, 4, sd, ss, sbox, 0);
        }
      }
      if (rc) return rc;
      e.tstore = 1;
      L->stem_rgb = 1;
    }
    return OSAM_OK;
  }
  int rc;
  L->pair = choose_pair(p, L->mode);
  // Narrow window-form layers keep all nine weight taps in shared memory (A_W3R): one channel chunk, one
  // N tile, BN ≤ 64; the 64 × 64 taps (72 KB) fit beside the windows only as a CTA pair's halves.
  // Measured on B200 (batch 64): 32 → 32 at 160² 0.106 → 0.065 ms, at 80² 0.030 → 0.019 ms; 64 → 64 at
  // 80² 4–5 % faster; on small grids the once-per-CTA weight load does not pay (−4 %), hence the tile
  // thresholds.  OSAM_FPROP_W3R=0|1 forces it (1: whenever the geometry allows).
  // The stride-2 window form takes resident weights under the same conditions (A_W3S2R).
  const int w3r_env = env_switch("OSAM_FPROP_W3R");
  const long long w3_tiles = (long long)d.tiles_m * p->ntn;
  if ((L->mode == A_W3 || L->mode == A_W3S2) && w3r_env != 0 && p->ntn == 1 && g.C == p->BK &&
      (p->BN == 32 || p->BN == 64) && (w3r_env == 1 || w3_tiles >= (p->BN == 32 ? 600 : 1600))) {
    // the nine taps (this CTA's rows) and two windows within the 96 KB ring of a two-CTA-per-SM kernel
    const long long win = (L->mode == A_W3S2 ? 272 : 160) * 2LL * p->BK;
    auto fits = [&](int pair) { return 9LL * (pair ? p->BN / 2 : p->BN) * 2 * p->BK + 2 * win <= 96 * 1024; };
    bool ok = fits(L->pair);
    if (!ok && !L->pair && env_switch("OSAM_FPROP_PAIR") != 0 && fits(1)) {
      L->pair = 1;
      ok = true;
    }
    if (ok) L->mode = L->mode == A_W3 ? A_W3R : A_W3S2R;
  }
  const uint32_t b_rows = (uint32_t)(L->pair ? p->BN / 2 : p->BN);  // weight rows per CTA
  if (p->mode == A_GEMM) {
    const uint64_t dims[2] = {(uint64_t)g.C, (uint64_t)p->M};
    const uint64_t str[1] = {(uint64_t)g.C * 2};
    const uint32_t box[2] = {(uint32_t)p->BK, 128};
    rc = make_map(&L->ta, x, 2, dims, str, box, row_bytes);
  } else if (p->mode == A_S1) {
    const uint64_t dims[4] = {(uint64_t)g.C, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)g.N};
    const uint64_t str[3] = {(uint64_t)g.C * 2, (uint64_t)g.W * g.C * 2, (uint64_t)g.H * g.W * g.C * 2};
    if (L->mode == A_W3 || L->mode == A_W3R) {  // one (th + 2)-row × ni-image × tw-column window per box,
                                                // a (C, W, N, H) view
      const uint64_t wdims[4] = {(uint64_t)g.C, (uint64_t)g.W, (uint64_t)g.N, (uint64_t)g.H};
      const uint64_t wstr[3] = {str[0], str[2], str[1]};
      const uint32_t box[4] = {(uint32_t)p->BK, (uint32_t)d.tw, (uint32_t)d.tn, (uint32_t)(d.th + 2)};
      rc = make_map(&L->ta, x, 4, wdims, wstr, box, row_bytes);
    } else {  // the th × tw × tn tile of one tap
      const uint32_t box[4] = {(uint32_t)p->BK, (uint32_t)p->tw, (uint32_t)p->th, (uint32_t)p->tn};
      rc = make_map(&L->ta, x, 4, dims, str, box, row_bytes);
    }
  } else {
    const uint64_t dims[5] = {(uint64_t)2 * g.C, (uint64_t)g.W / 2, 2, (uint64_t)g.H / 2, (uint64_t)g.N};
    const uint64_t str[4] = {(uint64_t)4 * g.C, (uint64_t)g.W * g.C * 2, (uint64_t)2 * g.W * g.C * 2,
                             (uint64_t)g.H * g.W * g.C * 2};
    // stride-2 window form: 8 columns × both row parities × 17 row pairs of one image per box
    const bool s2w = mode_s2_window(L->mode);
    const uint32_t box[5] = {(uint32_t)p->BK, (uint32_t)(s2w ? 8 : p->tw), s2w ? 2u : 1u,
                             (uint32_t)(s2w ? 17 : p->th), (uint32_t)(s2w ? 1 : p->tn)};
    rc = make_map(&L->ta, x, 5, dims, str, box, row_bytes);
  }
  if (rc) return rc;

  const void* wb = w;
  if (p->transposed && !w_gemm_ready) {
    const size_t need = (size_t)g.C * 4 * g.K * 2;
    if (!ws || ws_bytes < need) return fail(OSAM_ERR_INVALID, "transposed conv needs %zu workspace bytes", need);
    L->wt_src = static_cast<const __half*>(w);
    L->wt_dst = static_cast<__half*>(ws);
    wb = ws;
  }
  if (p->transposed) {
    const uint64_t dims[2] = {(uint64_t)g.C, (uint64_t)4 * g.K};
    const uint64_t str[1] = {(uint64_t)g.C * 2};
    const uint32_t box[2] = {(uint32_t)p->BK, b_rows};
    rc = make_map(&L->tb, wb, 2, dims, str, box, row_bytes);
  } else {
    const uint64_t rsc = (uint64_t)g.R * g.S * g.C;
    const uint64_t dims[2] = {rsc, (uint64_t)g.K};
    const uint64_t str[1] = {rsc * 2};
    const uint32_t box[2] = {(uint32_t)p->BK, b_rows};
    rc = make_map(&L->tb, wb, 2, dims, str, box, row_bytes);
  }
  return rc;
}

cudaError_t conv_launch(const ConvLaunch& L, cudaStream_t st) {
  if (L.mode == A_STEM) return L.stem_rgb ? launch_conv_stem_rgb(L, st) : launch_conv_stem(L.x, L.w, L.d, L.BN, st);
  if (L.wt_src) {
    cudaError_t e = launch_convt_weight_relayout(L.wt_src, L.wt_dst, L.d.C, 4, L.d.K, st);
    if (e != cudaSuccess) return e;
  }
  if (L.mode == A_WIN) return launch_conv_win(L, st);
  return launch_conv_fprop(L, st);
}

cudaError_t conv_prime(const ConvLaunch& L) {
  if (L.mode == A_STEM) return cudaSuccess;
  if (L.mode == A_WIN) return launch_conv_win(L, nullptr, true);
  return launch_conv_fprop(L, nullptr, true);
}

}  // namespace osam

using namespace osam;

extern "C" {

int osam_conv_plan_create(const osam_conv_geom* g, int transposed, osam_conv_plan** out) {
  if (!g || !out) return fail(OSAM_ERR_INVALID, "NULL argument");
  *out = nullptr;
  osam_conv_plan* p = new (std::nothrow) osam_conv_plan;
  if (!p) return fail(OSAM_ERR_NOMEM, "out of host memory");
  int rc = plan_init(g, transposed, p);
  if (rc) {
    delete p;
    return rc;
  }
  // the host-mapped error word exists from the first plan on (allocated here, never inside a launch)
  if ((rc = error_word_init()) != OSAM_OK || !device_error_word()) {
    delete p;
    return rc ? rc : fail(OSAM_ERR_CUDA, "no device error word");
  }
  plan_dgrad(p);
  *out = p;
  return OSAM_OK;
}

int osam_conv_plan_destroy(osam_conv_plan* p) {
  if (p)
    for (int i = 0; i < 4; i++) delete p->dg[i];
  delete p;
  return OSAM_OK;
}

static size_t dgrad_workspace_bytes(const osam_conv_plan* p) {
  if (p->dg_direct) return 0;
  if (p->dg_chunk) return ((size_t)p->g.C * p->g.R * p->g.S * p->g.K * 2 + 255) & ~size_t(255);
  size_t b = 0;
  for (int i = 0; i < p->n_dg; i++)
    b = (size_t)p->dg_woff[i] * 2 + (((size_t)p->g.C * p->dg_R[i] * p->dg_S[i] * p->g.K * 2 + 255) & ~size_t(255));
  return b;
}

int osam_conv_dgrad(const osam_conv_plan* p, const void* dz, const void* w, void* dx, float beta, void* ws,
                    size_t ws_bytes, osam_stream_t stream) {
  return conv_dgrad_ex(p, dz, w, dx, beta, ws, ws_bytes, reinterpret_cast<cudaStream_t>(stream), nullptr);
}

}  // extern "C"

namespace osam {
size_t dgrad_prelaid_bytes(const osam_conv_plan* p) {
  const osam_conv_geom& g = p->g;
  if (!p || p->dg_direct || p->n_dg == 0) return 0;
  if (p->dg_chunk) return ((size_t)g.C * g.R * g.S * g.K * 2 + 255) & ~size_t(255);
  return dgrad_workspace_bytes(p);
}

int dgrad_jobs(const osam_conv_plan* p, const __half* w, __half* prelaid, DgradJob* out) {
  if (!p || p->dg_direct || p->n_dg == 0) return 0;
  const osam_conv_geom& g = p->g;
  const int n = p->dg_chunk ? 1 : p->n_dg;
  for (int i = 0; i < n; i++) {
    DgradJob& j = out[i];
    j.w = w;
    j.dst = prelaid + p->dg_woff[i];
    j.K = g.K;
    j.R = g.R;
    j.S = g.S;
    j.C = g.C;
    j.Rs = p->dg_chunk ? g.R : p->dg_R[i];
    j.Ss = p->dg_chunk ? g.S : p->dg_S[i];
    for (int q = 0; q < 8; q++) {
      j.r[q] = q < j.Rs ? p->dg_rmap[i][q] : 0;
      j.s[q] = q < j.Ss ? p->dg_smap[i][q] : 0;
    }
    j.n = (long long)g.C * j.Rs * j.Ss * g.K;
  }
  return n;
}

int conv_dgrad_ex(const osam_conv_plan* p, const void* dz, const void* w, void* dx, float beta, void* ws,
                  size_t ws_bytes, cudaStream_t st_in, const __half* prelaid) {
  const osam_stream_t stream = reinterpret_cast<osam_stream_t>(st_in);
  if (!p || !dz || !w || !dx) return fail(OSAM_ERR_INVALID, "NULL plan or operand");
  const osam_conv_geom& g1 = p->g;
  if (!p->transposed && g1.K == 1 && g1.R == 1 && g1.S == 1 && g1.stride == 1 && g1.pad == 0 && g1.C % 8 == 0) {
    if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(dx)) & 15)
      return fail(OSAM_ERR_INVALID, "dgrad: w and dx must be 16-byte aligned");
    cudaError_t e = launch_dgrad_k1(static_cast<const __half*>(dz), static_cast<const __half*>(w),
                                    static_cast<__half*>(dx), p->M, g1.C, beta, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? OSAM_OK : cuda_fail(e, "osam_conv_dgrad (K = 1) launch");
  }
  if (p->n_dg == 0) return fail(OSAM_ERR_UNSUPPORTED, "dgrad: geometry not supported (stride, kernel or channels)");
  const size_t need = prelaid ? 0 : dgrad_workspace_bytes(p);
  if (need && (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255)))
    return fail(OSAM_ERR_INVALID, "dgrad needs %zu workspace bytes (256-byte aligned)", need);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p->dg_direct) {  // transposed conv: a stride-2 2×2 forward conv over dy with the same weight array
    ConvLaunch L;
    int rc = conv_prepare(p->dg[0], dz, w, nullptr, beta, dx, nullptr, 0, &L);
    if (rc) return rc;
    cudaError_t e = conv_launch(L, st);
    return e == cudaSuccess ? OSAM_OK : cuda_fail(e, "osam_conv_dgrad (transposed) launch");
  }
  const osam_conv_geom& g = p->g;
  __half* wsub = prelaid ? const_cast<__half*>(prelaid) : static_cast<__half*>(ws);
  if (p->dg_chunk) {  // one weight re-layout, then one sub-conv per slice of dx's channels
    cudaError_t e = prelaid ? cudaSuccess
                            : launch_dgrad_weights(static_cast<const __half*>(w), wsub, g.K, g.R, g.S, g.C, g.R, g.S,
                                                   p->dg_rmap[0], p->dg_smap[0], st);
    if (e != cudaSuccess) return cuda_fail(e, "osam_conv_dgrad weight re-layout");
    for (int i = 0; i < p->n_dg; i++) {
      ConvLaunch L;
      const int c0 = p->dg_chunk * i;
      int rc = conv_prepare(p->dg[i], dz, wsub + (size_t)c0 * g.R * g.S * g.K, nullptr, beta, dx, nullptr, 0, &L, false,
                            nullptr, 0, g.C, c0);
      if (rc) return rc;
      e = conv_launch(L, st);
      if (e != cudaSuccess) return cuda_fail(e, "osam_conv_dgrad launch");
    }
    return OSAM_OK;
  }
  for (int i = 0; i < p->n_dg && !prelaid; i++) {
    cudaError_t e = launch_dgrad_weights(static_cast<const __half*>(w), wsub + p->dg_woff[i], g.K, g.R, g.S, g.C,
                                         p->dg_R[i], p->dg_S[i], p->dg_rmap[i], p->dg_smap[i], st);
    if (e != cudaSuccess) return cuda_fail(e, "osam_conv_dgrad weight re-layout");
  }
  for (int i = 0; i < p->n_dg; i++) {
    ConvLaunch L;
    int rc = conv_prepare(p->dg[i], dz, wsub + p->dg_woff[i], nullptr, beta, dx, nullptr, 0, &L, false, nullptr,
                          p->dg_par[i]);
    if (rc) return rc;
    cudaError_t e = conv_launch(L, st);
    if (e != cudaSuccess) return cuda_fail(e, "osam_conv_dgrad launch");
  }
  return OSAM_OK;
}

}  // namespace osam

extern "C" {

static size_t wgrad_workspace_bytes(const osam_conv_plan* p) {
  const osam_conv_geom& g = p->g;
  return ((size_t)g.K * g.R * g.S * g.C * 4 + 255) & ~size_t(255);
}

static int sm_count() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

// Weight gradient of a small-C plan (R·S·C ≤ 32, the RGB stem): patch-gather tcgen05 kernel over runs of
// 128 consecutive output pixels (conv_wgrad.cu), one CTA pair per SM.
static int wgrad_stem(const osam_conv_plan* p, const void* x, const void* dz, void* dw, float* dw32, float beta,
                      void* ws, size_t ws_bytes, osam_stream_t stream, bool direct) {
  const osam_conv_geom& g = p->g;
  if (g.K != 32 && g.K != 64) return fail(OSAM_ERR_UNSUPPORTED, "small-C wgrad: K must be 32 or 64 (K=%d)", g.K);
  const size_t need = wgrad_workspace_bytes(p);
  if (!direct && (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255)))
    return fail(OSAM_ERR_INVALID, "wgrad needs %zu workspace bytes (256-byte aligned)", need);
  if ((reinterpret_cast<uintptr_t>(dz) & 15) || (reinterpret_cast<uintptr_t>(x) & 1))
    return fail(OSAM_ERR_INVALID, "wgrad: dz must be 16-byte aligned, x 2-byte aligned");
  if (p->M >= (1LL << 31) - 128) return fail(OSAM_ERR_UNSUPPORTED, "small-C wgrad: too many output pixels");
  WgradLaunch L{};
  ConvDev& d = L.d;
  d.N = g.N; d.H = g.H; d.W = g.W; d.C = g.C; d.K = g.K;
  d.P = p->P; d.Q = p->Q; d.R = g.R; d.S = g.S; d.stride = g.stride; d.pad = g.pad;
  d.M = p->M;
  d.err = device_error_word();
  if (!d.err) return fail(OSAM_ERR_CUDA, "cannot allocate the device error word");
  L.mode = A_STEM;
  L.xp = static_cast<const __half*>(x);
  L.direct = direct;
  L.acc = direct ? dw32 : static_cast<float*>(ws);
  L.dw = static_cast<__half*>(dw);
  L.dw32 = dw32;
  L.n_out = (long long)g.K * g.R * g.S * g.C;
  L.beta = beta;
  {
    const uint64_t dims[2] = {(uint64_t)g.K, (uint64_t)p->M};
    const uint64_t str[1] = {(uint64_t)g.K * 2};
    const uint32_t box[2] = {(uint32_t)g.K, 128};
    const int rc = make_map(&L.tdz, dz, 2, dims, str, box, g.K * 2);
    if (rc) return rc;
  }
  const long long tiles = (p->M + 127) / 128;
  const long long ctas = std::min<long long>(tiles, 2LL * sm_count());
  L.tiles_per_split = (int)((tiles + ctas - 1) / ctas);
  L.grid = (int)((tiles + L.tiles_per_split - 1) / L.tiles_per_split);
  cudaError_t e = launch_conv_wgrad(L, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSAM_OK : cuda_fail(e, "osam_conv_wgrad (small-C) launch");
}

size_t osam_conv_workspace_size(const osam_conv_plan* p) {
  if (!p) return 0;
  if (p->transposed) {
    const size_t relayout = ((size_t)p->g.C * 4 * p->g.K * 2 + 255) & ~size_t(255);
    return p->dg_direct ? std::max(relayout, wgrad_workspace_bytes(p->dg[0])) : relayout;
  }
  return std::max(dgrad_workspace_bytes(p), wgrad_workspace_bytes(p));
}

static int wgrad_impl(const osam_conv_plan* p, const void* x, const void* dz, void* dw, float* dw32, float beta,
                      void* ws, size_t ws_bytes, osam_stream_t stream, bool direct = false);

int osam_conv_wgrad(const osam_conv_plan* p, const void* x, const void* dz, void* dw, float beta, void* ws,
                    size_t ws_bytes, osam_stream_t stream) {
  if (!dw) return fail(OSAM_ERR_INVALID, "NULL plan or operand");
  return wgrad_impl(p, x, dz, dw, nullptr, beta, ws, ws_bytes, stream);
}

}  // extern "C"

namespace osam {
int conv_wgrad_f32(const osam_conv_plan* p, const void* x, const void* dz, float* dw32, float beta, void* ws,
                   size_t ws_bytes, cudaStream_t st, bool direct) {
  if (!dw32) return fail(OSAM_ERR_INVALID, "NULL fp32 weight-gradient output");
  if (direct && beta != 0.f) return fail(OSAM_ERR_INVALID, "direct weight gradient with beta");
  return wgrad_impl(p, x, dz, nullptr, dw32, beta, ws, ws_bytes, reinterpret_cast<osam_stream_t>(st), direct);
}
}  // namespace osam

extern "C" {

// Window form of the weight gradient (conv_wgrad.cu, k_conv_wgrad_win): 3×3 / pad-1 convs with 32 or 64
// input channels, stride 1 or 2 (even input sizes); returns the dz channels per CTA (GEMM N block), or 0
// when the per-tap form runs.  OSAM_WGRAD_WIN=0 turns it off.
static int wgrad_window_nb(const osam_conv_plan* p) {
  const osam_conv_geom& g = p->g;
  if (p->transposed || g.R != 3 || g.S != 3 || g.pad != 1 || (g.C != 32 && g.C != 64)) return 0;
  if (!(p->mode == A_S1 && g.stride == 1) && !(p->mode == A_S2 && g.stride == 2 && g.H % 2 == 0 && g.W % 2 == 0))
    return 0;
  if (env_switch("OSAM_WGRAD_WIN") == 0) return 0;
  for (int nb : {64, 32})
    if (g.K % nb == 0 && wgrad_win_supported(g.C / 32, nb)) return nb;
  return 0;
}

// 128-pixel tile of the stride-1 window form: th rows × ni images × tw columns with ni·tw ∈ {8, 16} (so a
// row tap is a whole number of 512-byte swizzle atoms), the least padded work and halo.
static void choose_wgrad_window_tile(int N, int P, int Q, int* tn, int* th, int* tw) {
  double best = -1.0;
  for (int rows : {8, 16})
    for (int w = 16; w >= 2; w /= 2) {
      if (w > rows || rows / w > N) continue;
      const int n = rows / w, h = 128 / rows;
      const double cost = (double)cdivll(Q, w) * cdivll(P, h) * cdivll(N, n) * (h + 2) / h;
      if (best < 0 || cost < best - 1e-9) {
        best = cost;
        *tn = n;
        *th = h;
        *tw = w;
      }
    }
}

static int wgrad_window(const osam_conv_plan* p, const void* x, const void* dz, WgradLaunch& L, int NB,
                        osam_stream_t stream) {
  const osam_conv_geom& g = p->g;
  ConvDev& d = L.d;
  const bool s2 = g.stride == 2;
  L.win = 1;
  L.CB = g.C / 32;
  L.NB = NB;
  if (s2) {
    d.tn = 1;
    d.th = 16;
    d.tw = 8;
  } else {
    choose_wgrad_window_tile(g.N, p->P, p->Q, &d.tn, &d.th, &d.tw);
  }
  d.tiles_q = (int)cdivll(p->Q, d.tw);
  d.tiles_p = (int)cdivll(p->P, d.th);
  const long long tiles = (long long)d.tiles_q * d.tiles_p * cdivll(g.N, d.tn);
  if (tiles > 0x7fffffffLL) return fail(OSAM_ERR_UNSUPPORTED, "wgrad: too many tiles");
  d.tiles_m = (int)tiles;
  L.win_bytes = s2 ? 32 * 2 * 8 * 2 * 17 : 32 * 2 * d.tw * d.tn * (d.th + 2);
  const int dz_ch = NB >= 64 ? 64 : 32;
  int rc;
  {  // dz as (K, Q, N, P): the tile's pixel rows run (row, image, column)
    const uint64_t dims[4] = {(uint64_t)g.K, (uint64_t)p->Q, (uint64_t)g.N, (uint64_t)p->P};
    const uint64_t str[3] = {(uint64_t)g.K * 2, (uint64_t)p->P * p->Q * g.K * 2, (uint64_t)p->Q * g.K * 2};
    const uint32_t box[4] = {(uint32_t)dz_ch, (uint32_t)d.tw, (uint32_t)d.tn, (uint32_t)d.th};
    rc = make_map(&L.tdz, dz, 4, dims, str, box, dz_ch * 2);
  }
  if (rc == OSAM_OK && !s2) {  // x as (C, W, N, H), a window of th + 2 rows
    const uint64_t dims[4] = {(uint64_t)g.C, (uint64_t)g.W, (uint64_t)g.N, (uint64_t)g.H};
    const uint64_t str[3] = {(uint64_t)g.C * 2, (uint64_t)g.H * g.W * g.C * 2, (uint64_t)g.W * g.C * 2};
    const uint32_t box[4] = {32u, (uint32_t)d.tw, (uint32_t)d.tn, (uint32_t)d.th + 2};
    rc = make_map(&L.tx, x, 4, dims, str, box, 64);
  } else if (rc == OSAM_OK) {  // the parity view (2C, W/2, 2, H/2, N), 17 row pairs × both parities × 8 columns
    const uint64_t dims[5] = {(uint64_t)2 * g.C, (uint64_t)g.W / 2, 2, (uint64_t)g.H / 2, (uint64_t)g.N};
    const uint64_t str[4] = {(uint64_t)4 * g.C, (uint64_t)g.W * g.C * 2, (uint64_t)2 * g.W * g.C * 2,
                             (uint64_t)g.H * g.W * g.C * 2};
    const uint32_t box[5] = {32u, 8u, 2u, 17u, 1u};
    rc = make_map(&L.tx, x, 5, dims, str, box, 64);
  }
  if (rc) return rc;
  // one CTA per SM: (GEMM N block, run of consecutive tiles)
  const int nblk = g.K / NB;
  long long nsplit = std::max(1, sm_count() / nblk);
  if (nsplit > tiles) nsplit = tiles;
  L.tiles_per_split = (int)cdivll(tiles, nsplit);
  L.nsplit = (int)cdivll(tiles, L.tiles_per_split);
  L.grid = nblk * L.nsplit;
  cudaError_t e = launch_conv_wgrad(L, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSAM_OK : cuda_fail(e, "osam_conv_wgrad (window form) launch");
}

static int wgrad_impl(const osam_conv_plan* p, const void* x, const void* dz, void* dw, float* dw32, float beta,
                      void* ws, size_t ws_bytes, osam_stream_t stream, bool direct) {
  if (!p || !x || !dz || (!dw && !dw32)) return fail(OSAM_ERR_INVALID, "NULL plan or operand");
  const osam_conv_geom& g = p->g;
  if (p->transposed) {
    // dW[c][r][s][k] = Σ_{p,q} x[p][q][c]·dy[2p+r][2q+s][k]: the weight gradient of the stride-2 2×2 conv
    // dg[0] (input dy, output x-shaped) with x in the role of its output gradient
    if (!p->dg_direct) return fail(OSAM_ERR_UNSUPPORTED, "wgrad: transposed conv other than kernel = stride = 2");
    return wgrad_impl(p->dg[0], dz, x, dw, dw32, beta, ws, ws_bytes, stream, direct);
  }
  if (p->mode == A_STEM) return wgrad_stem(p, x, dz, dw, dw32, beta, ws, ws_bytes, stream, direct);
  if (g.K == 1 && g.R == 1 && g.S == 1 && g.stride == 1 && g.pad == 0 && g.C % 8 == 0) {
    const size_t need1 = wgrad_workspace_bytes(p);
    if (!direct && (!ws || ws_bytes < need1 || (reinterpret_cast<uintptr_t>(ws) & 255)))
      return fail(OSAM_ERR_INVALID, "wgrad needs %zu workspace bytes (256-byte aligned)", need1);
    if (reinterpret_cast<uintptr_t>(x) & 15) return fail(OSAM_ERR_INVALID, "wgrad: x must be 16-byte aligned");
    cudaError_t e = launch_wgrad_k1(static_cast<const __half*>(x), static_cast<const __half*>(dz), static_cast<float*>(ws),
                                    static_cast<__half*>(dw), dw32, p->M, g.C, beta, direct,
                                    reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? OSAM_OK : cuda_fail(e, "osam_conv_wgrad (K = 1) launch");
  }
  if (p->transposed || (p->mode != A_S1 && p->mode != A_S2) || g.C % 32 || g.K % 32)
    return fail(OSAM_ERR_UNSUPPORTED, "wgrad: transposed, small-C or non-32-multiple channels");
  const size_t need = wgrad_workspace_bytes(p);
  if (!direct && (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255)))
    return fail(OSAM_ERR_INVALID, "wgrad needs %zu workspace bytes (256-byte aligned)", need);
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dz)) & 15)
    return fail(OSAM_ERR_INVALID, "wgrad: operands must be 16-byte aligned");
  WgradLaunch L{};
  ConvDev& d = L.d;
  d.N = g.N; d.H = g.H; d.W = g.W; d.C = g.C; d.K = g.K;
  d.P = p->P; d.Q = p->Q; d.R = g.R; d.S = g.S; d.stride = g.stride; d.pad = g.pad;
  d.tn = p->tn; d.th = p->th; d.tw = p->tw; d.tiles_q = p->tiles_q; d.tiles_p = p->tiles_p;
  d.tiles_m = p->tiles_m;
  d.err = device_error_word();
  if (!d.err) return fail(OSAM_ERR_CUDA, "cannot allocate the device error word");
  L.AB = g.K % 64 == 0 ? 64 : 32;
  L.BB = g.C % 64 == 0 ? 64 : 32;
  L.BN = g.C <= 32 ? 32 : (g.C <= 64 ? 64 : (g.C <= 128 ? 128 : 256));
  if (L.BB == 32 && L.BN != 32) L.BB = 64;  // C = 96, 160, …: 64-channel boxes, the tail zero-filled
  L.mode = p->mode;
  L.direct = direct;
  L.acc = direct ? dw32 : static_cast<float*>(ws);
  L.dw = static_cast<__half*>(dw);
  L.dw32 = dw32;
  L.n_out = (long long)g.K * g.R * g.S * g.C;
  L.beta = beta;
  if (int nbw = wgrad_window_nb(p)) return wgrad_window(p, x, dz, L, nbw, stream);
  int rc = OSAM_OK;
  {
    const uint64_t dims[4] = {(uint64_t)g.K, (uint64_t)p->Q, (uint64_t)p->P, (uint64_t)g.N};
    const uint64_t str[3] = {(uint64_t)g.K * 2, (uint64_t)p->Q * g.K * 2, (uint64_t)p->P * p->Q * g.K * 2};
    const uint32_t box[4] = {(uint32_t)L.AB, (uint32_t)p->tw, (uint32_t)p->th, (uint32_t)p->tn};
    rc = make_map(&L.tdz, dz, 4, dims, str, box, L.AB * 2);
  }
  if (rc == OSAM_OK && p->mode == A_S1) {
    const uint64_t dims[4] = {(uint64_t)g.C, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)g.N};
    const uint64_t str[3] = {(uint64_t)g.C * 2, (uint64_t)g.W * g.C * 2, (uint64_t)g.H * g.W * g.C * 2};
    const uint32_t box[4] = {(uint32_t)L.BB, (uint32_t)p->tw, (uint32_t)p->th, (uint32_t)p->tn};
    rc = make_map(&L.tx, x, 4, dims, str, box, L.BB * 2);
  } else if (rc == OSAM_OK) {
    const uint64_t dims[5] = {(uint64_t)2 * g.C, (uint64_t)g.W / 2, 2, (uint64_t)g.H / 2, (uint64_t)g.N};
    const uint64_t str[4] = {(uint64_t)4 * g.C, (uint64_t)g.W * g.C * 2, (uint64_t)2 * g.W * g.C * 2,
                             (uint64_t)g.H * g.W * g.C * 2};
    const uint32_t box[5] = {(uint32_t)L.BB, (uint32_t)p->tw, 1, (uint32_t)p->th, (uint32_t)p->tn};
    rc = make_map(&L.tx, x, 5, dims, str, box, L.BB * 2);
  }
  if (rc) return rc;
  // split the pixel tiles so that ≈ 2 CTAs per SM are launched
  const long long nob = (long long)g.R * g.S * ((g.K + 127) / 128) * ((g.C + L.BN - 1) / L.BN);
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  long long nsplit = (2LL * sms + nob - 1) / nob;
  if (nsplit > p->tiles_m) nsplit = p->tiles_m;
  if (nsplit < 1) nsplit = 1;
  L.tiles_per_split = (int)((p->tiles_m + nsplit - 1) / nsplit);
  L.nsplit = (int)((p->tiles_m + L.tiles_per_split - 1) / L.tiles_per_split);
  if (nob * L.nsplit > 0x7fffffffLL) return fail(OSAM_ERR_UNSUPPORTED, "wgrad grid too large");
  L.grid = (int)(nob * L.nsplit);
  cudaError_t e = launch_conv_wgrad(L, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSAM_OK : cuda_fail(e, "osam_conv_wgrad launch");
}

int64_t osam_conv_out_elems(const osam_conv_plan* p) {
  if (!p) return 0;
  if (p->transposed) return (int64_t)p->g.N * 2 * p->g.H * 2 * p->g.W * p->g.K;
  return (int64_t)p->M * p->g.K;
}

int osam_conv_fwd(const osam_conv_plan* p, const void* x, const void* w, void* y, float beta, void* ws,
                  size_t ws_bytes, osam_stream_t stream) {
  ConvLaunch L;
  int rc = conv_prepare(p, x, w, nullptr, beta, y, ws, ws_bytes, &L);
  if (rc) return rc;
  cudaError_t e = conv_launch(L, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSAM_OK : cuda_fail(e, "osam_conv_fwd launch");
}

int osam_conv_fwd_fused(const osam_conv_plan* p, const void* x, const void* w, const osam_epilogue* ep, void* ws,
                        size_t ws_bytes, osam_stream_t stream) {
  if (!ep) return fail(OSAM_ERR_INVALID, "NULL epilogue");
  ConvLaunch L;
  int rc = conv_prepare(p, x, w, ep, 0.f, nullptr, ws, ws_bytes, &L);
  if (rc) return rc;
  cudaError_t e = conv_launch(L, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSAM_OK : cuda_fail(e, "osam_conv_fwd_fused launch");
}

int osam_sppf_fwd(void* cat, int N, int H, int W, int c, osam_stream_t stream) {
  if (!cat || N < 1 || H < 1 || W < 1 || c < 32 || c % 32) return fail(OSAM_ERR_INVALID, "sppf arguments");
  if (reinterpret_cast<uintptr_t>(cat) & 15) return fail(OSAM_ERR_INVALID, "sppf buffer not 16-byte aligned");
  if ((size_t)2 * H * W * 32 * 2 > 200 * 1024) return fail(OSAM_ERR_UNSUPPORTED, "sppf map too large (%dx%d)", H, W);
  cudaError_t e = launch_sppf(static_cast<__half*>(cat), N, H, W, c, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSAM_OK : cuda_fail(e, "osam_sppf_fwd launch");
}

int osam_sppf_bwd(const void* cat, void* dcat, int N, int H, int W, int c, osam_stream_t stream) {
  if (!cat || !dcat || N < 1 || H < 1 || W < 1 || c < 8 || c % 8) return fail(OSAM_ERR_INVALID, "sppf_bwd arguments");
  if ((reinterpret_cast<uintptr_t>(cat) | reinterpret_cast<uintptr_t>(dcat)) & 15)
    return fail(OSAM_ERR_INVALID, "sppf_bwd buffers not 16-byte aligned");
  if (sppf_bwd_smem_bytes(H, W) > 227 * 1024) return fail(OSAM_ERR_UNSUPPORTED, "sppf_bwd map too large (%dx%d)", H, W);
  cudaError_t e = launch_sppf_bwd(static_cast<const __half*>(cat), static_cast<__half*>(dcat), N, H, W, c,
                                  reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSAM_OK : cuda_fail(e, "osam_sppf_bwd launch");
}

int osam_device_error(void) {
  if (!device_error_word()) return fail(OSAM_ERR_CUDA, "no device error word");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "osam_device_error sync");
  int v = 0;
  if (g_err_host) {
    v = *g_err_host;
    *g_err_host = 0;
  }
  // the device variable (kernels launched before the mapped word existed) and the static-scratch entry
  // point's own word: read and clear them on every call
  int* w = nullptr;
  {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_err_mu);
    w = dev >= 0 && dev < 64 ? g_err_static[dev] : nullptr;
  }
  if (w) {
    int vd = 0;
    if ((e = cudaMemcpy(&vd, w, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
      return cuda_fail(e, "osam_device_error read");
    if (vd && (e = cudaMemset(w, 0, sizeof(int))) != cudaSuccess) return cuda_fail(e, "osam_device_error clear");
    if (!v) v = vd;
  }
  const int vs = static_scratch_take_error();
  if (!v) v = vs;
  if (v) set_last_error("device kernel reported error %d", v);
  return v;
}

int osam_device_error_peek(void) {
  const int v = g_err_host ? *g_err_host : 0;
  if (v) set_last_error("device kernel reported error %d", v);
  return v;
}

int osam_selftest_wait_timeout(unsigned long long budget_ns, osam_stream_t stream) {
  if (budget_ns == 0 || budget_ns > 5000000000ull) return fail(OSAM_ERR_INVALID, "budget must be in (0, 5 s]");
  int* w = device_error_word();
  if (!w) return fail(OSAM_ERR_CUDA, "no device error word");
  k_selftest_wait<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(budget_ns, w);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OSAM_OK : cuda_fail(e, "osam_selftest_wait_timeout launch");
}

const char* osam_last_error(void) { return g_last_error; }

}  // extern "C"
