// Transposed-conv forward that allocates nothing: osam_convt_fwd_static_scratch (include/osam.h).
//
// osam_conv_fwd on a transposed plan needs a caller-provided workspace, because the GEMM reads the
// weights in a K-major layout that differs from the (C_in, R, S, C_out) layout callers hold; the
// re-laid-out copy is scratch memory.  Some callers can neither allocate device memory nor hand out a
// workspace — a host that owns the whole device budget and gives a plugin only a stream, or a loop that
// must never reach the allocator (cudaMalloc may synchronise the device; the reference's trainer, for
// one, allocates everything once at start-up, src/core.h:56-66).  For them the scratch lives here, in a
// file-scope device array of fixed size that every GPU loading this library holds until the process
// exits.
//
// Host code never dereferences g_convt_scratch: in host code that name is only a host-side stand-in.
// Its device address is looked up once per device, with that device current, by cudaGetSymbolAddress;
// the first call of the entry point on a device does that lookup.  No path here calls cudaMalloc,
// cudaFree or any allocating library routine — timeouts of these launches go to a static error word
// of this file, which osam_device_error() reads and clears together with the library's own word.
#include <mutex>

#include "conv_internal.h"

namespace osam {
namespace {

// Capacity of the static scratch: C_in · 4 · C_out fp16 weights ≤ 256 KiB, i.e. C_in · C_out ≤ 32768
// (the model's proto upsample, 128 → 128, uses 128 KiB).
constexpr size_t kConvtScratchBytes = 256 * 1024;

static __device__ __align__(256) unsigned char g_convt_scratch[kConvtScratchBytes];
static __device__ int g_convt_err;

struct Slot {
  void* scratch = nullptr;
  int* err = nullptr;
  bool ready = false;
};
Slot g_slot[64];
std::mutex g_slot_mu;

// Device addresses of the static array and error word for the current device (looked up once).
int current_slot(Slot** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_last_error("osam_convt_fwd_static_scratch: no current device (%s)", cudaGetErrorString(e));
    return OSAM_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lk(g_slot_mu);
  Slot& s = g_slot[dev];
  if (!s.ready) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_convt_scratch);
    if (e != cudaSuccess || !p) {
      set_last_error("osam_convt_fwd_static_scratch: cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
      return OSAM_ERR_CUDA;
    }
    void* q = nullptr;
    e = cudaGetSymbolAddress(&q, g_convt_err);
    if (e != cudaSuccess || !q) {
      set_last_error("osam_convt_fwd_static_scratch: cudaGetSymbolAddress(error word) failed: %s",
                     cudaGetErrorString(e));
      return OSAM_ERR_CUDA;
    }
    s.scratch = p;
    s.err = static_cast<int*>(q);
    s.ready = true;
  }
  *out = &s;
  return OSAM_OK;
}

}  // namespace

int static_scratch_take_error() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lk(g_slot_mu);
  if (!g_slot[dev].ready) return 0;
  int v = 0;
  if (cudaMemcpy(&v, g_slot[dev].err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return 0;
  if (v) cudaMemset(g_slot[dev].err, 0, sizeof(int));
  return v;
}

}  // namespace osam

extern "C" int osam_convt_fwd_static_scratch(const osam_conv_plan* plan, const void* x, const void* w, void* y,
                                             float beta, osam_stream_t stream) {
  using namespace osam;
  if (!plan || !plan->transposed) {
    set_last_error("osam_convt_fwd_static_scratch: needs a transposed-conv plan");
    return OSAM_ERR_INVALID;
  }
  const size_t need = (size_t)plan->g.C * plan->g.R * plan->g.S * plan->g.K * sizeof(__half);
  if (need > kConvtScratchBytes) {
    set_last_error("osam_convt_fwd_static_scratch: weights need %zu bytes of scratch; the static array holds %zu "
                   "bytes (C_in*C_out <= 32768)", need, kConvtScratchBytes);
    return OSAM_ERR_INVALID;
  }
  Slot* s = nullptr;
  int rc = current_slot(&s);
  if (rc) return rc;
  ConvLaunch L;
  rc = conv_prepare(plan, x, w, nullptr, beta, y, s->scratch, kConvtScratchBytes, &L, false, s->err);
  if (rc) return rc;
  cudaError_t e = conv_launch(L, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_last_error("osam_convt_fwd_static_scratch launch: %s", cudaGetErrorString(e));
    return OSAM_ERR_CUDA;
  }
  return OSAM_OK;
}
