// Data-parallel gradient exchange of the training pass over NCCL (C ABI: osam_dp_*).
//
// The reference trains on one GPU.  Its multi-GPU plan is plain data parallelism: the batch is sharded over
// one process per GPU, every rank holds the whole model, and the fp32 parameter gradients are averaged with
// ncclAllReduce before the optimizer step reads them (src/optim.cu:15-34, :170-175 need global gradients).
// Here the model's gradient arena keeps the nodes in REVERSE order, so the gradients of nodes [first, n)
// are one contiguous range: the backward runs in buckets (node ranges, last node first), and after each
// bucket an event on the caller's stream lets a communication stream all-reduce that bucket (ncclAvg:
// sum and ÷ world in one collective) while the backward of the earlier nodes continues.  At the end the
// caller's stream waits for the communication stream, so whatever the caller enqueues next (the
// optimizer) sees averaged gradients.
//
// NCCL itself is found at run time: the libnccl.so.2 already loaded in the process (for example by a
// framework that also uses it), else the system one; only its C API is used.  Communicators made here are
// non-blocking (ncclConfig_t::blocking = 0).  osam_dp_wait is the host-side guard: it polls the exchange's
// completion event and ncclCommGetAsyncError with a deadline, and on an error or when the deadline passes
// (a peer died or stopped calling in) it aborts the communicator (ncclCommAbort) and returns an error
// instead of hanging.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "conv_internal.h"

namespace osam {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*abort_comm)(ncclComm_t) = nullptr;
  ncclResult_t (*finalize)(ncclComm_t) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*user_rank)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*get_version)(int*) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
  char why[256] = "";
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the one already in the process, if any
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      snprintf(api.why, sizeof(api.why), "libnccl.so.2 not found: %s", dlerror());
      return;
    }
    auto sym = [&](const char* n) { return dlsym(h, n); };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.init_rank_config = reinterpret_cast<decltype(api.init_rank_config)>(sym("ncclCommInitRankConfig"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
    api.async_error = reinterpret_cast<decltype(api.async_error)>(sym("ncclCommGetAsyncError"));
    api.abort_comm = reinterpret_cast<decltype(api.abort_comm)>(sym("ncclCommAbort"));
    api.finalize = reinterpret_cast<decltype(api.finalize)>(sym("ncclCommFinalize"));
    api.destroy = reinterpret_cast<decltype(api.destroy)>(sym("ncclCommDestroy"));
    api.comm_count = reinterpret_cast<decltype(api.comm_count)>(sym("ncclCommCount"));
    api.user_rank = reinterpret_cast<decltype(api.user_rank)>(sym("ncclCommUserRank"));
    api.get_version = reinterpret_cast<decltype(api.get_version)>(sym("ncclGetVersion"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    api.ok = api.get_unique_id && api.init_rank_config && api.all_reduce && api.async_error && api.abort_comm &&
             api.finalize && api.destroy && api.comm_count && api.user_rank && api.error_string;
    if (!api.ok) snprintf(api.why, sizeof(api.why), "libnccl.so.2 lacks the non-blocking communicator API");
  });
  return api;
}

int dp_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_last_error("%s", buf);
  return code;
}

const char* nccl_str(ncclResult_t r) { return nccl().error_string ? nccl().error_string(r) : "?"; }

// A non-blocking communicator may answer ncclInProgress: poll its state until it settles or `ms` pass.
ncclResult_t settle(ncclComm_t c, ncclResult_t r, int ms) {
  const auto t0 = std::chrono::steady_clock::now();
  while (r == ncclInProgress) {
    if (nccl().async_error(c, &r) != ncclSuccess) return ncclSystemError;
    if (r != ncclInProgress) break;
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(ms)) return ncclInProgress;
    std::this_thread::yield();
  }
  return r;
}

struct DpBucket {
  int first, count;    // nodes [first, first + count)
  int64_t off, n;      // arena elements [off, off + n)
};

}  // namespace
}  // namespace osam

struct osam_dp {
  osam_model* model = nullptr;
  ncclComm_t comm = nullptr;
  bool owns_comm = false;
  bool aborted = false;
  int world = 1, rank = 0;
  float* arena = nullptr;
  int64_t arena_n = 0;
  std::vector<osam::DpBucket> buckets;
  cudaStream_t comm_stream = nullptr;
  std::vector<cudaEvent_t> ready;  // per bucket: its backward is issued (recorded on the caller's stream)
  cudaEvent_t done = nullptr;      // the last exchange has finished (recorded on the communication stream)
};

namespace {
using namespace osam;

// Buckets in backward order (last node first): a bucket closes once it holds at least `elems` gradients;
// nodes without parameters ride along with the bucket being filled; the arena ranges are then widened to
// tile the arena, alignment padding included, so one collective per bucket covers every element once.
std::vector<DpBucket> plan(osam_model* m, int64_t arena_n, int64_t elems) {
  const int n = osam_model_num_launches(m);
  std::vector<DpBucket> out;
  int hi = n;
  int64_t lo_off = -1, hi_end = -1, acc = 0;
  for (int i = n - 1; i >= 0; i--) {
    int64_t off = 0, cnt = 0;
    osam_model_node_grad_range(m, i, &off, &cnt);
    if (cnt) {
      lo_off = lo_off < 0 ? off : std::min(lo_off, off);
      hi_end = std::max(hi_end, off + cnt);
      acc += cnt;
    }
    if ((acc >= elems && lo_off >= 0) || i == 0) {
      if (lo_off >= 0) {
        out.push_back(DpBucket{i, hi - i, lo_off, hi_end - lo_off});
      } else if (!out.empty()) {
        out.back().first = i;
        out.back().count += hi - i;
      }
      hi = i;
      lo_off = hi_end = -1;
      acc = 0;
    }
  }
  // widen to tile [0, arena_n): each bucket runs to where the next (by offset) starts
  std::vector<DpBucket*> by_off;
  for (auto& b : out) by_off.push_back(&b);
  std::sort(by_off.begin(), by_off.end(), [](const DpBucket* a, const DpBucket* b) { return a->off < b->off; });
  if (!by_off.empty()) by_off.front()->n += by_off.front()->off, by_off.front()->off = 0;
  for (size_t k = 0; k + 1 < by_off.size(); k++) by_off[k]->n = by_off[k + 1]->off - by_off[k]->off;
  if (!by_off.empty()) by_off.back()->n = arena_n - by_off.back()->off;
  return out;
}

int finish_create(osam_dp* d, size_t bucket_bytes, osam_dp** out) {
  int rc = osam_model_grad_arena(d->model, &d->arena, &d->arena_n);
  if (rc) return rc;
  const int64_t elems = std::max<int64_t>(1, (int64_t)(bucket_bytes / sizeof(float)));
  d->buckets = plan(d->model, d->arena_n, elems);
  cudaError_t e;
  int lo = 0, hi = 0;
  cudaDeviceGetStreamPriorityRange(&lo, &hi);
  if ((e = cudaStreamCreateWithPriority(&d->comm_stream, cudaStreamNonBlocking, hi)) != cudaSuccess)
    return dp_fail(OSAM_ERR_CUDA, "osam_dp: communication stream: %s", cudaGetErrorString(e));
  d->ready.assign(d->buckets.size(), nullptr);
  for (auto& ev : d->ready)
    if ((e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming)) != cudaSuccess)
      return dp_fail(OSAM_ERR_CUDA, "osam_dp: events: %s", cudaGetErrorString(e));
  if ((e = cudaEventCreateWithFlags(&d->done, cudaEventDisableTiming)) != cudaSuccess)
    return dp_fail(OSAM_ERR_CUDA, "osam_dp: events: %s", cudaGetErrorString(e));
  *out = d;
  return OSAM_OK;
}

void release(osam_dp* d) {
  if (!d) return;
  if (d->comm_stream) cudaStreamSynchronize(d->comm_stream);
  for (auto ev : d->ready)
    if (ev) cudaEventDestroy(ev);
  if (d->done) cudaEventDestroy(d->done);
  if (d->comm_stream) cudaStreamDestroy(d->comm_stream);
  if (d->comm && d->owns_comm) {
    if (d->aborted) {
      // already aborted: nothing left to free
    } else {
      ncclResult_t r = nccl().finalize(d->comm);
      r = settle(d->comm, r, 10000);
      if (r == ncclSuccess) nccl().destroy(d->comm);
      else nccl().abort_comm(d->comm);
    }
  }
  delete d;
}

}  // namespace

extern "C" {

int osam_dp_unique_id(unsigned char id[128]) {
  if (!id) return dp_fail(OSAM_ERR_INVALID, "osam_dp_unique_id: NULL");
  if (!nccl().ok) return dp_fail(OSAM_ERR_UNSUPPORTED, "osam_dp_unique_id: %s", nccl().why);
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
  ncclUniqueId u;
  const ncclResult_t r = nccl().get_unique_id(&u);
  if (r != ncclSuccess) return dp_fail(OSAM_ERR_CUDA, "ncclGetUniqueId: %s", nccl_str(r));
  std::memcpy(id, &u, sizeof(u));
  return OSAM_OK;
}

int osam_dp_create(osam_model* m, int world, int rank, const unsigned char id[128], size_t bucket_bytes,
                   int init_timeout_ms, osam_dp** out) {
  if (!m || !out || world < 1 || rank < 0 || rank >= world || (world > 1 && !id))
    return dp_fail(OSAM_ERR_INVALID, "osam_dp_create: arguments");
  *out = nullptr;
  auto* d = new osam_dp;
  d->model = m;
  d->world = world;
  d->rank = rank;
  if (world > 1) {
    if (!nccl().ok) {
      delete d;
      return dp_fail(OSAM_ERR_UNSUPPORTED, "osam_dp_create: %s", nccl().why);
    }
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // every call returns at once; osam_dp_wait polls and can abort
    ncclResult_t r = nccl().init_rank_config(&d->comm, world, u, rank, &cfg);
    r = settle(d->comm, r, init_timeout_ms > 0 ? init_timeout_ms : 120000);
    if (r != ncclSuccess) {
      if (d->comm) nccl().abort_comm(d->comm);
      delete d;
      return dp_fail(r == ncclInProgress ? OSAM_ERR_TIMEOUT : OSAM_ERR_CUDA, "ncclCommInitRankConfig: %s",
                     r == ncclInProgress ? "the other ranks did not join in time" : nccl_str(r));
    }
    d->owns_comm = true;
  }
  const int rc = finish_create(d, bucket_bytes, out);
  if (rc) release(d);
  return rc;
}

int osam_dp_create_from_comm(osam_model* m, void* nccl_comm, size_t bucket_bytes, osam_dp** out) {
  if (!m || !out || !nccl_comm) return dp_fail(OSAM_ERR_INVALID, "osam_dp_create_from_comm: arguments");
  if (!nccl().ok) return dp_fail(OSAM_ERR_UNSUPPORTED, "osam_dp_create_from_comm: %s", nccl().why);
  *out = nullptr;
  auto* d = new osam_dp;
  d->model = m;
  d->comm = static_cast<ncclComm_t>(nccl_comm);
  if (nccl().comm_count(d->comm, &d->world) != ncclSuccess || nccl().user_rank(d->comm, &d->rank) != ncclSuccess) {
    delete d;
    return dp_fail(OSAM_ERR_INVALID, "osam_dp_create_from_comm: not a usable NCCL communicator");
  }
  const int rc = finish_create(d, bucket_bytes, out);
  if (rc) release(d);
  return rc;
}

int osam_dp_num_buckets(const osam_dp* d) { return d ? (int)d->buckets.size() : 0; }

int osam_dp_bucket(const osam_dp* d, int i, int* first, int* count, int64_t* off, int64_t* n) {
  if (!d || i < 0 || i >= (int)d->buckets.size()) return dp_fail(OSAM_ERR_INVALID, "osam_dp_bucket: index");
  const DpBucket& b = d->buckets[i];
  if (first) *first = b.first;
  if (count) *count = b.count;
  if (off) *off = b.off;
  if (n) *n = b.n;
  return OSAM_OK;
}

int osam_dp_backward(osam_dp* d, osam_stream_t stream) {
  if (!d) return dp_fail(OSAM_ERR_INVALID, "osam_dp_backward: NULL");
  if (d->aborted) return dp_fail(OSAM_ERR_CUDA, "osam_dp_backward: the communicator was aborted");
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  for (size_t k = 0; k < d->buckets.size(); k++) {
    const DpBucket& b = d->buckets[k];
    int rc = osam_model_backward_nodes(d->model, b.first, b.count, stream);
    if (rc) return rc;
    if (d->world == 1) continue;
    if ((e = cudaEventRecord(d->ready[k], st)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(d->comm_stream, d->ready[k], 0)) != cudaSuccess)
      return dp_fail(OSAM_ERR_CUDA, "osam_dp_backward: %s", cudaGetErrorString(e));
    ncclResult_t r = nccl().all_reduce(d->arena + b.off, d->arena + b.off, (size_t)b.n, ncclFloat32, ncclAvg, d->comm,
                                       d->comm_stream);
    r = settle(d->comm, r, 60000);
    if (r != ncclSuccess) {
      nccl().abort_comm(d->comm);
      d->aborted = true;
      return dp_fail(OSAM_ERR_CUDA, "ncclAllReduce (bucket %zu): %s", k,
                     r == ncclInProgress ? "could not be enqueued in time" : nccl_str(r));
    }
  }
  if (d->world > 1) {
    if ((e = cudaEventRecord(d->done, d->comm_stream)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(st, d->done, 0)) != cudaSuccess)
      return dp_fail(OSAM_ERR_CUDA, "osam_dp_backward: %s", cudaGetErrorString(e));
  }
  return OSAM_OK;
}

int osam_dp_wait(osam_dp* d, int timeout_ms) {
  if (!d) return dp_fail(OSAM_ERR_INVALID, "osam_dp_wait: NULL");
  if (d->world == 1) return OSAM_OK;
  if (d->aborted) return dp_fail(OSAM_ERR_CUDA, "osam_dp_wait: the communicator was aborted");
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    const cudaError_t q = cudaEventQuery(d->done);
    if (q == cudaSuccess) return OSAM_OK;
    if (q != cudaErrorNotReady) return dp_fail(OSAM_ERR_CUDA, "osam_dp_wait: %s", cudaGetErrorString(q));
    ncclResult_t r = ncclSuccess;
    if (nccl().async_error(d->comm, &r) != ncclSuccess || (r != ncclSuccess && r != ncclInProgress)) {
      nccl().abort_comm(d->comm);
      d->aborted = true;
      return dp_fail(OSAM_ERR_CUDA, "osam_dp_wait: NCCL reported %s; communicator aborted", nccl_str(r));
    }
    if (timeout_ms >= 0 && std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
      nccl().abort_comm(d->comm);
      d->aborted = true;
      return dp_fail(OSAM_ERR_TIMEOUT, "osam_dp_wait: the gradient exchange did not finish within %d ms; "
                     "communicator aborted", timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int osam_dp_destroy(osam_dp* d) {
  release(d);
  return OSAM_OK;
}

}  // extern "C"
