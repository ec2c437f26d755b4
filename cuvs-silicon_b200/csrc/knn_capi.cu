// knn_capi.cu -- the engine behind include/cuvs_b200.h.
//
// Host orchestration of the exact search, replacing
// MetalContext::search_brute_force (src/metal_context.mm:139-255):
//
//   reference (per call)                      this engine
//   -------------------------------------     ------------------------------------
//   first call: fp16 dataset + d_norms on     knn_index_build: rows -> HBM fp16
//     one CPU thread, cached by (ptr,N,D)       (ld-padded) + norms, one kernel
//   Q x D fp16 + q_norms on the host          queries -> device, convert kernel
//   MPS GEMM -> Q x N fp32 in memory          fused scan kernel (TMA + tcgen05),
//   l2_topk_from_cross (K <= 16)                Q x N stays on chip, any k<=256
//   copy Q x K out                            merge kernel -> caller's buffers
//
// Multi-GPU: one process per GPU, each index holds a contiguous row shard;
// the per-rank top-k lists are all-gathered with NCCL and merged on every
// rank.  NCCL is created non-blocking and every wait on it is bounded by a
// host deadline, after which the communicator is aborted (KNN_ENCCL).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <dlfcn.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>
#include <nccl.h>

#include <algorithm>
#include <array>
#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "cuvs_b200.h"
#include "knn_internal.h"

using knn::Plan;

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_dispatch{0};

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

#define KNN_CUDA(call)                                                                   \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return fail(e_ == cudaErrorMemoryAllocation ? KNN_ENOMEM : KNN_ECUDA, "%s: %s (%s)", \
                  #call, cudaGetErrorString(e_), cudaGetErrorName(e_));                  \
  } while (0)

// Device buffer that only grows.
struct DevBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
  bool grew = false;  // set when ensure() reallocated (pointers changed)
  int ensure(size_t need) {
    if (need <= bytes) return KNN_OK;
    grew = true;
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
    const size_t want = need + need / 4;
    cudaError_t e = cudaMalloc(&ptr, want);
    if (e != cudaSuccess) {
      ptr = nullptr;
      return fail(KNN_ENOMEM, "cudaMalloc(%zu) failed: %s", want, cudaGetErrorString(e));
    }
    bytes = want;
    return KNN_OK;
  }
  void release() {
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
  }
  template <typename T>
  T* as() const {
    return static_cast<T*>(ptr);
  }
};

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// K-major fp16 matrix [rows][ld] as a TMA map with 64 x box_rows boxes and
// 128-byte swizzle.
int encode_rows(CUtensorMap* map, const __half* base, int64_t rows, int64_t ld,
                uint32_t box_rows) {
  auto enc = get_encode();
  if (!enc) return fail(KNN_ECUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld * 2) % 16 != 0)
    return fail(KNN_ECUDA, "TMA base/stride not 16-byte aligned");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(ld), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(knn::kKChunk), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KNN_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return KNN_OK;
}

int64_t row_ld(int64_t dim) {
  if (dim < knn::kKChunk) return knn::kKChunk;
  return (dim + 7) / 8 * 8;
}

// Device address of page-locked host memory (nullptr for anything else).
// Page-locked memory is addressable by the device under unified virtual
// addressing, so kernels may read or write it in place.
void* pinned_device_ptr(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

// 0 = host memory, 1 = device memory of `device`, -1 = other device.
int classify(const void* p, int device) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged)
    return a.device == device ? 1 : -1;
  return 0;
}


// NCCL is resolved at run time, the first time a communicator is needed.
// dlopen("libnccl.so.2") returns the copy the process already holds (for
// example the one a framework loaded) or else the system library, so the
// engine never forces a second NCCL version into a process.
struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) =
      nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.why = dlerror();
      return;
    }
    bool all = true;
    auto get = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (!fn) all = false;
    };
    get(api.GetUniqueId, "ncclGetUniqueId");
    get(api.CommInitRankConfig, "ncclCommInitRankConfig");
    get(api.CommGetAsyncError, "ncclCommGetAsyncError");
    get(api.CommAbort, "ncclCommAbort");
    get(api.CommDestroy, "ncclCommDestroy");
    get(api.AllGather, "ncclAllGather");
    get(api.GetErrorString, "ncclGetErrorString");
    api.ok = all;
    if (!all) api.why = "libnccl.so.2 lacks a required symbol";
  });
  return api;
}

const char* nccl_str(ncclResult_t r) {
  return nccl().GetErrorString ? nccl().GetErrorString(r) : "nccl unavailable";
}

}  // namespace

struct knn_index {
  int device = 0;
  int num_sms = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  std::mutex mu;

  // dataset (this rank's shard)
  int64_t n = 0, dim = 0, ld = 0;
  int64_t row_offset = 0, total_rows = 0;
  int metric = KNN_METRIC_L2_EXPANDED;
  __half* data = nullptr;
  float* norms = nullptr;
  CUtensorMap xmap;       // 256-row boxes (full tiles)
  CUtensorMap xmap_tail;  // 32-row boxes (a work unit's narrower last tile)
  CUtensorMap xmap_half;  // 128-row boxes (a CTA's half of a full tile with CTA pairs)

  // exact fp32 re-ranking (knn_index_set_rerank): the fp32 rows are kept
  // by a build made while re-ranking is enabled
  bool rerank = false;
  float* rows32 = nullptr;     // n x dim fp32 rows
  float* max_norm2 = nullptr;  // device scalar: largest |x16|^2
  int* uncert_dev = nullptr;
  int* uncert_host = nullptr;  // pinned
  int64_t last_uncertified = 0, last_widened = 0;

  // per-search scratch
  DevBuf q32, q16, qnorm, part_d, part_i, out_d, out_i, gather_send, gather_recv;
  DevBuf cand_d, cand_i, rr_d, rr_i, pilot, thr, xdec, bound;
  int* err_dev = nullptr;
  int* err_host = nullptr;  // pinned

  // multi-GPU
  ncclComm_t comm = nullptr;
  int n_ranks = 1, rank = 0;
  // peer exchange over NVLink (see knn::Exchange): own buffer, every rank's
  // buffer as this GPU addresses it, capacity in (query, rank) list entries
  bool peer_enabled = true;
  float* xbuf = nullptr;
  float* xpeer[knn::kMaxRanks] = {};
  int64_t xcap = 0;
  uint32_t* epoch_dev = nullptr;  // the exchange epoch (see knn::Exchange)
  uint64_t peer_wait_ns = knn::kPeerWaitDefaultNs;

  // CUDA graphs of the device-side search pipeline, replayed when a search
  // repeats the buffers and shape of a captured one.  `generation` changes
  // whenever a pointer a graph captured may have changed (scratch growth,
  // rebuild, stream or communicator change) and invalidates every graph.
  struct GraphEntry {
    const void* queries;
    const void* neighbors;
    const void* distances;
    int in_place;  // bit 0: queries, bit 1: outputs used in place (page-locked host memory),
                   // bit 2: internal-order lists (knn_index_search_lists)
    int64_t nq, k, ks;
    bool i64;
    cudaStream_t stream;
    uint64_t generation;
    int launches;
    cudaGraphExec_t exec;
  };
  bool use_graphs = true;
  uint64_t generation = 1;
  std::vector<GraphEntry> graphs;

  // set for the duration of knn_index_search_lists: results stay in the
  // internal order (inner product: -q.x ascending) for a later merge
  bool lists_mode = false;

  // profiling: one (before scan, after scan, after merge) event triple per
  // search, read back when the stats are requested
  bool profiling = false;
  cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
  std::vector<std::array<cudaEvent_t, 3>> prof_events;
  size_t prof_used = 0;
  double scan_ms = 0.0, merge_ms = 0.0;
  int64_t scan_launches = 0, kernel_launches = 0;
};

namespace {

int poll_nccl(knn_index* h, double seconds) {
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = nccl().CommGetAsyncError(h->comm, &st);
    if (r != ncclSuccess) return fail(KNN_ENCCL, "ncclCommGetAsyncError: %s", nccl_str(r));
    if (st == ncclSuccess) return KNN_OK;
    if (st != ncclInProgress) {
      nccl().CommAbort(h->comm);
      h->comm = nullptr;
      return fail(KNN_ENCCL, "NCCL async error: %s", nccl_str(st));
    }
    const double waited =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (waited > seconds) {
      nccl().CommAbort(h->comm);
      h->comm = nullptr;
      return fail(KNN_ENCCL, "NCCL operation did not complete within %.0f s", seconds);
    }
    // spin for the first millisecond (enqueueing normally takes microseconds),
    // then back off
    if (waited < 1e-3) {
      std::this_thread::yield();
    } else {
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
  }
}

int sync_stream(knn_index* h);
void drop_exchange(knn_index* h);

// Exchange buffer capacity: (query, rank) list entries; searches with more
// queries x k use the NCCL all-gather instead.
constexpr int64_t kExchangeCapQK = 65536;

// Allocates this rank's exchange buffer, all-gathers the CUDA IPC handles
// with NCCL and maps every peer's buffer.  On any failure the peer exchange
// stays off (searches use the NCCL all-gather); the return value only
// reports NCCL failures, which also break the fallback.
int setup_exchange(knn_index* h) {
  drop_exchange(h);
  if (h->n_ranks > knn::kMaxRanks) return KNN_OK;
  const int64_t words = knn::exchange_words(h->n_ranks, kExchangeCapQK);
  cudaIpcMemHandle_t mine;
  std::memset(&mine, 0, sizeof(mine));
  bool ok = cudaMalloc(&h->xbuf, static_cast<size_t>(words) * 4) == cudaSuccess;
  if (ok) ok = cudaMemset(h->xbuf, 0, static_cast<size_t>(words) * 4) == cudaSuccess;
  if (ok) ok = cudaMalloc(&h->epoch_dev, sizeof(uint32_t)) == cudaSuccess;
  if (ok) ok = cudaMemset(h->epoch_dev, 0, sizeof(uint32_t)) == cudaSuccess;
  if (ok) ok = cudaIpcGetMemHandle(&mine, h->xbuf) == cudaSuccess;
  cudaGetLastError();
  // every rank takes part in the all-gather, even with a failed allocation
  // (a zero handle marks it), so no rank is left waiting
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  void* dev = nullptr;
  if (cudaMalloc(&dev, hb * (h->n_ranks + 1)) != cudaSuccess) {
    cudaGetLastError();
    drop_exchange(h);
    return fail(KNN_ENOMEM, "exchange handle buffer allocation failed");
  }
  std::vector<cudaIpcMemHandle_t> all(h->n_ranks);
  cudaMemcpy(static_cast<char*>(dev) + hb * h->n_ranks, &mine, hb, cudaMemcpyHostToDevice);
  ncclResult_t r = nccl().AllGather(static_cast<char*>(dev) + hb * h->n_ranks, dev, hb,
                                    ncclUint8, h->comm, h->stream);
  int st = KNN_OK;
  if (r == ncclInProgress) st = poll_nccl(h, 60.0);
  else if (r != ncclSuccess) st = fail(KNN_ENCCL, "ncclAllGather(handles): %s", nccl_str(r));
  if (st == KNN_OK) st = sync_stream(h);
  if (st == KNN_OK &&
      cudaMemcpy(all.data(), dev, hb * h->n_ranks, cudaMemcpyDeviceToHost) != cudaSuccess)
    st = fail(KNN_ECUDA, "exchange handle copy failed");
  cudaFree(dev);
  if (st != KNN_OK) {
    drop_exchange(h);
    return st;
  }
  cudaIpcMemHandle_t zero;
  std::memset(&zero, 0, sizeof(zero));
  for (int p = 0; p < h->n_ranks && ok; ++p) {
    if (std::memcmp(&all[p], &zero, hb) == 0) ok = false;  // that rank has no buffer
  }
  for (int p = 0; p < h->n_ranks && ok; ++p) {
    if (p == h->rank) {
      h->xpeer[p] = h->xbuf;
      continue;
    }
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, all[p], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = false;
      break;
    }
    h->xpeer[p] = static_cast<float*>(ptr);
  }
  // Every rank must agree on using the exchange (a peer that could not map
  // would otherwise never receive lists): agree through one more all-gather
  // of the local verdict.
  int32_t verdict = ok ? 1 : 0;
  int32_t* vdev = nullptr;
  if (cudaMalloc(&vdev, sizeof(int32_t) * (h->n_ranks + 1)) == cudaSuccess) {
    cudaMemcpy(vdev + h->n_ranks, &verdict, sizeof(int32_t), cudaMemcpyHostToDevice);
    r = nccl().AllGather(vdev + h->n_ranks, vdev, 1, ncclInt32, h->comm, h->stream);
    st = KNN_OK;
    if (r == ncclInProgress) st = poll_nccl(h, 60.0);
    else if (r != ncclSuccess) st = fail(KNN_ENCCL, "ncclAllGather(verdict): %s", nccl_str(r));
    if (st == KNN_OK) st = sync_stream(h);
    std::vector<int32_t> v(h->n_ranks, 0);
    if (st == KNN_OK)
      cudaMemcpy(v.data(), vdev, sizeof(int32_t) * h->n_ranks, cudaMemcpyDeviceToHost);
    cudaFree(vdev);
    if (st != KNN_OK) {
      drop_exchange(h);
      return st;
    }
    for (int32_t x : v) ok = ok && x == 1;
  } else {
    cudaGetLastError();
    ok = false;  // (peers then time out of nothing: they use NCCL only if all agree)
  }
  if (!ok) {
    drop_exchange(h);
    return KNN_OK;
  }
  h->xcap = kExchangeCapQK;
  return KNN_OK;
}

// Waits for the index stream; with a communicator attached the wait is a
// poll bounded by a deadline so a lost peer cannot hang the caller.
int sync_stream(knn_index* h) {
  if (!h->comm) {
    KNN_CUDA(cudaStreamSynchronize(h->stream));
    return KNN_OK;
  }
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t e = cudaStreamQuery(h->stream);
    if (e == cudaSuccess) return KNN_OK;
    if (e != cudaErrorNotReady) return fail(KNN_ECUDA, "stream: %s", cudaGetErrorString(e));
    ncclResult_t st = ncclSuccess;
    nccl().CommGetAsyncError(h->comm, &st);
    if (st != ncclSuccess && st != ncclInProgress) {
      nccl().CommAbort(h->comm);
      h->comm = nullptr;
      return fail(KNN_ENCCL, "NCCL async error: %s", nccl_str(st));
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > 60.0) {
      nccl().CommAbort(h->comm);
      h->comm = nullptr;
      return fail(KNN_ENCCL, "search on the communicator did not complete within 60 s");
    }
    std::this_thread::yield();
  }
}

// Closes the peer mappings and frees this rank's exchange buffer.
void drop_exchange(knn_index* h) {
  for (int r = 0; r < knn::kMaxRanks; ++r) {
    if (h->xpeer[r] && h->xpeer[r] != h->xbuf) cudaIpcCloseMemHandle(h->xpeer[r]);
    h->xpeer[r] = nullptr;
  }
  if (h->xbuf) cudaFree(h->xbuf);
  if (h->epoch_dev) cudaFree(h->epoch_dev);
  h->xbuf = nullptr;
  h->epoch_dev = nullptr;
  h->xcap = 0;
}

void drop_graphs(knn_index* h) {
  for (auto& g : h->graphs)
    if (g.exec) cudaGraphExecDestroy(g.exec);
  h->graphs.clear();
}

// Adds the durations of the recorded event triples (the stream must be idle).
int drain_profile(knn_index* h) {
  for (size_t i = 0; i < h->prof_used; ++i) {
    float a = 0.f, b = 0.f;
    KNN_CUDA(cudaEventElapsedTime(&a, h->prof_events[i][0], h->prof_events[i][1]));
    KNN_CUDA(cudaEventElapsedTime(&b, h->prof_events[i][1], h->prof_events[i][2]));
    h->scan_ms += a;
    h->merge_ms += b;
  }
  h->prof_used = 0;
  return KNN_OK;
}

// Returns the next free event triple (synchronising and draining when the
// pool is full).
int next_profile_slot(knn_index* h, std::array<cudaEvent_t, 3>** out) {
  constexpr size_t kMaxPending = 4096;
  if (h->prof_used == kMaxPending) {
    KNN_CUDA(cudaStreamSynchronize(h->stream));
    int st = drain_profile(h);
    if (st != KNN_OK) return st;
  }
  if (h->prof_used == h->prof_events.size()) {
    std::array<cudaEvent_t, 3> t{};
    for (auto& e : t) KNN_CUDA(cudaEventCreate(&e));
    h->prof_events.push_back(t);
  }
  *out = &h->prof_events[h->prof_used++];
  return KNN_OK;
}

int check_device_error(knn_index* h) {
  if (*h->err_host != 0) {
    const int code = *h->err_host;
    *h->err_host = 0;
    cudaMemsetAsync(h->err_dev, 0, sizeof(int), h->stream);
    cudaStreamSynchronize(h->stream);
    if (code == knn::kErrTimeoutPeer)
      return fail(KNN_ETIMEOUT,
                  "a peer's list did not arrive within %.3f s of this rank's own (device "
                  "code %d): every rank must issue each search within that bound "
                  "(knn_index_set_peer_timeout); attach the communicator again before the "
                  "next search", static_cast<double>(h->peer_wait_ns) * 1e-9, code);
    if (code == knn::kErrBounds)
      return fail(KNN_ECUDA, "a device bounds check failed (debug build, device code %d)", code);
    return fail(KNN_ETIMEOUT, "scan kernel gave up on a bounded wait (device code %d)", code);
  }
  return KNN_OK;
}

int validate_search(knn_index* h, const float* queries, int64_t nq, int64_t k,
                    const void* neighbors, const float* distances) {
  if (!h) return fail(KNN_EINVAL, "null index");
  if (nq < 0 || k < 0) return fail(KNN_EINVAL, "negative n_queries or k");
  if (nq == 0 || k == 0) return KNN_OK;
  // reference: src/cagra.cpp:100-103
  if (!queries || !neighbors || !distances)
    return fail(KNN_EINVAL, "search requires valid query and output buffers");
  if (!h->data) return fail(KNN_EINVAL, "index has no dataset (build it first)");
  if (k > KNN_MAX_K) return fail(KNN_EUNSUPPORTED, "k = %lld exceeds the maximum %d",
                                 (long long)k, KNN_MAX_K);
  return KNN_OK;
}

// Whether a search of nq queries x k on an index with a communicator
// exchanges its lists through the NVLink peer buffers (else NCCL).
bool uses_peer_exchange(const knn_index* h, int64_t nq, int64_t k) {
  return h->comm && h->peer_enabled && h->xcap > 0 && h->epoch_dev && nq * k <= h->xcap;
}

// Everything a search enqueues on the device between the query upload and
// the result download: query conversion, scan, merge(s) and the all-gather.
// Captured into a CUDA graph when the search is replayable.
// With re-ranking, the scan keeps ks > k candidates per query, a merge
// orders them, and the re-rank kernel replaces the scan's distances by the
// exact fp32 ones; the k-lists it writes then take the place of the scan's
// per-unit lists in the exchange between ranks.
int enqueue_pipeline(knn_index* h, const float* qsrc, int64_t nq, int64_t k, int64_t ks,
                     bool rerank, const Plan& plan, float* dst_d, void* dst_i, bool out_i64,
                     std::array<cudaEvent_t, 3>* prof, int* launches_out) {
  int st;
  const size_t qk = static_cast<size_t>(nq) * k;
  const int64_t nq_pad = knn::padded_query_rows(plan);
  if (rerank) KNN_CUDA(cudaMemsetAsync(h->uncert_dev, 0, sizeof(int), h->stream));
  KNN_CUDA(knn::launch_convert_rows(qsrc, false, nq, nq_pad, h->dim, h->q16.as<__half>(),
                                    h->ld, h->qnorm.as<float>(), h->stream,
                                    h->bound.as<uint32_t>(), nq, h->epoch_dev,
                                    plan.spread != 0));
  CUtensorMap qmap;
  if ((st = encode_rows(&qmap, h->q16.as<__half>(), nq_pad, h->ld, knn::kQueryRows)) != KNN_OK)
    return st;

  knn::ScanParams p;
  p.row_norms = h->norms;
  p.query_norms = h->qnorm.as<float>();
  p.part_d = h->part_d.as<float>();
  p.part_i = h->part_i.as<uint32_t>();
  p.err = h->err_dev;
  p.n_rows = h->n;
  p.n_queries = nq;
  p.n_gran = (h->n + plan.gran_rows - 1) / plan.gran_rows;
  p.q_rows = nq_pad;
  p.pair = static_cast<int32_t>(plan.pair);
  p.compact = static_cast<int32_t>(plan.compact);
  p.heap_rows = static_cast<int32_t>(plan.heap_rows);
  p.spread = static_cast<int32_t>(plan.spread);
  p.gran_rows = static_cast<int32_t>(plan.gran_rows);
  p.unit_queries = static_cast<int32_t>(plan.unit_queries);
  p.ld = h->ld;
  p.k = static_cast<int32_t>(ks);
  p.query_block = static_cast<int32_t>(plan.query_block);
  p.query_tiles = static_cast<int32_t>(plan.query_tiles);
  p.splits = static_cast<int32_t>(plan.splits);
  p.units = static_cast<int32_t>(plan.units);
  p.k_chunks = static_cast<int32_t>((h->ld + knn::kKChunk - 1) / knn::kKChunk);
  p.stages = static_cast<int32_t>(plan.stages);
  p.dataset_evict_first = plan.query_tiles == 1 ? 1 : 0;
  p.metric = h->metric;
  p.pilot = 0;
  p.pilot_out = nullptr;
  p.thr_init = nullptr;
  p.bound = nullptr;
  const bool neg = h->metric == KNN_METRIC_INNER_PRODUCT && !h->lists_mode;

  if (prof) KNN_CUDA(cudaEventRecord((*prof)[0], h->stream));
  // with timing events between kernels, launch them plainly serialised
  const bool overlap = prof == nullptr;
  int launches = 2;
  if (ks >= knn::kPilotMinK) {
    // large k: a pilot pass over one tile per unit bounds every query's k-th
    // distance, and the main pass filters with that bound from its first tile
    p.pilot = 1;
    p.pilot_out = h->pilot.as<float>();
    KNN_CUDA(knn::launch_scan(qmap, h->xmap, h->xmap_tail, h->xmap_half, p, plan, h->stream, overlap));
    KNN_CUDA(knn::launch_pilot_threshold(p.pilot_out, static_cast<int>(plan.splits),
                                         static_cast<int>(ks), nq, h->thr.as<float>(),
                                         h->stream));
    p.pilot = 0;
    p.pilot_out = nullptr;
    p.thr_init = h->thr.as<float>();
    launches += 2;
  }
  p.bound = h->bound.as<uint32_t>();
  KNN_CUDA(knn::launch_scan(qmap, h->xmap, h->xmap_tail, h->xmap_half, p, plan, h->stream, overlap));
  if (prof) KNN_CUDA(cudaEventRecord((*prof)[1], h->stream));

  // the lists the final stage merges: the scan's per-unit lists, or one
  // re-ranked list per query
  const float* ld = p.part_d;
  const uint32_t* li = p.part_i;
  int64_t l_stride = ks, q_stride = plan.splits * ks, off = h->row_offset;
  int n_lists = static_cast<int>(plan.splits);
  const int64_t part_len = nq * plan.splits * ks;  // entries of the per-unit lists
  int64_t l_len = part_len;
  if (rerank) {
    float* cd = h->cand_d.as<float>();
    uint32_t* ci = h->cand_i.as<uint32_t>();
    KNN_CUDA(knn::launch_merge(p.part_d, p.part_i, ks, plan.splits * ks,
                               static_cast<int>(plan.splits), static_cast<int>(ks), nq, 0, cd,
                               ci, false, h->stream, overlap, nullptr, false, h->err_dev,
                               part_len));
    if (!h->comm) {
      KNN_CUDA(knn::launch_rerank(qsrc, h->rows32, h->dim, cd, ci, static_cast<int>(ks),
                                  static_cast<int>(k), nq, h->metric, h->max_norm2,
                                  h->row_offset, dst_d, dst_i, out_i64, neg, h->uncert_dev,
                                  h->stream));
      if (prof) KNN_CUDA(cudaEventRecord((*prof)[2], h->stream));
      *launches_out = launches + 2;
      return KNN_OK;
    }
    float* rd = h->rr_d.as<float>();
    uint32_t* ri = h->rr_i.as<uint32_t>();
    KNN_CUDA(knn::launch_rerank(qsrc, h->rows32, h->dim, cd, ci, static_cast<int>(ks),
                                static_cast<int>(k), nq, h->metric, h->max_norm2,
                                h->row_offset, rd, ri, false, false, h->uncert_dev,
                                h->stream));
    launches += 2;
    ld = rd;
    li = ri;
    l_stride = k;
    q_stride = k;
    n_lists = 1;
    off = 0;
    l_len = nq * k;
  }
  if (!h->comm) {
    KNN_CUDA(knn::launch_merge(ld, li, l_stride, q_stride, n_lists, static_cast<int>(k), nq,
                               off, dst_d, dst_i, out_i64, h->stream, overlap, nullptr, neg,
                               h->err_dev, l_len));
    launches += 1;
  } else if (uses_peer_exchange(h, nq, k)) {
    // peer exchange, one kernel: each query's block merges this rank's lists,
    // writes the result into every rank's exchange buffer over NVLink as
    // epoch-tagged words, collects every rank's list for the query from its
    // own buffer (bounded wait) and merges them
    knn::Exchange ex = {};
    for (int r = 0; r < h->n_ranks; ++r) ex.base[r] = h->xpeer[r];
    ex.cap_qk = h->xcap;
    ex.n_ranks = h->n_ranks;
    ex.rank = h->rank;
    ex.epoch = h->epoch_dev;
    ex.wait_ns = h->peer_wait_ns;
    ex.err = h->err_dev;
    ex.in_len = l_len;
    ex.mode = 1;
    ex.dec_d = h->xdec.as<float>();
    ex.dec_i = reinterpret_cast<uint32_t*>(ex.dec_d + qk * h->n_ranks);
    KNN_CUDA(knn::launch_merge(ld, li, l_stride, q_stride, n_lists, static_cast<int>(k), nq, off,
                               dst_d, dst_i, out_i64, h->stream, overlap, &ex, neg));
    launches += 1;
  } else {
    // local merge into the send buffer: [dist k floats | idx k uint32] per query
    const size_t list_bytes = qk * 8;
    float* send_d = h->gather_send.as<float>();
    uint32_t* send_i = reinterpret_cast<uint32_t*>(send_d + qk);
    KNN_CUDA(knn::launch_merge(ld, li, l_stride, q_stride, n_lists, static_cast<int>(k), nq, off,
                               send_d, send_i, false, h->stream, overlap, nullptr, false,
                               h->err_dev, l_len));
    ncclResult_t r = nccl().AllGather(h->gather_send.ptr, h->gather_recv.ptr, list_bytes,
                                      ncclUint8, h->comm, h->stream);
    if (r == ncclInProgress) {
      if ((st = poll_nccl(h, 60.0)) != KNN_OK) return st;
    } else if (r != ncclSuccess) {
      return fail(KNN_ENCCL, "ncclAllGather: %s", nccl_str(r));
    }
    // rank r's block: [qk dist][qk idx]; list l of query q at dist + l*2qk + q*k
    const float* rd = h->gather_recv.as<float>();
    const uint32_t* ri = reinterpret_cast<const uint32_t*>(rd + qk);
    KNN_CUDA(knn::launch_merge(rd, ri, static_cast<int64_t>(2 * qk), k, h->n_ranks,
                               static_cast<int>(k), nq, 0, dst_d, dst_i, out_i64, h->stream,
                               overlap, nullptr, neg, h->err_dev,
                               static_cast<int64_t>(2 * qk) * h->n_ranks));
    launches += 2;
  }
  if (prof) KNN_CUDA(cudaEventRecord((*prof)[2], h->stream));
  *launches_out = launches;
  return KNN_OK;
}

// One search pass (h->mu held, device set, buffers classified: cq/cn/cd are
// 1 for device and 0 for host memory).  ks: candidates the scan keeps per
// query (k, or more when re-ranking).
int search_pass(knn_index* h, const float* queries, int64_t nq, int64_t k, int64_t ks,
                bool rerank, void* neighbors, float* distances, bool out_i64, bool sync,
                int cq, int cn, int cd) {
  int st;
  Plan plan;
  const int pst = knn::plan_search(h->n, h->dim, nq, ks, h->num_sms, &plan);
  if (pst != 0) return fail(pst, "k = %lld is outside the engine's limits", (long long)ks);

  // Page-locked host buffers are used in place: the query conversion reads
  // the queries from host memory and the last kernel writes the results
  // there, with no staging copies (the re-rank kernel, which reads the fp32
  // queries many times, keeps the device copy).
  const void* q_pin = cq == 0 && !rerank ? pinned_device_ptr(queries) : nullptr;
  void* d_pin = cd == 0 && cn == 0 ? pinned_device_ptr(distances) : nullptr;
  void* n_pin = d_pin ? pinned_device_ptr(neighbors) : nullptr;
  if (!n_pin) d_pin = nullptr;
  // which host buffers are used in place (a graph key: a buffer that is no
  // longer page-locked must not be replayed into)
  const int in_place = (q_pin ? 1 : 0) | (d_pin ? 2 : 0) | (h->lists_mode ? 4 : 0);

  // scratch: everything is sized before any work is enqueued or captured
  const size_t qk = static_cast<size_t>(nq) * k;
  const size_t idx_bytes = qk * (out_i64 ? 8 : 4);
  const int64_t nq_pad = knn::padded_query_rows(plan);
  DevBuf* bufs[] = {&h->q16,    &h->qnorm,       &h->part_d,      &h->part_i,
                    &h->q32,    &h->out_d,       &h->out_i,       &h->gather_send,
                    &h->gather_recv, &h->cand_d, &h->cand_i, &h->rr_d, &h->rr_i,
                    &h->pilot, &h->thr, &h->xdec, &h->bound};
  for (DevBuf* b : bufs) b->grew = false;
  if ((st = h->q16.ensure(static_cast<size_t>(nq_pad) * h->ld * 2)) != KNN_OK) return st;
  if ((st = h->qnorm.ensure(static_cast<size_t>(nq) * 4)) != KNN_OK) return st;
  if ((st = h->bound.ensure(static_cast<size_t>(nq) * 4)) != KNN_OK) return st;
  if ((st = h->part_d.ensure(static_cast<size_t>(plan.partial_bytes / 2))) != KNN_OK) return st;
  if ((st = h->part_i.ensure(static_cast<size_t>(plan.partial_bytes / 2))) != KNN_OK) return st;
  if (cq == 0 && !q_pin && (st = h->q32.ensure(static_cast<size_t>(nq) * h->dim * 4)) != KNN_OK)
    return st;
  if (cd == 0 && !d_pin && (st = h->out_d.ensure(qk * 4)) != KNN_OK) return st;
  if (cn == 0 && !n_pin && (st = h->out_i.ensure(idx_bytes)) != KNN_OK) return st;
  if (h->comm) {
    if ((st = h->gather_send.ensure(qk * 8)) != KNN_OK) return st;
    if ((st = h->gather_recv.ensure(qk * 8 * h->n_ranks)) != KNN_OK) return st;
    if ((st = h->xdec.ensure(qk * 8 * h->n_ranks)) != KNN_OK) return st;
  }
  if (ks >= knn::kPilotMinK) {
    if ((st = h->pilot.ensure(static_cast<size_t>(nq) * plan.splits * 32 * 4)) != KNN_OK)
      return st;
    if ((st = h->thr.ensure(static_cast<size_t>(nq) * 4)) != KNN_OK) return st;
  }
  if (rerank) {
    const size_t qks = static_cast<size_t>(nq) * ks;
    if ((st = h->cand_d.ensure(qks * 4)) != KNN_OK) return st;
    if ((st = h->cand_i.ensure(qks * 4)) != KNN_OK) return st;
    if (h->comm && (st = h->rr_d.ensure(qk * 4)) != KNN_OK) return st;
    if (h->comm && (st = h->rr_i.ensure(qk * 4)) != KNN_OK) return st;
  }
  for (DevBuf* b : bufs) {
    if (b->grew) {
      ++h->generation;
      drop_graphs(h);
      break;
    }
  }

  const float* qsrc = queries;
  if (q_pin) {
    qsrc = static_cast<const float*>(q_pin);
  } else if (cq == 0) {
    KNN_CUDA(cudaMemcpyAsync(h->q32.ptr, queries, static_cast<size_t>(nq) * h->dim * 4,
                             cudaMemcpyHostToDevice, h->stream));
    qsrc = h->q32.as<float>();
  }
  float* dst_d = d_pin ? static_cast<float*>(d_pin) : cd == 0 ? h->out_d.as<float>() : distances;
  void* dst_i = n_pin ? n_pin : cn == 0 ? h->out_i.ptr : neighbors;

  int launches = 0;
  std::array<cudaEvent_t, 3>* prof = nullptr;
  if (h->profiling) {
    if ((st = next_profile_slot(h, &prof)) != KNN_OK) return st;
  }
  // Replay a graph for searches that repeat buffers + shape.  Host buffers
  // qualify too: the graph reads and writes either them in place (page-
  // locked, part of the key) or the staging buffers (whose reallocation
  // bumps the generation).  With a communicator only the peer exchange is
  // replayed (its epoch lives in device memory, so its kernels take the same
  // arguments every search); the NCCL all-gather path is launched directly
  // (replaying the captured all-gather measured slower at 8 ranks).
  const bool graphable =
      h->use_graphs && !prof && (!h->comm || uses_peer_exchange(h, nq, k));
  knn_index::GraphEntry* hit = nullptr;
  if (graphable) {
    for (auto& g : h->graphs) {
      if (g.queries == queries && g.neighbors == neighbors && g.distances == distances &&
          g.in_place == in_place && g.nq == nq && g.k == k && g.ks == ks && g.i64 == out_i64 &&
          g.stream == h->stream && g.generation == h->generation) {
        hit = &g;
        break;
      }
    }
    if (hit && hit->exec == nullptr) {
      // second search with this key: capture it now (the first ran directly,
      // which also performed the one-time per-device kernel set-up)
      h->graphs.erase(h->graphs.begin() + (hit - h->graphs.data()));
      hit = nullptr;
    } else if (!hit) {
      if (h->graphs.size() >= 8) {
        if (h->graphs.front().exec) cudaGraphExecDestroy(h->graphs.front().exec);
        h->graphs.erase(h->graphs.begin());
      }
      h->graphs.push_back({queries, neighbors, distances, in_place, nq, k, ks, out_i64,
                           h->stream, h->generation, 0, nullptr});
      goto direct;
    }
    if (!hit) {
      cudaGraph_t graph = nullptr;
      cudaGraphExec_t exec = nullptr;
      bool ok = cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal) ==
                cudaSuccess;
      int cst = KNN_OK;
      if (ok) {
        cst = enqueue_pipeline(h, qsrc, nq, k, ks, rerank, plan, dst_d, dst_i, out_i64, nullptr,
                               &launches);
        ok = cudaStreamEndCapture(h->stream, &graph) == cudaSuccess && cst == KNN_OK;
      }
      if (ok) ok = cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
      if (graph) cudaGraphDestroy(graph);
      cudaGetLastError();
      if (ok) {
        if (h->graphs.size() >= 8) {
          if (h->graphs.front().exec) cudaGraphExecDestroy(h->graphs.front().exec);
          h->graphs.erase(h->graphs.begin());
        }
        h->graphs.push_back({queries, neighbors, distances, in_place, nq, k, ks, out_i64,
                             h->stream, h->generation, launches, exec});
        hit = &h->graphs.back();
      } else {
        // capture is not available here: run searches directly from now on
        if (exec) cudaGraphExecDestroy(exec);
        h->use_graphs = false;
        if (cst != KNN_OK) return cst;
      }
    }
  }
direct:
  if (hit) {
    KNN_CUDA(cudaGraphLaunch(hit->exec, h->stream));
    launches = hit->launches;
  } else {
    if ((st = enqueue_pipeline(h, qsrc, nq, k, ks, rerank, plan, dst_d, dst_i, out_i64, prof,
                               &launches)) != KNN_OK)
      return st;
  }
  if (rerank)
    KNN_CUDA(cudaMemcpyAsync(h->uncert_host, h->uncert_dev, sizeof(int), cudaMemcpyDeviceToHost,
                             h->stream));

  if (cd == 0 && !d_pin)
    KNN_CUDA(cudaMemcpyAsync(distances, dst_d, qk * 4, cudaMemcpyDeviceToHost, h->stream));
  if (cn == 0 && !n_pin)
    KNN_CUDA(cudaMemcpyAsync(neighbors, dst_i, idx_bytes, cudaMemcpyDeviceToHost, h->stream));
  g_dispatch.fetch_add(launches);
  h->kernel_launches += launches;
  h->scan_launches += 1;

  if (!sync) return KNN_OK;
  KNN_CUDA(cudaMemcpyAsync(h->err_host, h->err_dev, sizeof(int), cudaMemcpyDeviceToHost,
                           h->stream));
  if ((st = sync_stream(h)) != KNN_OK) return st;
  if (rerank) h->last_uncertified = *h->uncert_host;
  return check_device_error(h);
}

// Core search.  out_i64: neighbours are int64.  sync: block and check.
// A blocking re-ranked search on one device whose result is not certified
// for some query is repeated once with the largest candidate count.
int search_impl(knn_index* h, const float* queries, int64_t nq, int64_t k, void* neighbors,
                float* distances, bool out_i64, bool sync, bool require_device,
                bool lists = false) {
  int st = validate_search(h, queries, nq, k, neighbors, distances);
  if (st != KNN_OK || nq == 0 || k == 0) return st;
  std::lock_guard<std::mutex> lock(h->mu);
  KNN_CUDA(cudaSetDevice(h->device));
  if (lists && h->comm)
    return fail(KNN_EINVAL, "knn_index_search_lists: the index has a communicator attached");
  struct ListsMode {
    knn_index* h;
    ~ListsMode() { h->lists_mode = false; }
  } lists_guard{h};
  h->lists_mode = lists;

  const int cq = classify(queries, h->device);
  const int cn = classify(neighbors, h->device);
  const int cd = classify(distances, h->device);
  if (cq < 0 || cn < 0 || cd < 0)
    return fail(KNN_EINVAL, "buffer lives on a different device than the index");
  if (require_device && (cq == 0 || cn == 0 || cd == 0))
    return fail(KNN_EINVAL, "knn_index_search_async requires device buffers");

  const bool rerank = h->rerank && h->rows32;
  int64_t ks = rerank ? knn::rerank_candidates(k) : k;
  h->last_widened = 0;
  while (true) {
    st = search_pass(h, queries, nq, k, ks, rerank, neighbors, distances, out_i64, sync, cq, cn,
                     cd);
    if (st != KNN_OK || !sync || !rerank || h->last_uncertified == 0 || h->comm ||
        ks >= knn::kMaxK)
      return st;
    h->last_widened = h->last_uncertified;
    ks = knn::kMaxK;
  }
}

int build_impl(knn_index* h, const void* rows, int dtype, int64_t n, int64_t dim, int metric,
               int64_t row_offset, int64_t total_rows) {
  if (!h) return fail(KNN_EINVAL, "null index");
  // reference: src/cagra.cpp:26-28
  if (metric != KNN_METRIC_L2_EXPANDED && metric != KNN_METRIC_INNER_PRODUCT)
    return fail(KNN_EINVAL, "metric %d is not L2Expanded (0) or InnerProduct (1)", metric);
  // reference: src/cagra.cpp:29-32
  if (!rows || n <= 0 || dim <= 0)
    return fail(KNN_EINVAL, "build requires a non-empty dataset");
  if (dtype != KNN_DTYPE_F32 && dtype != KNN_DTYPE_F16)
    return fail(KNN_EINVAL, "unknown dtype %d", dtype);
  if (row_offset < 0 || total_rows < row_offset + n)
    return fail(KNN_EINVAL, "shard [%lld, %lld) outside %lld rows", (long long)row_offset,
                (long long)(row_offset + n), (long long)total_rows);
  if (total_rows >= static_cast<int64_t>(KNN_NO_INDEX))
    return fail(KNN_EUNSUPPORTED, "at most 2^32 - 2 rows (uint32 neighbour indices)");
  if (n > (int64_t(1) << 31) - 256)
    return fail(KNN_EUNSUPPORTED, "at most 2^31 - 256 rows per device");
  if (dim > (int64_t(1) << 20)) return fail(KNN_EUNSUPPORTED, "dim above 2^20");

  std::lock_guard<std::mutex> lock(h->mu);
  KNN_CUDA(cudaSetDevice(h->device));
  const int where = classify(rows, h->device);
  if (where < 0) return fail(KNN_EINVAL, "dataset lives on a different device than the index");

  if (h->rerank && dtype != KNN_DTYPE_F32)
    return fail(KNN_EINVAL, "re-ranking keeps the fp32 rows: build from fp32 rows");

  if (h->data) cudaFree(h->data);
  if (h->norms) cudaFree(h->norms);
  if (h->rows32) cudaFree(h->rows32);
  h->data = nullptr;
  h->norms = nullptr;
  h->rows32 = nullptr;
  h->n = 0;

  const int64_t ld = row_ld(dim);
  KNN_CUDA(cudaMalloc(&h->data, static_cast<size_t>(n) * ld * 2));
  KNN_CUDA(cudaMalloc(&h->norms, static_cast<size_t>(n) * 4));
  const size_t esz = dtype == KNN_DTYPE_F16 ? 2 : 4;
  if (h->rerank) {
    // keep the fp32 rows on the device and convert from that copy
    KNN_CUDA(cudaMalloc(&h->rows32, static_cast<size_t>(n) * dim * 4));
    KNN_CUDA(cudaMemcpyAsync(h->rows32, rows, static_cast<size_t>(n) * dim * 4, cudaMemcpyDefault,
                             h->stream));
    KNN_CUDA(knn::launch_convert_rows(h->rows32, false, n, n, dim, h->data, ld, h->norms,
                                      h->stream));
    KNN_CUDA(knn::launch_max_norm(h->norms, n, h->max_norm2, h->stream));
    g_dispatch.fetch_add(2);
  } else if (where == 1) {
    KNN_CUDA(knn::launch_convert_rows(rows, dtype == KNN_DTYPE_F16, n, n, dim, h->data, ld,
                                      h->norms, h->stream));
    g_dispatch.fetch_add(1);
  } else {
    // host rows: stage through a device buffer in chunks of <= 256 MiB
    const int64_t chunk = std::max<int64_t>(1, (int64_t(256) << 20) / (dim * esz));
    DevBuf stage;
    int st = stage.ensure(static_cast<size_t>(std::min(chunk, n)) * dim * esz);
    if (st != KNN_OK) return st;
    for (int64_t r0 = 0; r0 < n; r0 += chunk) {
      const int64_t rr = std::min(chunk, n - r0);
      const char* src = static_cast<const char*>(rows) + static_cast<size_t>(r0) * dim * esz;
      cudaError_t e = cudaMemcpyAsync(stage.ptr, src, static_cast<size_t>(rr) * dim * esz,
                                      cudaMemcpyHostToDevice, h->stream);
      if (e == cudaSuccess)
        e = knn::launch_convert_rows(stage.ptr, dtype == KNN_DTYPE_F16, rr, rr, dim,
                                     h->data + static_cast<size_t>(r0) * ld, ld, h->norms + r0,
                                     h->stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
      if (e != cudaSuccess) {
        stage.release();
        return fail(KNN_ECUDA, "dataset upload: %s", cudaGetErrorString(e));
      }
      g_dispatch.fetch_add(1);
    }
    stage.release();
  }
  KNN_CUDA(cudaStreamSynchronize(h->stream));
  int st = encode_rows(&h->xmap, h->data, n, ld, knn::kTileRows);
  if (st == KNN_OK) st = encode_rows(&h->xmap_tail, h->data, n, ld, knn::kTailBox);
  if (st == KNN_OK) st = encode_rows(&h->xmap_half, h->data, n, ld, knn::kTileRows / 2);
  if (st != KNN_OK) return st;
  ++h->generation;
  drop_graphs(h);
  h->n = n;
  h->dim = dim;
  h->ld = ld;
  h->metric = metric;
  h->row_offset = row_offset;
  h->total_rows = total_rows;
  return KNN_OK;
}

// Builds the index from rows already in the engine's storage format: fp16
// rows (host or device, n x dim, dense) and their fp32 norms as a previous
// build computed them (knn_index_device_norms); nothing is converted.
int build_prepared_impl(knn_index* h, const void* rows16, const float* norms, int64_t n,
                        int64_t dim, int metric, int64_t row_offset, int64_t total_rows) {
  if (!h) return fail(KNN_EINVAL, "null index");
  if (metric != KNN_METRIC_L2_EXPANDED && metric != KNN_METRIC_INNER_PRODUCT)
    return fail(KNN_EINVAL, "metric %d is not L2Expanded (0) or InnerProduct (1)", metric);
  if (!rows16 || !norms || n <= 0 || dim <= 0)
    return fail(KNN_EINVAL, "build requires a non-empty dataset and its norms");
  if (row_offset < 0 || total_rows < row_offset + n)
    return fail(KNN_EINVAL, "shard [%lld, %lld) outside %lld rows", (long long)row_offset,
                (long long)(row_offset + n), (long long)total_rows);
  if (total_rows >= static_cast<int64_t>(KNN_NO_INDEX))
    return fail(KNN_EUNSUPPORTED, "at most 2^32 - 2 rows (uint32 neighbour indices)");
  if (n > (int64_t(1) << 31) - 256)
    return fail(KNN_EUNSUPPORTED, "at most 2^31 - 256 rows per device");
  if (dim > (int64_t(1) << 20)) return fail(KNN_EUNSUPPORTED, "dim above 2^20");
  std::lock_guard<std::mutex> lock(h->mu);
  KNN_CUDA(cudaSetDevice(h->device));
  if (classify(rows16, h->device) < 0 || classify(norms, h->device) < 0)
    return fail(KNN_EINVAL, "dataset lives on a different device than the index");
  if (h->rerank)
    return fail(KNN_EINVAL, "re-ranking keeps the fp32 rows: build from fp32 rows");
  if (h->data) cudaFree(h->data);
  if (h->norms) cudaFree(h->norms);
  if (h->rows32) cudaFree(h->rows32);
  h->data = nullptr;
  h->norms = nullptr;
  h->rows32 = nullptr;
  h->n = 0;
  const int64_t ld = row_ld(dim);
  KNN_CUDA(cudaMalloc(&h->data, static_cast<size_t>(n) * ld * 2));
  KNN_CUDA(cudaMalloc(&h->norms, static_cast<size_t>(n) * 4));
  if (ld != dim) KNN_CUDA(cudaMemsetAsync(h->data, 0, static_cast<size_t>(n) * ld * 2, h->stream));
  KNN_CUDA(cudaMemcpy2DAsync(h->data, static_cast<size_t>(ld) * 2, rows16,
                             static_cast<size_t>(dim) * 2, static_cast<size_t>(dim) * 2,
                             static_cast<size_t>(n), cudaMemcpyDefault, h->stream));
  KNN_CUDA(cudaMemcpyAsync(h->norms, norms, static_cast<size_t>(n) * 4, cudaMemcpyDefault,
                           h->stream));
  KNN_CUDA(cudaStreamSynchronize(h->stream));
  int st = encode_rows(&h->xmap, h->data, n, ld, knn::kTileRows);
  if (st == KNN_OK) st = encode_rows(&h->xmap_tail, h->data, n, ld, knn::kTailBox);
  if (st == KNN_OK) st = encode_rows(&h->xmap_half, h->data, n, ld, knn::kTileRows / 2);
  if (st != KNN_OK) return st;
  ++h->generation;
  drop_graphs(h);
  h->n = n;
  h->dim = dim;
  h->ld = ld;
  h->metric = metric;
  h->row_offset = row_offset;
  h->total_rows = total_rows;
  return KNN_OK;
}

// Streams rows [r0, r1) of a dataset file into the index (see
// knn_index_build_file).  The host reads chunk c + 1 into one pinned buffer
// while the device copies chunk c out of the other (a pitched copy that
// drops the fvecs record headers on the way) and converts it to fp16 rows
// and norms; at most two chunks are ever held on the host.
int build_file_impl(knn_index* h, const char* path, int format, int metric, int n_ranks,
                    int rank) {
  if (!h || !path) return fail(KNN_EINVAL, "null index or path");
  if (format != KNN_FILE_FVECS && format != KNN_FILE_BIN_F32)
    return fail(KNN_EINVAL, "unknown file format %d", format);
  if (metric != KNN_METRIC_L2_EXPANDED && metric != KNN_METRIC_INNER_PRODUCT)
    return fail(KNN_EINVAL, "metric %d is not L2Expanded (0) or InnerProduct (1)", metric);
  if (n_ranks < 1 || rank < 0 || rank >= n_ranks)
    return fail(KNN_EINVAL, "rank %d of %d", rank, n_ranks);
  const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return fail(KNN_EINVAL, "cannot open %s: %s", path, std::strerror(errno));
  struct FdCloser {
    int fd;
    ~FdCloser() { ::close(fd); }
  } closer{fd};
  struct stat sb;
  if (::fstat(fd, &sb) != 0) return fail(KNN_EINVAL, "cannot stat %s", path);
  const int64_t fsize = static_cast<int64_t>(sb.st_size);
  auto pread_all = [&](void* dst, int64_t bytes, int64_t off) -> bool {
    char* p = static_cast<char*>(dst);
    while (bytes > 0) {
      const ssize_t r = ::pread(fd, p, static_cast<size_t>(bytes), static_cast<off_t>(off));
      if (r < 0 && errno == EINTR) continue;
      if (r <= 0) return false;
      p += r;
      bytes -= r;
      off += r;
    }
    return true;
  };
  // shape: rows, dim, record size and where row 0 starts
  int64_t total = 0, dim = 0, rec = 0, base = 0, lead = 0;
  if (format == KNN_FILE_FVECS) {
    int32_t d0 = 0;
    if (fsize < 4 || !pread_all(&d0, 4, 0) || d0 <= 0)
      return fail(KNN_EINVAL, "%s: not an fvecs file (first row width %d)", path, (int)d0);
    dim = d0;
    rec = 4 + 4 * dim;
    if (fsize % rec != 0)
      return fail(KNN_EINVAL, "%s: %lld bytes is not a whole number of %lld-byte rows", path,
                  (long long)fsize, (long long)rec);
    total = fsize / rec;
    lead = 4;
  } else {
    int32_t hdr[2] = {0, 0};
    if (fsize < 8 || !pread_all(hdr, 8, 0) || hdr[0] <= 0 || hdr[1] <= 0)
      return fail(KNN_EINVAL, "%s: not a .bin matrix (shape %d x %d)", path, (int)hdr[0],
                  (int)hdr[1]);
    total = hdr[0];
    dim = hdr[1];
    rec = 4 * dim;
    base = 8;
    if (fsize != base + total * rec)
      return fail(KNN_EINVAL, "%s: %lld bytes, %lld expected for %lld x %lld", path,
                  (long long)fsize, (long long)(base + total * rec), (long long)total,
                  (long long)dim);
  }
  int64_t r0 = 0, r1 = 0;
  {
    const int64_t per = (total + n_ranks - 1) / n_ranks;
    r0 = std::min<int64_t>(total, static_cast<int64_t>(rank) * per);
    r1 = std::min<int64_t>(total, r0 + per);
  }
  const int64_t n = r1 - r0;
  if (n <= 0) return fail(KNN_EINVAL, "%s: rank %d of %d holds no rows", path, rank, n_ranks);
  if (total >= static_cast<int64_t>(KNN_NO_INDEX))
    return fail(KNN_EUNSUPPORTED, "at most 2^32 - 2 rows (uint32 neighbour indices)");
  if (n > (int64_t(1) << 31) - 256) return fail(KNN_EUNSUPPORTED, "at most 2^31 - 256 rows per device");
  if (dim > (int64_t(1) << 20)) return fail(KNN_EUNSUPPORTED, "dim above 2^20");

  std::lock_guard<std::mutex> lock(h->mu);
  KNN_CUDA(cudaSetDevice(h->device));
  if (h->data) cudaFree(h->data);
  if (h->norms) cudaFree(h->norms);
  if (h->rows32) cudaFree(h->rows32);
  h->data = nullptr;
  h->norms = nullptr;
  h->rows32 = nullptr;
  h->n = 0;
  const int64_t ld = row_ld(dim);
  KNN_CUDA(cudaMalloc(&h->data, static_cast<size_t>(n) * ld * 2));
  KNN_CUDA(cudaMalloc(&h->norms, static_cast<size_t>(n) * 4));
  if (h->rerank) KNN_CUDA(cudaMalloc(&h->rows32, static_cast<size_t>(n) * dim * 4));

  const int64_t chunk = std::max<int64_t>(1, (int64_t(64) << 20) / rec);
  const int64_t chunk_rows = std::min(chunk, n);
  void* pinned[2] = {nullptr, nullptr};
  DevBuf stage[2];
  cudaEvent_t done[2] = {nullptr, nullptr};
  int st = KNN_OK;
  auto cleanup = [&]() {
    for (int b = 0; b < 2; ++b) {
      if (done[b]) {
        cudaEventSynchronize(done[b]);
        cudaEventDestroy(done[b]);
      }
      if (pinned[b]) cudaFreeHost(pinned[b]);
      stage[b].release();
    }
  };
  for (int b = 0; b < 2 && st == KNN_OK; ++b) {
    if (cudaMallocHost(&pinned[b], static_cast<size_t>(chunk_rows * rec)) != cudaSuccess ||
        cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming) != cudaSuccess)
      st = fail(KNN_ENOMEM, "pinned staging buffers");
    else if (!h->rerank)
      st = stage[b].ensure(static_cast<size_t>(chunk_rows) * dim * 4);
  }
  int c = 0;
  for (int64_t a = 0; a < n && st == KNN_OK; a += chunk, ++c) {
    const int b = c & 1;
    const int64_t rr = std::min(chunk, n - a);
    // the buffer's previous copy must have left it before it is refilled
    if (cudaEventSynchronize(done[b]) != cudaSuccess) {
      st = fail(KNN_ECUDA, "dataset upload: %s", cudaGetErrorString(cudaGetLastError()));
      break;
    }
    char* raw = static_cast<char*>(pinned[b]);
    if (!pread_all(raw, rr * rec, base + (r0 + a) * rec)) {
      st = fail(KNN_EINVAL, "%s: read failed at row %lld", path, (long long)(r0 + a));
      break;
    }
    if (format == KNN_FILE_FVECS) {
      for (int64_t r = 0; r < rr; ++r) {
        int32_t w;
        std::memcpy(&w, raw + r * rec, 4);
        if (w != dim) {
          st = fail(KNN_EINVAL, "%s: row %lld has width %d, expected %lld", path,
                    (long long)(r0 + a + r), (int)w, (long long)dim);
          break;
        }
      }
      if (st != KNN_OK) break;
    }
    float* dst = h->rerank ? h->rows32 + a * dim : stage[b].as<float>();
    cudaError_t e = cudaMemcpy2DAsync(dst, static_cast<size_t>(dim) * 4, raw + lead,
                                      static_cast<size_t>(rec), static_cast<size_t>(dim) * 4,
                                      static_cast<size_t>(rr), cudaMemcpyHostToDevice, h->stream);
    if (e == cudaSuccess)
      e = knn::launch_convert_rows(dst, false, rr, rr, dim, h->data + a * ld, ld, h->norms + a,
                                   h->stream);
    if (e == cudaSuccess) e = cudaEventRecord(done[b], h->stream);
    if (e != cudaSuccess) st = fail(KNN_ECUDA, "dataset upload: %s", cudaGetErrorString(e));
    g_dispatch.fetch_add(1);
  }
  if (st == KNN_OK && h->rerank) {
    const cudaError_t e = knn::launch_max_norm(h->norms, n, h->max_norm2, h->stream);
    if (e != cudaSuccess) st = fail(KNN_ECUDA, "max norm: %s", cudaGetErrorString(e));
  }
  if (st == KNN_OK && cudaStreamSynchronize(h->stream) != cudaSuccess)
    st = fail(KNN_ECUDA, "dataset upload: %s", cudaGetErrorString(cudaGetLastError()));
  cleanup();
  if (st == KNN_OK) st = encode_rows(&h->xmap, h->data, n, ld, knn::kTileRows);
  if (st == KNN_OK) st = encode_rows(&h->xmap_tail, h->data, n, ld, knn::kTailBox);
  if (st == KNN_OK) st = encode_rows(&h->xmap_half, h->data, n, ld, knn::kTileRows / 2);
  if (st != KNN_OK) {
    cudaFree(h->data);
    cudaFree(h->norms);
    if (h->rows32) cudaFree(h->rows32);
    h->data = nullptr;
    h->norms = nullptr;
    h->rows32 = nullptr;
    return st;
  }
  ++h->generation;
  drop_graphs(h);
  h->n = n;
  h->dim = dim;
  h->ld = ld;
  h->metric = metric;
  h->row_offset = r0;
  h->total_rows = total;
  return KNN_OK;
}

}  // namespace

extern "C" {

const char* knn_last_error(void) { return g_last_error.c_str(); }

const char* knn_status_string(int status) {
  switch (status) {
    case KNN_OK: return "KNN_OK";
    case KNN_EINVAL: return "KNN_EINVAL";
    case KNN_ECUDA: return "KNN_ECUDA";
    case KNN_ENCCL: return "KNN_ENCCL";
    case KNN_ETIMEOUT: return "KNN_ETIMEOUT";
    case KNN_ENOMEM: return "KNN_ENOMEM";
    case KNN_EUNSUPPORTED: return "KNN_EUNSUPPORTED";
    default: return "KNN_UNKNOWN";
  }
}

int knn_index_create(int device, knn_index** out) {
  if (!out) return fail(KNN_EINVAL, "null output handle");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    cudaGetLastError();
    return fail(KNN_ECUDA, "no CUDA device available (%s)", cudaGetErrorString(e));
  }
  if (device < 0 || device >= count)
    return fail(KNN_EINVAL, "device %d out of range (%d devices)", device, count);
  cudaDeviceProp prop;
  KNN_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(KNN_EUNSUPPORTED, "device %d is sm_%d%d; this engine is built for sm_100a",
                device, prop.major, prop.minor);
  KNN_CUDA(cudaSetDevice(device));
  knn_index* h = new knn_index();
  h->device = device;
  h->num_sms = prop.multiProcessorCount;
  e = cudaStreamCreateWithFlags(&h->own_stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&h->err_dev, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(h->err_dev, 0, sizeof(int));
  if (e == cudaSuccess) e = cudaMallocHost(&h->err_host, sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&h->uncert_dev, sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&h->max_norm2, sizeof(float));
  if (e == cudaSuccess) e = cudaMallocHost(&h->uncert_host, sizeof(int));
  for (int i = 0; i < 4 && e == cudaSuccess; ++i) e = cudaEventCreate(&h->ev[i]);
  if (e != cudaSuccess) {
    knn_index_destroy(h);
    return fail(KNN_ECUDA, "index setup: %s", cudaGetErrorString(e));
  }
  *h->err_host = 0;
  *h->uncert_host = 0;
  h->stream = h->own_stream;
  *out = h;
  return KNN_OK;
}

int knn_index_destroy(knn_index* h) {
  if (!h) return KNN_OK;
  cudaSetDevice(h->device);
  if (h->stream) cudaStreamSynchronize(h->stream);
  drop_graphs(h);
  drop_exchange(h);
  if (h->comm) nccl().CommDestroy(h->comm);
  for (DevBuf* b : {&h->q32, &h->q16, &h->qnorm, &h->part_d, &h->part_i, &h->out_d, &h->out_i,
                    &h->gather_send, &h->gather_recv, &h->cand_d, &h->cand_i, &h->rr_d,
                    &h->rr_i, &h->pilot, &h->thr, &h->xdec, &h->bound})
    b->release();
  if (h->data) cudaFree(h->data);
  if (h->norms) cudaFree(h->norms);
  if (h->rows32) cudaFree(h->rows32);
  if (h->max_norm2) cudaFree(h->max_norm2);
  if (h->uncert_dev) cudaFree(h->uncert_dev);
  if (h->uncert_host) cudaFreeHost(h->uncert_host);
  if (h->err_dev) cudaFree(h->err_dev);
  if (h->err_host) cudaFreeHost(h->err_host);
  for (auto& ev : h->ev)
    if (ev) cudaEventDestroy(ev);
  for (auto& t : h->prof_events)
    for (auto& ev : t) cudaEventDestroy(ev);
  if (h->own_stream) cudaStreamDestroy(h->own_stream);
  delete h;
  return KNN_OK;
}

int knn_index_set_stream(knn_index* h, void* stream) {
  if (!h) return fail(KNN_EINVAL, "null index");
  std::lock_guard<std::mutex> lock(h->mu);
  h->stream = stream ? static_cast<cudaStream_t>(stream) : h->own_stream;
  return KNN_OK;  // graphs are keyed on the stream
}

int knn_index_build(knn_index* h, const void* rows, int dtype, int64_t n, int64_t dim,
                    int metric) {
  return build_impl(h, rows, dtype, n, dim, metric, 0, n);
}

int knn_index_build_shard(knn_index* h, const void* rows, int dtype, int64_t n, int64_t dim,
                          int metric, int64_t row_offset, int64_t total_rows) {
  return build_impl(h, rows, dtype, n, dim, metric, row_offset, total_rows);
}

int knn_index_build_file(knn_index* h, const char* path, int format, int metric, int n_ranks,
                         int rank) {
  return build_file_impl(h, path, format, metric, n_ranks, rank);
}

int knn_index_copy_rows(knn_index* h, void* out, int dtype) {
  if (!h || !out) return fail(KNN_EINVAL, "null index or output");
  if (!h->data) return fail(KNN_EINVAL, "index has no dataset");
  if (dtype != KNN_DTYPE_F16 && dtype != KNN_DTYPE_F32) return fail(KNN_EINVAL, "unknown dtype");
  std::lock_guard<std::mutex> lock(h->mu);
  KNN_CUDA(cudaSetDevice(h->device));
  const int where = classify(out, h->device);
  if (where < 0) return fail(KNN_EINVAL, "output lives on a different device than the index");
  if (dtype == KNN_DTYPE_F16) {
    KNN_CUDA(cudaMemcpy2DAsync(out, static_cast<size_t>(h->dim) * 2, h->data,
                               static_cast<size_t>(h->ld) * 2, static_cast<size_t>(h->dim) * 2,
                               static_cast<size_t>(h->n), cudaMemcpyDefault, h->stream));
    KNN_CUDA(cudaStreamSynchronize(h->stream));
    return KNN_OK;
  }
  if (h->rows32) {
    // the fp32 rows as given to the build
    KNN_CUDA(cudaMemcpyAsync(out, h->rows32, static_cast<size_t>(h->n) * h->dim * 4,
                             cudaMemcpyDefault, h->stream));
    KNN_CUDA(cudaStreamSynchronize(h->stream));
    return KNN_OK;
  }
  if (where == 1) return fail(KNN_EINVAL, "fp32 rows can only be copied to host memory");
  // widen chunk by chunk through a pinned-free host bounce buffer
  const int64_t chunk = std::max<int64_t>(1, (int64_t(64) << 20) / (h->dim * 2));
  std::vector<__half> tmp(static_cast<size_t>(std::min(chunk, h->n) * h->dim));
  float* dst = static_cast<float*>(out);
  for (int64_t r0 = 0; r0 < h->n; r0 += chunk) {
    const int64_t rr = std::min(chunk, h->n - r0);
    KNN_CUDA(cudaMemcpy2DAsync(tmp.data(), static_cast<size_t>(h->dim) * 2,
                               h->data + static_cast<size_t>(r0) * h->ld,
                               static_cast<size_t>(h->ld) * 2, static_cast<size_t>(h->dim) * 2,
                               static_cast<size_t>(rr), cudaMemcpyDeviceToHost, h->stream));
    KNN_CUDA(cudaStreamSynchronize(h->stream));
    for (int64_t i = 0; i < rr * h->dim; ++i)
      dst[static_cast<size_t>(r0 * h->dim + i)] = __half2float(tmp[static_cast<size_t>(i)]);
  }
  return KNN_OK;
}

int knn_index_build_prepared(knn_index* h, const void* rows_f16, const float* norms,
                             int64_t n, int64_t dim, int metric, int64_t row_offset,
                             int64_t total_rows) {
  return build_prepared_impl(h, rows_f16, norms, n, dim, metric, row_offset, total_rows);
}

int knn_index_device_rows(knn_index* h, const void** rows_f16, int64_t* ld) {
  if (!h || !rows_f16 || !ld) return fail(KNN_EINVAL, "null index or output");
  std::lock_guard<std::mutex> lock(h->mu);
  if (!h->data) return fail(KNN_EINVAL, "index has no dataset");
  *rows_f16 = h->data;
  *ld = h->ld;
  return KNN_OK;
}

int knn_index_device_norms(knn_index* h, const float** norms) {
  if (!h || !norms) return fail(KNN_EINVAL, "null index or output");
  std::lock_guard<std::mutex> lock(h->mu);
  if (!h->data) return fail(KNN_EINVAL, "index has no dataset");
  *norms = h->norms;
  return KNN_OK;
}

int knn_index_device(const knn_index* h) { return h ? h->device : -1; }

int64_t knn_index_rows(const knn_index* h) { return h ? h->n : 0; }
int64_t knn_index_dim(const knn_index* h) { return h ? h->dim : 0; }

int knn_index_search(knn_index* h, const float* queries, int64_t nq, int64_t k,
                     uint32_t* neighbors, float* distances) {
  return search_impl(h, queries, nq, k, neighbors, distances, false, true, false);
}

int knn_index_search_i64(knn_index* h, const float* queries, int64_t nq, int64_t k,
                         int64_t* neighbors, float* distances) {
  return search_impl(h, queries, nq, k, neighbors, distances, true, true, false);
}

int knn_index_search_async(knn_index* h, const float* queries, int64_t nq, int64_t k,
                           uint32_t* neighbors, float* distances) {
  return search_impl(h, queries, nq, k, neighbors, distances, false, false, true);
}

int knn_index_search_lists(knn_index* h, const float* queries, int64_t nq, int64_t k,
                           uint32_t* list_i, float* list_d) {
  return search_impl(h, queries, nq, k, list_i, list_d, false, false, true, true);
}

int knn_merge_lists(int device, void* stream, const float* lists_d, const uint32_t* lists_i,
                    int n_lists, int64_t nq, int64_t k, int metric, void* neighbors,
                    int neighbors_i64, float* distances) {
  if (n_lists <= 0 || nq < 0 || k < 0 || k > KNN_MAX_K)
    return fail(KNN_EINVAL, "knn_merge_lists: n_lists %d, n_queries %lld, k %lld", n_lists,
                (long long)nq, (long long)k);
  if (metric != KNN_METRIC_L2_EXPANDED && metric != KNN_METRIC_INNER_PRODUCT)
    return fail(KNN_EINVAL, "metric %d is not L2Expanded (0) or InnerProduct (1)", metric);
  if (nq == 0 || k == 0) return KNN_OK;
  if (!lists_d || !lists_i || !neighbors || !distances)
    return fail(KNN_EINVAL, "knn_merge_lists: null buffer");
  KNN_CUDA(cudaSetDevice(device));
  for (const void* p : {static_cast<const void*>(lists_d), static_cast<const void*>(lists_i),
                        static_cast<const void*>(neighbors), static_cast<const void*>(distances)})
    if (classify(p, device) != 1)
      return fail(KNN_EINVAL, "knn_merge_lists: every buffer must be memory of device %d", device);
  const int64_t per = nq * k;
  KNN_CUDA(knn::launch_merge(lists_d, lists_i, per, k, n_lists, static_cast<int>(k), nq, 0,
                             distances, neighbors, neighbors_i64 != 0,
                             static_cast<cudaStream_t>(stream),
                             false, nullptr, metric == KNN_METRIC_INNER_PRODUCT, nullptr,
                             per * n_lists));
  g_dispatch.fetch_add(1);
  return KNN_OK;
}

int knn_index_sync(knn_index* h) {
  if (!h) return fail(KNN_EINVAL, "null index");
  std::lock_guard<std::mutex> lock(h->mu);
  KNN_CUDA(cudaSetDevice(h->device));
  KNN_CUDA(cudaMemcpyAsync(h->err_host, h->err_dev, sizeof(int), cudaMemcpyDeviceToHost,
                           h->stream));
  int st = sync_stream(h);
  if (st != KNN_OK) return st;
  if (h->rerank && h->rows32) h->last_uncertified = *h->uncert_host;
  return check_device_error(h);
}

int knn_index_set_rerank(knn_index* h, int enabled) {
  if (!h) return fail(KNN_EINVAL, "null index");
  std::lock_guard<std::mutex> lock(h->mu);
  KNN_CUDA(cudaSetDevice(h->device));
  h->rerank = enabled != 0;
  if (!h->rerank && h->rows32) {
    KNN_CUDA(cudaStreamSynchronize(h->stream));
    cudaFree(h->rows32);
    h->rows32 = nullptr;
  }
  h->last_uncertified = 0;
  h->last_widened = 0;
  ++h->generation;
  drop_graphs(h);
  if (h->rerank && h->data && !h->rows32)
    return fail(KNN_EINVAL,
                "the index was built without its fp32 rows: build it again to re-rank");
  return KNN_OK;
}

int knn_index_rerank_stats(knn_index* h, int64_t* uncertified, int64_t* widened) {
  if (!h) return fail(KNN_EINVAL, "null index");
  std::lock_guard<std::mutex> lock(h->mu);
  if (uncertified) *uncertified = h->last_uncertified;
  if (widened) *widened = h->last_widened;
  return KNN_OK;
}

double knn_rerank_bound(int metric, double r, double query_norm, double row_norm, int64_t dim) {
  if (dim <= 0 || query_norm < 0 || row_norm < 0) return -1.0;
  return knn::rerank_bound(metric, r, query_norm, row_norm, dim);
}

int knn_plan_search(int64_t n_rows, int64_t dim, int64_t nq, int64_t k, int num_sms,
                    knn_plan* out) {
  if (!out) return fail(KNN_EINVAL, "null plan");
  if (n_rows <= 0 || dim <= 0 || nq <= 0 || k <= 0)
    return fail(KNN_EINVAL, "plan needs positive n_rows, dim, n_queries and k");
  Plan p;
  const int st = knn::plan_search(n_rows, dim, nq, k, num_sms, &p);
  if (st != 0) return fail(st, "k = %lld is outside the engine's limits", (long long)k);
  out->query_block = p.query_block;
  out->query_tiles = p.query_tiles;
  out->row_tiles = p.row_tiles;
  out->splits = p.splits;
  out->units = p.units;
  out->grid = p.grid;
  out->stages = p.stages;
  out->smem_bytes = p.smem_bytes;
  out->partial_bytes = p.partial_bytes;
  out->pair = p.pair;
  out->unit_queries = p.unit_queries;
  out->compact_heap = p.compact;
  return KNN_OK;
}

int knn_shard_range(int64_t n_rows, int n_ranks, int rank, int64_t* begin, int64_t* end) {
  if (n_rows < 0 || n_ranks <= 0 || rank < 0 || rank >= n_ranks || !begin || !end)
    return fail(KNN_EINVAL, "invalid shard request");
  const int64_t per = (n_rows + n_ranks - 1) / n_ranks;
  int64_t b = per * rank;
  int64_t e = b + per;
  if (b > n_rows) b = n_rows;
  if (e > n_rows) e = n_rows;
  *begin = b;
  *end = e;
  return KNN_OK;
}

int knn_comm_unique_id(void* out) {
  if (!out) return fail(KNN_EINVAL, "null output");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  ncclUniqueId id;
  if (!nccl().ok) return fail(KNN_ENCCL, "NCCL unavailable: %s", nccl().why.c_str());
  ncclResult_t r = nccl().GetUniqueId(&id);
  if (r != ncclSuccess) return fail(KNN_ENCCL, "ncclGetUniqueId: %s", nccl_str(r));
  std::memcpy(out, &id, sizeof(id));
  return KNN_OK;
}

int knn_index_attach_comm(knn_index* h, const void* uid, int n_ranks, int rank) {
  if (!h || !uid || n_ranks <= 0 || rank < 0 || rank >= n_ranks)
    return fail(KNN_EINVAL, "invalid communicator request");
  std::lock_guard<std::mutex> lock(h->mu);
  KNN_CUDA(cudaSetDevice(h->device));
  if (h->comm) {
    nccl().CommDestroy(h->comm);
    h->comm = nullptr;
  }
  drop_exchange(h);
  ++h->generation;
  drop_graphs(h);
  if (n_ranks == 1) {
    h->n_ranks = 1;
    h->rank = 0;
    return KNN_OK;
  }
  ncclUniqueId id;
  std::memcpy(&id, uid, sizeof(id));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  if (!nccl().ok) return fail(KNN_ENCCL, "NCCL unavailable: %s", nccl().why.c_str());
  ncclResult_t r = nccl().CommInitRankConfig(&h->comm, n_ranks, id, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    h->comm = nullptr;
    return fail(KNN_ENCCL, "ncclCommInitRankConfig: %s", nccl_str(r));
  }
  int st = poll_nccl(h, 120.0);
  if (st != KNN_OK) return st;
  h->n_ranks = n_ranks;
  h->rank = rank;
  return setup_exchange(h);
}

int knn_index_set_peer_exchange(knn_index* h, int enabled) {
  if (!h) return fail(KNN_EINVAL, "null index");
  std::lock_guard<std::mutex> lock(h->mu);
  KNN_CUDA(cudaSetDevice(h->device));
  h->peer_enabled = enabled != 0;
  ++h->generation;
  drop_graphs(h);
  return KNN_OK;
}

int knn_index_set_peer_timeout(knn_index* h, int64_t microseconds) {
  if (!h) return fail(KNN_EINVAL, "null index");
  if (microseconds < 1000 || microseconds > 600000000)
    return fail(KNN_EINVAL, "peer timeout %lld us outside [1 ms, 600 s]",
                (long long)microseconds);
  std::lock_guard<std::mutex> lock(h->mu);
  KNN_CUDA(cudaSetDevice(h->device));
  h->peer_wait_ns = static_cast<uint64_t>(microseconds) * 1000u;
  ++h->generation;  // the bound is a kernel argument of captured searches
  drop_graphs(h);
  return KNN_OK;
}

int knn_index_set_graphs(knn_index* h, int enabled) {
  if (!h) return fail(KNN_EINVAL, "null index");
  std::lock_guard<std::mutex> lock(h->mu);
  KNN_CUDA(cudaSetDevice(h->device));
  drop_graphs(h);
  h->use_graphs = enabled != 0;
  return KNN_OK;
}

int knn_index_set_profiling(knn_index* h, int enabled) {
  if (!h) return fail(KNN_EINVAL, "null index");
  h->profiling = enabled != 0;
  return KNN_OK;
}

int knn_index_kernel_stats(knn_index* h, double* scan_ms, double* merge_ms,
                           int64_t* scan_launches, int64_t* kernel_launches) {
  if (!h) return fail(KNN_EINVAL, "null index");
  {
    std::lock_guard<std::mutex> lock(h->mu);
    KNN_CUDA(cudaSetDevice(h->device));
    KNN_CUDA(cudaStreamSynchronize(h->stream));
    const int st = drain_profile(h);
    if (st != KNN_OK) return st;
  }
  if (scan_ms) *scan_ms = h->scan_ms;
  if (merge_ms) *merge_ms = h->merge_ms;
  if (scan_launches) *scan_launches = h->scan_launches;
  if (kernel_launches) *kernel_launches = h->kernel_launches;
  return KNN_OK;
}

int knn_index_reset_kernel_stats(knn_index* h) {
  if (!h) return fail(KNN_EINVAL, "null index");
  std::lock_guard<std::mutex> lock(h->mu);
  h->prof_used = 0;
  h->scan_ms = h->merge_ms = 0.0;
  h->scan_launches = h->kernel_launches = 0;
  return KNN_OK;
}

int knn_selftest_bounded_wait(int device, int64_t limit_us) {
  if (limit_us <= 0 || limit_us > 2000000) return fail(KNN_EINVAL, "limit_us out of range");
  KNN_CUDA(cudaSetDevice(device));
  int* err = nullptr;
  KNN_CUDA(cudaMalloc(&err, sizeof(int)));
  int host = 0;
  cudaError_t e = cudaMemset(err, 0, sizeof(int));
  if (e == cudaSuccess)
    e = knn::launch_bounded_wait_selftest(err, static_cast<uint64_t>(limit_us) * 1000u, nullptr);
  if (e == cudaSuccess) e = cudaMemcpy(&host, err, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(err);
  if (e != cudaSuccess) return fail(KNN_ECUDA, "self-test: %s", cudaGetErrorString(e));
  g_dispatch.fetch_add(1);
  if (host != 0)
    return fail(KNN_ETIMEOUT, "bounded wait gave up as designed (device code %d)", host);
  return fail(KNN_ECUDA, "bounded wait returned without timing out");
}

uint64_t knn_dispatch_count(void) { return g_dispatch.load(); }
void knn_reset_dispatch_count(void) { g_dispatch.store(0); }

}  // extern "C"

// ---------------------------------------------------------------------------
// Search without allocation (knn_index_search_noalloc).
//
// For callers that must not allocate device memory while they search: code
// that runs under a memory pool or budget owned by someone else (a serving
// framework that has pre-reserved the GPU), code that must not trigger the
// implicit device synchronisation cudaMalloc/cudaFree can cause, or code
// that runs where allocation is forbidden outright.  The per-search scratch
// (fp16 queries, query norms, per-unit top-k lists, and host staging when
// the caller passes host buffers) lives in one file-scope device array of
// KNN_NOALLOC_SCRATCH_BYTES that every GPU loading this library holds until
// the process exits.  The index itself must already be built.
//
// Host code cannot use the array's name as a device address: the address is
// taken with cudaGetSymbolAddress once per device, with that device
// current, on the first call of this entry point on that device; make that
// first call before any stream capture.
//
// Every call on a device shares the one array and it keeps the previous
// call's contents.  Nothing in it needs clearing: each kernel overwrites
// every scratch byte that a later kernel reads (every query row, every
// (query, split, rank) list entry).  Calls through this entry point on the
// same device are serialised by a host lock and each call blocks until its
// results are in place; work that overlaps on the GPU with a call of this
// entry point and also uses this array (for instance from another thread
// that bypasses the call) would race.
static __device__ __align__(256) unsigned char g_noalloc_scratch[KNN_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu[kNoAllocMaxDevices];
void* g_noalloc_base[kNoAllocMaxDevices] = {};

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

int noalloc_search(knn_index* h, const float* queries, int64_t nq, int64_t k,
                   uint32_t* neighbors, float* distances) {
  int st = validate_search(h, queries, nq, k, neighbors, distances);
  if (st != KNN_OK || nq == 0 || k == 0) return st;
  if (h->comm) return fail(KNN_EUNSUPPORTED, "the no-allocation search does not run on a communicator");
  if (h->rerank) return fail(KNN_EUNSUPPORTED, "the no-allocation search does not re-rank");
  if (h->device < 0 || h->device >= kNoAllocMaxDevices)
    return fail(KNN_EUNSUPPORTED, "device %d beyond the no-allocation table", h->device);
  std::lock_guard<std::mutex> dev_lock(g_noalloc_mu[h->device]);
  std::lock_guard<std::mutex> lock(h->mu);
  KNN_CUDA(cudaSetDevice(h->device));
  if (!g_noalloc_base[h->device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(KNN_ECUDA, "cudaGetSymbolAddress(no-allocation scratch): %s",
                  cudaGetErrorString(e));
    g_noalloc_base[h->device] = p;
  }
  unsigned char* base = static_cast<unsigned char*>(g_noalloc_base[h->device]);

  const int cq = classify(queries, h->device);
  const int cn = classify(neighbors, h->device);
  const int cd = classify(distances, h->device);
  if (cq < 0 || cn < 0 || cd < 0)
    return fail(KNN_EINVAL, "buffer lives on a different device than the index");

  Plan plan;
  const int pst = knn::plan_search(h->n, h->dim, nq, k, h->num_sms, &plan);
  if (pst != 0) return fail(pst, "k = %lld is outside the engine's limits", (long long)k);

  // carve the scratch array
  const size_t qk = static_cast<size_t>(nq) * k;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    unsigned char* p = base + off;
    off += align256(bytes);
    return p;
  };
  const int64_t nq_pad = knn::padded_query_rows(plan);
  __half* q16 = reinterpret_cast<__half*>(take(static_cast<size_t>(nq_pad) * h->ld * 2));
  float* qnorm = reinterpret_cast<float*>(take(static_cast<size_t>(nq) * 4));
  float* part_d = reinterpret_cast<float*>(take(static_cast<size_t>(plan.partial_bytes / 2)));
  uint32_t* part_i = reinterpret_cast<uint32_t*>(take(static_cast<size_t>(plan.partial_bytes / 2)));
  float* q32 = cq == 0 ? reinterpret_cast<float*>(take(static_cast<size_t>(nq) * h->dim * 4)) : nullptr;
  float* out_d = cd == 0 ? reinterpret_cast<float*>(take(qk * 4)) : distances;
  uint32_t* out_i = cn == 0 ? reinterpret_cast<uint32_t*>(take(qk * 4)) : neighbors;
  if (off > static_cast<size_t>(KNN_NOALLOC_SCRATCH_BYTES))
    return fail(KNN_EUNSUPPORTED,
                "search needs %zu bytes of scratch; the no-allocation search has %d "
                "(use fewer queries or a smaller k, or knn_index_search)",
                off, KNN_NOALLOC_SCRATCH_BYTES);

  const float* qsrc = queries;
  if (cq == 0) {
    KNN_CUDA(cudaMemcpyAsync(q32, queries, static_cast<size_t>(nq) * h->dim * 4,
                             cudaMemcpyHostToDevice, h->stream));
    qsrc = q32;
  }
  KNN_CUDA(knn::launch_convert_rows(qsrc, false, nq, nq_pad, h->dim, q16, h->ld, qnorm,
                                    h->stream, nullptr, 0, nullptr, plan.spread != 0));
  CUtensorMap qmap;
  if ((st = encode_rows(&qmap, q16, nq_pad, h->ld, knn::kQueryRows)) != KNN_OK) return st;

  knn::ScanParams p;
  p.row_norms = h->norms;
  p.query_norms = qnorm;
  p.part_d = part_d;
  p.part_i = part_i;
  p.err = h->err_dev;
  p.n_rows = h->n;
  p.n_queries = nq;
  p.n_gran = (h->n + plan.gran_rows - 1) / plan.gran_rows;
  p.q_rows = nq_pad;
  p.pair = static_cast<int32_t>(plan.pair);
  p.compact = static_cast<int32_t>(plan.compact);
  p.heap_rows = static_cast<int32_t>(plan.heap_rows);
  p.spread = static_cast<int32_t>(plan.spread);
  p.gran_rows = static_cast<int32_t>(plan.gran_rows);
  p.unit_queries = static_cast<int32_t>(plan.unit_queries);
  p.ld = h->ld;
  p.k = static_cast<int32_t>(k);
  p.query_block = static_cast<int32_t>(plan.query_block);
  p.query_tiles = static_cast<int32_t>(plan.query_tiles);
  p.splits = static_cast<int32_t>(plan.splits);
  p.units = static_cast<int32_t>(plan.units);
  p.k_chunks = static_cast<int32_t>((h->ld + knn::kKChunk - 1) / knn::kKChunk);
  p.stages = static_cast<int32_t>(plan.stages);
  p.dataset_evict_first = plan.query_tiles == 1 ? 1 : 0;
  p.metric = h->metric;
  p.pilot = 0;
  p.pilot_out = nullptr;
  p.thr_init = nullptr;
  p.bound = nullptr;
  KNN_CUDA(knn::launch_scan(qmap, h->xmap, h->xmap_tail, h->xmap_half, p, plan, h->stream));
  KNN_CUDA(knn::launch_merge(part_d, part_i, k, plan.splits * k, static_cast<int>(plan.splits),
                             static_cast<int>(k), nq, h->row_offset, out_d, out_i, false,
                             h->stream, true, nullptr,
                             h->metric == KNN_METRIC_INNER_PRODUCT, h->err_dev,
                             nq * plan.splits * k));
  if (cd == 0)
    KNN_CUDA(cudaMemcpyAsync(distances, out_d, qk * 4, cudaMemcpyDeviceToHost, h->stream));
  if (cn == 0)
    KNN_CUDA(cudaMemcpyAsync(neighbors, out_i, qk * 4, cudaMemcpyDeviceToHost, h->stream));
  g_dispatch.fetch_add(3);
  h->kernel_launches += 3;
  h->scan_launches += 1;
  KNN_CUDA(cudaMemcpyAsync(h->err_host, h->err_dev, sizeof(int), cudaMemcpyDeviceToHost,
                           h->stream));
  KNN_CUDA(cudaStreamSynchronize(h->stream));
  return check_device_error(h);
}

}  // namespace

extern "C" int knn_index_search_noalloc(knn_index* h, const float* queries, int64_t nq,
                                        int64_t k, uint32_t* neighbors, float* distances) {
  return noalloc_search(h, queries, nq, k, neighbors, distances);
}
