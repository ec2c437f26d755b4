// cuvs_api.cpp -- the cuVS-compatible C++ API over the engine's C ABI.
//
// cagra::build / cagra::search keep the reference's declarations and
// validation (src/cagra.cpp:20-253) and run the exact search on the B200
// engine; brute_force::* are the cuVS brute-force entry points the engine
// adds.  Status codes from include/cuvs_b200.h become exceptions:
// KNN_EINVAL -> std::invalid_argument, everything else -> std::runtime_error,
// as the reference throws.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <limits>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuvs/neighbors/brute_force.hpp>
#include <cuvs/neighbors/cagra.hpp>
#include <cuvs_b200.h>

namespace {

void check(int status) {
  if (status == KNN_OK) return;
  const std::string msg = std::string(knn_status_string(status)) + ": " + knn_last_error();
  if (status == KNN_EINVAL) throw std::invalid_argument(msg);
  throw std::runtime_error(msg);
}

knn_index* new_handle(const raft::resources& res) {
  knn_index* h = nullptr;
  check(knn_index_create(res.device(), &h));
  if (res.cuda_stream()) {
    const int st = knn_index_set_stream(h, res.cuda_stream());
    if (st != KNN_OK) {
      knn_index_destroy(h);
      check(st);
    }
  }
  return h;
}

int metric_code(cuvs::distance::DistanceType m) {
  return m == cuvs::distance::DistanceType::L2Expanded ? KNN_METRIC_L2_EXPANDED
                                                       : KNN_METRIC_INNER_PRODUCT;
}

std::atomic<std::uint64_t> g_manual_dispatches{0};

// "CGRA" v1 container (src/cagra.cpp:268-276): magic, u32 version, i64 N,
// i64 D, u32 graph degree, u32 flags (bit0 dataset, bit1 nav), then the
// dataset (fp32), the graph (u32), and the navigation block.  Flag bit 2
// (unused by the reference, whose loader tests bits 0 and 1 only) marks a
// brute-force index built for the InnerProduct metric.
constexpr char kMagic[4] = {'C', 'G', 'R', 'A'};
constexpr std::uint32_t kFlagInnerProduct = 4u;

template <typename T>
void put(std::ofstream& f, const T& v) {
  f.write(reinterpret_cast<const char*>(&v), sizeof(T));
}
template <typename T>
T get(std::ifstream& f) {
  T v{};
  f.read(reinterpret_cast<char*>(&v), sizeof(T));
  return v;
}
template <typename T>
void put_vec(std::ofstream& f, const T* p, std::size_t n) {
  f.write(reinterpret_cast<const char*>(p), static_cast<std::streamsize>(n * sizeof(T)));
}
template <typename T>
void get_vec(std::ifstream& f, std::vector<T>& v, std::size_t n) {
  v.resize(n);
  f.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(n * sizeof(T)));
}

struct Header {
  std::int64_t n = 0, d = 0;
  std::uint32_t g = 0, flags = 0;
};

void write_header(std::ofstream& f, const Header& h) {
  f.write(kMagic, 4);
  put<std::uint32_t>(f, 1u);
  put(f, h.n);
  put(f, h.d);
  put(f, h.g);
  put(f, h.flags);
}

Header read_header(std::ifstream& f, const std::string& path) {
  char magic[4] = {};
  f.read(magic, 4);
  if (!f || std::memcmp(magic, kMagic, 4) != 0)
    throw std::runtime_error("load_index: invalid magic in " + path);
  if (get<std::uint32_t>(f) != 1u) throw std::runtime_error("load_index: unsupported version");
  Header h;
  h.n = get<std::int64_t>(f);
  h.d = get<std::int64_t>(f);
  h.g = get<std::uint32_t>(f);
  h.flags = get<std::uint32_t>(f);
  if (!f || h.n < 0 || h.d < 0) throw std::runtime_error("load_index: truncated header");
  return h;
}

}  // namespace

// ------------------------------------------------------------------ raft
void raft::resources::sync_stream() const {
  if (!stream_) return;
  cudaSetDevice(device_);
  const cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream_));
  if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
}

// ------------------------------------------------------- device dataset
namespace cuvs::neighbors::detail {

struct device_dataset {
  std::mutex mu;
  knn_index* handle = nullptr;
  ~device_dataset() {
    if (handle) knn_index_destroy(handle);
  }
};

std::shared_ptr<device_dataset> make_device_dataset() {
  return std::make_shared<device_dataset>();
}

}  // namespace cuvs::neighbors::detail

// ------------------------------------------------------------------ cagra
namespace cuvs::neighbors::cagra {

template <>
index<float, std::uint32_t> build<float, std::int64_t>(
    const raft::resources& res, const index_params& params,
    raft::device_matrix_view<const float, std::int64_t> dataset) {
  if (params.metric != cuvs::distance::DistanceType::L2Expanded)
    throw std::invalid_argument("the exact cagra index supports L2Expanded");
  if (dataset.data_handle() == nullptr || dataset.extent(0) <= 0 || dataset.extent(1) <= 0)
    throw std::invalid_argument("cagra build requires a non-empty dataset");
  const std::int64_t n = dataset.extent(0);
  const std::int64_t d = dataset.extent(1);
  std::vector<float> host;
  if (params.attach_dataset_on_build) {
    // The reference keeps a host copy (src/cagra.cpp:38-42); rows may live
    // on the device here, so copy with the runtime.
    host.resize(static_cast<std::size_t>(n * d));
    const cudaError_t e = cudaMemcpy(host.data(), dataset.data_handle(),
                                     host.size() * sizeof(float), cudaMemcpyDefault);
    if (e != cudaSuccess) {
      cudaGetLastError();
      std::memcpy(host.data(), dataset.data_handle(), host.size() * sizeof(float));
    }
  }
  index<float, std::uint32_t> idx(std::move(host), n, d);
  if (params.attach_dataset_on_build) {
    auto& dev = *idx.device();
    std::lock_guard<std::mutex> lock(dev.mu);
    dev.handle = new_handle(res);
    check(knn_index_build(dev.handle, dataset.data_handle(), KNN_DTYPE_F32, n, d,
                          KNN_METRIC_L2_EXPANDED));
  }
  return idx;
}

template <>
void search<float, std::uint32_t, std::int64_t>(
    const raft::resources& res, const search_params& params,
    const index<float, std::uint32_t>& idx,
    raft::device_matrix_view<const float, std::int64_t> queries,
    raft::device_matrix_view<std::uint32_t, std::int64_t> neighbors,
    raft::device_matrix_view<float, std::int64_t> distances) {
  (void)params;
  if (queries.data_handle() == nullptr || neighbors.data_handle() == nullptr ||
      distances.data_handle() == nullptr)
    throw std::invalid_argument("cagra search requires valid buffers");
  if (queries.extent(1) != idx.cols())
    throw std::invalid_argument("cagra search: query dimension mismatch");
  if (neighbors.extent(0) != queries.extent(0) || distances.extent(0) != queries.extent(0) ||
      neighbors.extent(1) != distances.extent(1))
    throw std::invalid_argument("cagra search: output shape mismatch");
  const std::int64_t q = queries.extent(0);
  const std::int64_t k = neighbors.extent(1);
  if (q == 0 || k == 0) return;
  auto& dev = *idx.device();
  std::lock_guard<std::mutex> lock(dev.mu);
  if (!dev.handle) {
    // index made by the constructor or load_index: build the device copy now
    // from the host rows (the reference's first-search cache fill,
    // src/metal_context.mm:155-175, but owned by the index)
    if (idx.dataset().empty() || idx.rows() <= 0)
      throw std::invalid_argument(
          "cagra search: the index holds no dataset (built with "
          "attach_dataset_on_build = false)");
    if (static_cast<std::int64_t>(idx.dataset().size()) != idx.rows() * idx.cols())
      throw std::invalid_argument("cagra search: dataset size does not match rows x cols");
    knn_index* h = new_handle(res);
    const int st = knn_index_build(h, idx.dataset().data(), KNN_DTYPE_F32, idx.rows(),
                                   idx.cols(), KNN_METRIC_L2_EXPANDED);
    if (st != KNN_OK) {
      knn_index_destroy(h);
      check(st);
    }
    dev.handle = h;
  }
  if (res.cuda_stream()) check(knn_index_set_stream(dev.handle, res.cuda_stream()));
  check(knn_index_search(dev.handle, queries.data_handle(), q, k, neighbors.data_handle(),
                         distances.data_handle()));
}

void save_index(const index<float, std::uint32_t>& idx, const std::string& path) {
  std::ofstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("save_index: cannot open " + path);
  Header h;
  h.n = idx.rows();
  h.d = idx.cols();
  h.g = idx.graph_degree();
  const bool has_dataset = !idx.dataset().empty();
  const bool has_nav = !idx.nav_nodes().empty();
  h.flags = (has_dataset ? 1u : 0u) | (has_nav ? 2u : 0u);
  write_header(f, h);
  if (has_dataset) put_vec(f, idx.dataset().data(), idx.dataset().size());
  put_vec(f, idx.knn_graph().data(), idx.knn_graph().size());
  if (has_nav) {
    put<std::uint32_t>(f, static_cast<std::uint32_t>(idx.nav_nodes().size()));
    put_vec(f, idx.nav_nodes().data(), idx.nav_nodes().size());
    put_vec(f, idx.nav_vectors().data(), idx.nav_vectors().size());
  }
  if (!f) throw std::runtime_error("save_index: write failed");
}

index<float, std::uint32_t> load_index(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("load_index: cannot open " + path);
  const Header h = read_header(f, path);
  std::vector<float> data;
  if (h.flags & 1u) get_vec(f, data, static_cast<std::size_t>(h.n * h.d));
  index<float, std::uint32_t> idx(std::move(data), h.n, h.d);
  std::vector<std::uint32_t> graph;
  get_vec(f, graph, static_cast<std::size_t>(h.n) * h.g);
  idx.set_knn_graph(std::move(graph), h.g);
  if (h.flags & 2u) {
    const auto nn = get<std::uint32_t>(f);
    std::vector<std::uint32_t> nodes;
    std::vector<float> vecs;
    get_vec(f, nodes, nn);
    get_vec(f, vecs, static_cast<std::size_t>(nn) * static_cast<std::size_t>(h.d));
    idx.set_nav_nodes(std::move(nodes));
    idx.set_nav_vectors(std::move(vecs));
  }
  if (!f) throw std::runtime_error("load_index: read failed");
  return idx;
}

std::uint64_t metal_dispatch_count() noexcept {
  return knn_dispatch_count() + g_manual_dispatches.load();
}

void reset_metal_dispatch_count() noexcept {
  knn_reset_dispatch_count();
  g_manual_dispatches.store(0);
}

void increment_metal_dispatch_count() noexcept { g_manual_dispatches.fetch_add(1); }

}  // namespace cuvs::neighbors::cagra

// ------------------------------------------------------------ brute_force
namespace cuvs::neighbors::brute_force {

namespace detail {

// Device buffer on one device that only grows (multi-device search scratch).
struct dev_buf {
  int device = -1;
  void* ptr = nullptr;
  std::size_t bytes = 0;
  void ensure(int dev, std::size_t need) {
    if (dev == device && need <= bytes) return;
    release();
    if (cudaSetDevice(dev) != cudaSuccess || cudaMalloc(&ptr, need) != cudaSuccess) {
      cudaGetLastError();
      ptr = nullptr;
      throw std::runtime_error("brute_force: device allocation of " + std::to_string(need) +
                               " bytes failed on device " + std::to_string(dev));
    }
    device = dev;
    bytes = need;
  }
  void release() noexcept {
    if (ptr) {
      cudaSetDevice(device);
      cudaFree(ptr);
    }
    ptr = nullptr;
    bytes = 0;
  }
  template <typename T>
  T* as() const {
    return static_cast<T*>(ptr);
  }
  ~dev_buf() { release(); }
};

// Per-index state of a search over several devices: one stream, one event
// and query / list buffers per shard on the shard's device, the gathered
// lists and the merged result on the first shard's device.
struct multi_device_scratch {
  std::mutex mu;
  std::vector<int> devices;
  std::vector<cudaStream_t> streams;
  std::vector<cudaEvent_t> done;
  std::vector<dev_buf> q, li, ld;
  dev_buf gi, gd, oi, od;
  ~multi_device_scratch() {
    for (std::size_t s = 0; s < streams.size(); ++s) {
      cudaSetDevice(devices[s]);
      cudaStreamSynchronize(streams[s]);
      cudaStreamDestroy(streams[s]);
      cudaEventDestroy(done[s]);
    }
  }
};

}  // namespace detail

template <>
void index<float>::closer::operator()(knn_index* h) const noexcept {
  knn_index_destroy(h);
}

template <>
void index<float>::adopt(knn_index* h, std::int64_t rows, std::int64_t dim,
                         std::int64_t row_offset, std::int64_t total_rows,
                         cuvs::distance::DistanceType metric, int device) {
  shard sh;
  sh.handle.reset(h);
  sh.device = device;
  sh.row_offset = row_offset;
  sh.rows = rows;
  if (shards_.empty()) {
    rows_ = 0;
    row_offset_ = row_offset;
  }
  shards_.push_back(std::move(sh));
  rows_ += rows;
  dim_ = dim;
  total_rows_ = total_rows;
  metric_ = metric;
}

template <>
detail::multi_device_scratch& index<float>::scratch() const {
  if (!scratch_) scratch_ = std::make_shared<detail::multi_device_scratch>();
  return *scratch_;
}

template <>
device_rows_view index<float>::dataset(int s) const {
  const void* p = nullptr;
  std::int64_t ld = 0;
  check(knn_index_device_rows(shard_handle(s), &p, &ld));
  device_rows_view v;
  v.data = static_cast<const std::uint16_t*>(p);
  v.rows = shard_rows(s);
  v.dim = dim_;
  v.ld = ld;
  return v;
}

template <>
raft::device_vector_view<const float, std::int64_t> index<float>::norms(int s) const {
  const float* p = nullptr;
  check(knn_index_device_norms(shard_handle(s), &p));
  return raft::device_vector_view<const float, std::int64_t>(p, shard_rows(s));
}

namespace {

// -1 host memory, else the device whose memory p is.
int memory_device(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) ? a.device : -1;
}

// Builds one shard on `device` from rows that may live on another device
// (copied there first) or in host memory.
knn_index* build_one(const raft::resources& res, int device, const float* rows,
                     std::int64_t n, std::int64_t d, std::int64_t row_offset,
                     std::int64_t total_rows, cuvs::distance::DistanceType metric) {
  raft::resources one(device, device == res.device() ? res.cuda_stream() : nullptr);
  knn_index* h = new_handle(one);
  detail::dev_buf tmp;
  const int where = memory_device(rows);
  if (where >= 0 && where != device) {
    try {
      tmp.ensure(device, static_cast<std::size_t>(n * d) * sizeof(float));
    } catch (...) {
      knn_index_destroy(h);
      throw;
    }
    if (cudaMemcpyPeer(tmp.ptr, device, rows, where, static_cast<std::size_t>(n * d) * 4) !=
        cudaSuccess) {
      knn_index_destroy(h);
      throw std::runtime_error("brute_force: copying a shard between devices failed");
    }
    rows = tmp.as<float>();
  }
  const int st = knn_index_build_shard(h, rows, KNN_DTYPE_F32, n, d, metric_code(metric),
                                       row_offset, total_rows);
  if (st != KNN_OK) {
    knn_index_destroy(h);
    check(st);
  }
  return h;
}

index<float> build_impl(const raft::resources& res,
                        raft::device_matrix_view<const float, std::int64_t> rows,
                        std::int64_t row_offset, std::int64_t total_rows,
                        cuvs::distance::DistanceType metric) {
  if (metric != cuvs::distance::DistanceType::L2Expanded &&
      metric != cuvs::distance::DistanceType::InnerProduct)
    throw std::invalid_argument("brute_force supports the L2Expanded and InnerProduct metrics");
  if (rows.data_handle() == nullptr || rows.extent(0) <= 0 || rows.extent(1) <= 0)
    throw std::invalid_argument("brute_force build requires a non-empty dataset");
  const std::vector<int> devices = res.devices();
  const std::int64_t n = rows.extent(0), d = rows.extent(1);
  index<float> idx;
  if (devices.size() == 1) {
    knn_index* h = new_handle(res);
    const int st = knn_index_build_shard(h, rows.data_handle(), KNN_DTYPE_F32, n, d,
                                         metric_code(metric), row_offset, total_rows);
    if (st != KNN_OK) {
      knn_index_destroy(h);
      check(st);
    }
    idx.adopt(h, n, d, row_offset, total_rows, metric, res.device());
    return idx;
  }
  if (row_offset != 0 || total_rows != n)
    throw std::invalid_argument("brute_force: a multi-device index holds a whole dataset");
  const int parts = static_cast<int>(devices.size());
  for (int s = 0; s < parts; ++s) {
    std::int64_t b = 0, e = 0;
    check(knn_shard_range(n, parts, s, &b, &e));
    if (e <= b) throw std::invalid_argument("brute_force: fewer rows than devices");
    knn_index* h = build_one(res, devices[static_cast<std::size_t>(s)],
                             rows.data_handle() + b * d, e - b, d, b, n, metric);
    idx.adopt(h, e - b, d, b, n, metric, devices[static_cast<std::size_t>(s)]);
  }
  return idx;
}

void check_shapes(const index<float>& idx, std::int64_t qrows, std::int64_t qcols,
                  std::int64_t nrows, std::int64_t ncols, std::int64_t drows,
                  std::int64_t dcols, const void* q, const void* n, const void* d) {
  if (!idx.handle()) throw std::invalid_argument("brute_force search on an empty index");
  if (!q || !n || !d) throw std::invalid_argument("brute_force search requires valid buffers");
  if (qcols != idx.dim()) throw std::invalid_argument("brute_force search: dimension mismatch");
  if (nrows != qrows || drows != qrows || ncols != dcols)
    throw std::invalid_argument("brute_force search: output shape mismatch");
}

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string("brute_force: ") + what + ": " + cudaGetErrorString(e));
  }
}

// Search over the shards of a multi-device index: every shard searches its
// rows on its own device and stream (knn_index_search_lists, global row
// indices), the lists are copied to the first shard's device, and one merge
// kernel there (knn_merge_lists) writes the result; the call blocks like a
// single-device search.
void search_shards(const raft::resources& res, const index<float>& idx, const float* queries,
                   std::int64_t nq, std::int64_t k, void* neighbors, bool i64,
                   float* distances) {
  (void)res;
  if (nq == 0 || k == 0) return;
  if (k > KNN_MAX_K) check(KNN_EUNSUPPORTED);
  auto& sc = idx.scratch();
  std::lock_guard<std::mutex> lock(sc.mu);
  const int parts = idx.n_shards();
  if (sc.streams.empty()) {
    for (int s = 0; s < parts; ++s) {
      const int dev = idx.shard_device(s);
      cudaStream_t st = nullptr;
      cudaEvent_t ev = nullptr;
      cuda_check(cudaSetDevice(dev), "set device");
      cuda_check(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "stream");
      cuda_check(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event");
      sc.devices.push_back(dev);
      sc.streams.push_back(st);
      sc.done.push_back(ev);
    }
    sc.q.resize(static_cast<std::size_t>(parts));
    sc.li.resize(static_cast<std::size_t>(parts));
    sc.ld.resize(static_cast<std::size_t>(parts));
  }
  const int dev0 = idx.shard_device(0);
  const std::size_t qk = static_cast<std::size_t>(nq * k);
  const std::size_t qbytes = static_cast<std::size_t>(nq * idx.dim()) * sizeof(float);
  sc.gd.ensure(dev0, qk * parts * sizeof(float));
  sc.gi.ensure(dev0, qk * parts * sizeof(std::uint32_t));
  sc.od.ensure(dev0, qk * sizeof(float));
  sc.oi.ensure(dev0, qk * (i64 ? 8 : 4));
  for (int s = 0; s < parts; ++s) {
    const int dev = idx.shard_device(s);
    const auto u = static_cast<std::size_t>(s);
    sc.q[u].ensure(dev, qbytes);
    sc.li[u].ensure(dev, qk * sizeof(std::uint32_t));
    sc.ld[u].ensure(dev, qk * sizeof(float));
  }
  for (int s = 0; s < parts; ++s) {
    const auto u = static_cast<std::size_t>(s);
    cuda_check(cudaSetDevice(idx.shard_device(s)), "set device");
    cuda_check(cudaMemcpyAsync(sc.q[u].ptr, queries, qbytes, cudaMemcpyDefault, sc.streams[u]),
               "query upload");
    check(knn_index_set_stream(idx.shard_handle(s), sc.streams[u]));
    check(knn_index_search_lists(idx.shard_handle(s), sc.q[u].as<float>(), nq, k,
                                 sc.li[u].as<std::uint32_t>(), sc.ld[u].as<float>()));
    cuda_check(cudaMemcpyAsync(sc.gd.as<float>() + qk * u, sc.ld[u].ptr, qk * sizeof(float),
                               cudaMemcpyDefault, sc.streams[u]),
               "list gather");
    cuda_check(cudaMemcpyAsync(sc.gi.as<std::uint32_t>() + qk * u, sc.li[u].ptr,
                               qk * sizeof(std::uint32_t), cudaMemcpyDefault, sc.streams[u]),
               "list gather");
    cuda_check(cudaEventRecord(sc.done[u], sc.streams[u]), "event");
  }
  cuda_check(cudaSetDevice(dev0), "set device");
  for (int s = 1; s < parts; ++s)
    cuda_check(cudaStreamWaitEvent(sc.streams[0], sc.done[static_cast<std::size_t>(s)], 0),
               "wait");
  const int metric = metric_code(idx.metric());
  check(knn_merge_lists(dev0, sc.streams[0], sc.gd.as<float>(), sc.gi.as<std::uint32_t>(), parts,
                        nq, k, metric, sc.oi.ptr, i64 ? 1 : 0, sc.od.as<float>()));
  cuda_check(cudaMemcpyAsync(distances, sc.od.ptr, qk * sizeof(float), cudaMemcpyDefault,
                             sc.streams[0]),
             "result download");
  cuda_check(cudaMemcpyAsync(neighbors, sc.oi.ptr, qk * (i64 ? 8 : 4), cudaMemcpyDefault,
                             sc.streams[0]),
             "result download");
  cuda_check(cudaStreamSynchronize(sc.streams[0]), "search");
  // device-side errors of every shard's kernels (bounded waits, debug
  // checks); then every shard goes back to its own stream, so no handle
  // keeps a stream of this scratch
  int first_error = KNN_OK;
  for (int s = 0; s < parts; ++s) {
    const int st = knn_index_sync(idx.shard_handle(s));
    if (first_error == KNN_OK) first_error = st;
    knn_index_set_stream(idx.shard_handle(s), nullptr);
  }
  check(first_error);
}

}  // namespace

index<float> build(const raft::resources& res,
                   raft::device_matrix_view<const float, std::int64_t> dataset,
                   cuvs::distance::DistanceType metric) {
  return build_impl(res, dataset, 0, dataset.extent(0), metric);
}

index<float> build(const raft::resources& res, const index_params& params,
                   raft::device_matrix_view<const float, std::int64_t> dataset) {
  return build_impl(res, dataset, 0, dataset.extent(0), params.metric);
}

index<float> build_shard(const raft::resources& res,
                         raft::device_matrix_view<const float, std::int64_t> shard,
                         std::int64_t row_offset, std::int64_t total_rows,
                         cuvs::distance::DistanceType metric) {
  if (res.devices().size() != 1)
    throw std::invalid_argument("brute_force::build_shard takes resources of one device");
  return build_impl(res, shard, row_offset, total_rows, metric);
}

void search(const raft::resources& res, const search_params& params, const index<float>& idx,
            raft::device_matrix_view<const float, std::int64_t> queries,
            raft::device_matrix_view<std::int64_t, std::int64_t> neighbors,
            raft::device_matrix_view<float, std::int64_t> distances) {
  (void)params;
  search(res, idx, queries, neighbors, distances);
}

void search(const raft::resources& res, const index<float>& idx,
            raft::device_matrix_view<const float, std::int64_t> queries,
            raft::device_matrix_view<std::int64_t, std::int64_t> neighbors,
            raft::device_matrix_view<float, std::int64_t> distances) {
  check_shapes(idx, queries.extent(0), queries.extent(1), neighbors.extent(0),
               neighbors.extent(1), distances.extent(0), distances.extent(1),
               queries.data_handle(), neighbors.data_handle(), distances.data_handle());
  if (idx.n_shards() > 1) {
    search_shards(res, idx, queries.data_handle(), queries.extent(0), neighbors.extent(1),
                  neighbors.data_handle(), true, distances.data_handle());
    return;
  }
  if (res.cuda_stream()) check(knn_index_set_stream(idx.handle(), res.cuda_stream()));
  check(knn_index_search_i64(idx.handle(), queries.data_handle(), queries.extent(0),
                             neighbors.extent(1), neighbors.data_handle(),
                             distances.data_handle()));
}

void search(const raft::resources& res, const index<float>& idx,
            raft::device_matrix_view<const float, std::int64_t> queries,
            raft::device_matrix_view<std::uint32_t, std::int64_t> neighbors,
            raft::device_matrix_view<float, std::int64_t> distances) {
  check_shapes(idx, queries.extent(0), queries.extent(1), neighbors.extent(0),
               neighbors.extent(1), distances.extent(0), distances.extent(1),
               queries.data_handle(), neighbors.data_handle(), distances.data_handle());
  if (idx.n_shards() > 1) {
    search_shards(res, idx, queries.data_handle(), queries.extent(0), neighbors.extent(1),
                  neighbors.data_handle(), false, distances.data_handle());
    return;
  }
  if (res.cuda_stream()) check(knn_index_set_stream(idx.handle(), res.cuda_stream()));
  check(knn_index_search(idx.handle(), queries.data_handle(), queries.extent(0),
                         neighbors.extent(1), neighbors.data_handle(),
                         distances.data_handle()));
}

// Flag bit 3: the dataset block holds fp16 rows followed by fp32 norms.
constexpr std::uint32_t kFlagFp16Payload = 8u;

void serialize(const raft::resources& res, const std::string& path, const index<float>& idx,
               payload format) {
  (void)res;
  if (!idx.handle()) throw std::invalid_argument("serialize: empty index");
  const std::int64_t n = idx.size(), d = idx.dim();
  std::ofstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("serialize: cannot open " + path);
  Header h;
  h.n = n;
  h.d = d;
  h.g = 0;
  h.flags = format == payload::fp32 ? 1u : kFlagFp16Payload;
  if (idx.metric() == cuvs::distance::DistanceType::InnerProduct) h.flags |= kFlagInnerProduct;
  write_header(f, h);
  if (format == payload::fp32) {
    std::vector<float> rows(static_cast<std::size_t>(n * d));
    for (int s = 0; s < idx.n_shards(); ++s)
      check(knn_index_copy_rows(idx.shard_handle(s),
                                rows.data() + (idx.shard_row_offset(s) - idx.row_offset()) * d,
                                KNN_DTYPE_F32));
    put_vec(f, rows.data(), rows.size());
  } else {
    std::vector<std::uint16_t> rows(static_cast<std::size_t>(n * d));
    std::vector<float> norms(static_cast<std::size_t>(n));
    for (int s = 0; s < idx.n_shards(); ++s) {
      const std::int64_t at = idx.shard_row_offset(s) - idx.row_offset();
      check(knn_index_copy_rows(idx.shard_handle(s), rows.data() + at * d, KNN_DTYPE_F16));
      const auto nv = idx.norms(s);
      cuda_check(cudaMemcpy(norms.data() + at, nv.data_handle(),
                            static_cast<std::size_t>(nv.size()) * sizeof(float),
                            cudaMemcpyDeviceToHost),
                 "norm download");
    }
    put_vec(f, rows.data(), rows.size());
    put_vec(f, norms.data(), norms.size());
  }
  if (!f) throw std::runtime_error("serialize: write failed");
}

index<float> deserialize(const raft::resources& res, const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("deserialize: cannot open " + path);
  const Header h = read_header(f, path);
  const auto metric = (h.flags & kFlagInnerProduct) ? cuvs::distance::DistanceType::InnerProduct
                                                    : cuvs::distance::DistanceType::L2Expanded;
  if (h.flags & kFlagFp16Payload) {
    std::vector<std::uint16_t> rows;
    std::vector<float> norms;
    get_vec(f, rows, static_cast<std::size_t>(h.n * h.d));
    get_vec(f, norms, static_cast<std::size_t>(h.n));
    if (!f) throw std::runtime_error("deserialize: read failed");
    if (h.n <= 0 || h.d <= 0) throw std::invalid_argument("deserialize: empty dataset");
    const std::vector<int> devices = res.devices();
    const int parts = static_cast<int>(devices.size());
    index<float> idx;
    for (int s = 0; s < parts; ++s) {
      std::int64_t b = 0, e = 0;
      check(knn_shard_range(h.n, parts, s, &b, &e));
      if (e <= b) throw std::invalid_argument("deserialize: fewer rows than devices");
      raft::resources one(devices[static_cast<std::size_t>(s)],
                          parts == 1 ? res.cuda_stream() : nullptr);
      knn_index* hd = new_handle(one);
      const int st = knn_index_build_prepared(hd, rows.data() + b * h.d, norms.data() + b,
                                              e - b, h.d, metric_code(metric), b, h.n);
      if (st != KNN_OK) {
        knn_index_destroy(hd);
        check(st);
      }
      idx.adopt(hd, e - b, h.d, b, h.n, metric, devices[static_cast<std::size_t>(s)]);
    }
    return idx;
  }
  if (!(h.flags & 1u)) throw std::invalid_argument("deserialize: file holds no dataset");
  std::vector<float> rows;
  get_vec(f, rows, static_cast<std::size_t>(h.n * h.d));
  if (!f) throw std::runtime_error("deserialize: read failed");
  return build(res,
               raft::make_device_matrix_view<const float, std::int64_t>(rows.data(), h.n, h.d),
               metric);
}

}  // namespace cuvs::neighbors::brute_force
