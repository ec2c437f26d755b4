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

template <>
void index<float>::closer::operator()(knn_index* h) const noexcept {
  knn_index_destroy(h);
}

template <>
void index<float>::adopt(knn_index* h, std::int64_t rows, std::int64_t dim,
                         std::int64_t row_offset, std::int64_t total_rows,
                         cuvs::distance::DistanceType metric, int device) {
  handle_.reset(h);
  rows_ = rows;
  dim_ = dim;
  row_offset_ = row_offset;
  total_rows_ = total_rows;
  metric_ = metric;
  device_ = device;
}

namespace {

index<float> build_impl(const raft::resources& res,
                        raft::device_matrix_view<const float, std::int64_t> rows,
                        std::int64_t row_offset, std::int64_t total_rows,
                        cuvs::distance::DistanceType metric) {
  if (metric != cuvs::distance::DistanceType::L2Expanded &&
      metric != cuvs::distance::DistanceType::InnerProduct)
    throw std::invalid_argument("brute_force supports the L2Expanded and InnerProduct metrics");
  if (rows.data_handle() == nullptr || rows.extent(0) <= 0 || rows.extent(1) <= 0)
    throw std::invalid_argument("brute_force build requires a non-empty dataset");
  knn_index* h = new_handle(res);
  const int st = knn_index_build_shard(h, rows.data_handle(), KNN_DTYPE_F32, rows.extent(0),
                                       rows.extent(1), metric_code(metric), row_offset,
                                       total_rows);
  if (st != KNN_OK) {
    knn_index_destroy(h);
    check(st);
  }
  index<float> idx;
  idx.adopt(h, rows.extent(0), rows.extent(1), row_offset, total_rows, metric, res.device());
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
  if (res.cuda_stream()) check(knn_index_set_stream(idx.handle(), res.cuda_stream()));
  check(knn_index_search(idx.handle(), queries.data_handle(), queries.extent(0),
                         neighbors.extent(1), neighbors.data_handle(),
                         distances.data_handle()));
}

void serialize(const raft::resources& res, const std::string& path, const index<float>& idx) {
  (void)res;
  if (!idx.handle()) throw std::invalid_argument("serialize: empty index");
  std::vector<float> rows(static_cast<std::size_t>(idx.size() * idx.dim()));
  check(knn_index_copy_rows(idx.handle(), rows.data(), KNN_DTYPE_F32));
  std::ofstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("serialize: cannot open " + path);
  Header h;
  h.n = idx.size();
  h.d = idx.dim();
  h.g = 0;
  h.flags = 1u;
  if (idx.metric() == cuvs::distance::DistanceType::InnerProduct) h.flags |= kFlagInnerProduct;
  write_header(f, h);
  put_vec(f, rows.data(), rows.size());
  if (!f) throw std::runtime_error("serialize: write failed");
}

index<float> deserialize(const raft::resources& res, const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("deserialize: cannot open " + path);
  const Header h = read_header(f, path);
  if (!(h.flags & 1u)) throw std::invalid_argument("deserialize: file holds no dataset");
  std::vector<float> rows;
  get_vec(f, rows, static_cast<std::size_t>(h.n * h.d));
  if (!f) throw std::runtime_error("deserialize: read failed");
  return build(res,
               raft::make_device_matrix_view<const float, std::int64_t>(rows.data(), h.n, h.d),
               (h.flags & kFlagInnerProduct) ? cuvs::distance::DistanceType::InnerProduct
                                             : cuvs::distance::DistanceType::L2Expanded);
}

}  // namespace cuvs::neighbors::brute_force
