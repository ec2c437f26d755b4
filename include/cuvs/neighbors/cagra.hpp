// cuvs::neighbors::cagra for the B200 exact k-NN engine.
//
// Source-compatible with the reference's header
// (include/cuvs/neighbors/cagra.hpp:12-124 of ysys143/cuvs-silicon): the same
// enums, parameter structs, index accessors and free functions, so the
// reference's callers (its FAISS adapter, its benchmark CLI, its dispatch-spy
// test) compile unchanged.  Behaviour is the reference's non-Apple path,
// where no graph is built (src/cagra.cpp:44-85 is Apple-only) and search is
// exact: search runs on the B200 engine (include/cuvs_b200.h) instead of
// the CPU loop of src/cagra.cpp:211-252, with the same output contract.
//
// The index keeps the reference's host copy of the dataset when
// attach_dataset_on_build is set (cagra.cpp:38-42) and, in addition, a
// handle to the device copy (fp16 rows + fp32 norms in HBM), created at
// build or, for an index made by the constructor or load_index, at the first
// search.  Copies of an index share that device copy.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

#include <cuvs/distance/distance.hpp>
#include <raft/core/resources.hpp>

namespace cuvs::neighbors::detail {
// Owner of one device index (defined in the library).
struct device_dataset;
std::shared_ptr<device_dataset> make_device_dataset();
}  // namespace cuvs::neighbors::detail

namespace cuvs::neighbors::cagra {

enum class search_algo {
  SINGLE_CTA = 0,
  MULTI_CTA = 1,
  MULTI_KERNEL = 2,
  AUTO = 100,
};

enum class hash_mode {
  HASH = 0,
  SMALL = 1,
  AUTO = 100,
};

// graph_degree and the graph-build knobs are accepted and ignored: like the
// reference off Apple, the index never carries a graph.
struct index_params {
  std::uint32_t intermediate_graph_degree = 128;
  std::uint32_t graph_degree = 64;
  bool attach_dataset_on_build = true;
  bool guarantee_connectivity = false;
  cuvs::distance::DistanceType metric = cuvs::distance::DistanceType::L2Expanded;
};

// Beam-search knobs, accepted and ignored: search is exact.
struct search_params {
  std::uint64_t max_queries = 0;
  std::uint64_t itopk_size = 64;
  std::uint64_t max_iterations = 0;
  search_algo algo = search_algo::AUTO;
  std::uint64_t team_size = 0;
  std::uint64_t search_width = 1;
  std::uint64_t min_iterations = 0;
  std::uint64_t thread_block_size = 0;
  hash_mode hashmap_mode = hash_mode::AUTO;
  std::uint64_t hashmap_min_bitlen = 0;
  float hashmap_max_fill_rate = 0.5F;
  std::uint32_t num_random_samplings = 1;
  std::uint64_t rand_xor_mask = 0x128394;
};

template <typename DataT, typename IndexT = std::uint32_t>
class index {
  static_assert(std::is_same_v<IndexT, std::uint32_t>,
                "the cuVS-compatible exact index reports uint32_t neighbour indices");

 public:
  using value_type = DataT;
  using index_type = IndexT;

  index() : device_(detail::make_device_dataset()) {}
  index(std::vector<DataT> dataset, std::int64_t rows, std::int64_t cols)
      : dataset_(std::move(dataset)),
        rows_(rows),
        cols_(cols),
        device_(detail::make_device_dataset()) {}

  const std::vector<DataT>& dataset() const noexcept { return dataset_; }
  const std::vector<IndexT>& knn_graph() const noexcept { return knn_graph_; }
  std::int64_t rows() const noexcept { return rows_; }
  std::int64_t cols() const noexcept { return cols_; }
  std::uint32_t graph_degree() const noexcept { return graph_degree_; }

  void set_knn_graph(std::vector<IndexT> g, std::uint32_t degree) {
    knn_graph_ = std::move(g);
    graph_degree_ = degree;
  }

  const std::vector<IndexT>& nav_nodes() const noexcept { return nav_nodes_; }
  const std::vector<DataT>& nav_vectors() const noexcept { return nav_vectors_; }
  void set_nav_nodes(std::vector<IndexT> n) { nav_nodes_ = std::move(n); }
  void set_nav_vectors(std::vector<DataT> v) { nav_vectors_ = std::move(v); }

  // Device copy of the dataset (shared by copies of this index).
  const std::shared_ptr<detail::device_dataset>& device() const noexcept { return device_; }

 private:
  std::vector<DataT> dataset_;
  std::vector<IndexT> knn_graph_;
  std::vector<IndexT> nav_nodes_;
  std::vector<DataT> nav_vectors_;
  std::uint32_t graph_degree_ = 0;
  std::int64_t rows_ = 0;
  std::int64_t cols_ = 0;
  std::shared_ptr<detail::device_dataset> device_;
};

// Validates (L2Expanded only; non-null, non-empty dataset), keeps a host copy
// when attach_dataset_on_build and loads the device copy.  Throws
// std::invalid_argument like src/cagra.cpp:26-32, std::runtime_error on
// device errors.
template <typename DataT, typename ExtentT>
index<DataT, std::uint32_t> build(const raft::resources& resources, const index_params& params,
                                  raft::device_matrix_view<const DataT, ExtentT> dataset);

// Exact k-NN (k = neighbors.extent(1)) on the B200 engine.  Squared L2,
// ascending by (distance, index); k > rows padded with UINT32_MAX / +inf.
// Throws std::invalid_argument for null buffers, dimension or shape
// mismatches (src/cagra.cpp:100-111) and for an index without a dataset.
template <typename DataT, typename IndexT, typename ExtentT>
void search(const raft::resources& resources, const search_params& params,
            const index<DataT, IndexT>& index,
            raft::device_matrix_view<const DataT, ExtentT> queries,
            raft::device_matrix_view<IndexT, ExtentT> neighbors,
            raft::device_matrix_view<float, ExtentT> distances);

// Reference container format "CGRA" v1 (src/cagra.cpp:268-366): magic,
// version, N, D, graph degree, flags (bit0 dataset, bit1 nav), graph,
// dataset, nav.  Files are interchangeable with the reference's.
void save_index(const index<float, std::uint32_t>& idx, const std::string& path);
index<float, std::uint32_t> load_index(const std::string& path);

// Dispatch spy (cagra.hpp:119-122 of the reference): counts the engine's
// kernel launches since the last reset, plus explicit increments.
std::uint64_t metal_dispatch_count() noexcept;
void reset_metal_dispatch_count() noexcept;
void increment_metal_dispatch_count() noexcept;

}  // namespace cuvs::neighbors::cagra
