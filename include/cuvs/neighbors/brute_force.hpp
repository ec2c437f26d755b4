// cuvs::neighbors::brute_force — exact k-NN index on B200.
//
// No counterpart header exists in the reference (ysys143/cuvs-silicon has
// only cagra.hpp; its exact path is cagra::search on a graph-less index).
// This adds the cuVS brute-force entry points with the caching semantics of
// the reference's MetalContext (src/metal_context.mm:22-55,155-175) moved
// into the index: the index owns the device fp16 rows and the fp32 row norms
// (d_norms), filled at build time, instead of a process-wide cache keyed on
// the dataset pointer.  An index may also hold one row shard of a larger
// dataset, searched across GPUs through an NCCL communicator
// (include/cuvs_b200.h, knn_index_attach_comm).
#pragma once

#include <cstdint>
#include <memory>
#include <string>

#include <cuvs/distance/distance.hpp>
#include <raft/core/resources.hpp>

struct knn_index;  // include/cuvs_b200.h

namespace cuvs::neighbors::brute_force {

struct index_params {
  cuvs::distance::DistanceType metric = cuvs::distance::DistanceType::L2Expanded;
};

struct search_params {};

template <typename T>
class index {
 public:
  index() = default;
  index(index&&) noexcept = default;
  index& operator=(index&&) noexcept = default;
  index(const index&) = delete;
  index& operator=(const index&) = delete;

  std::int64_t size() const noexcept { return rows_; }   // rows held by this index
  std::int64_t dim() const noexcept { return dim_; }
  std::int64_t row_offset() const noexcept { return row_offset_; }
  std::int64_t total_rows() const noexcept { return total_rows_; }
  cuvs::distance::DistanceType metric() const noexcept { return metric_; }
  int device() const noexcept { return device_; }
  knn_index* handle() const noexcept { return handle_.get(); }

  // Library-internal: adopt a built engine handle.
  void adopt(knn_index* h, std::int64_t rows, std::int64_t dim, std::int64_t row_offset,
             std::int64_t total_rows, cuvs::distance::DistanceType metric, int device);

 private:
  struct closer {
    void operator()(knn_index* h) const noexcept;
  };
  std::unique_ptr<knn_index, closer> handle_;
  std::int64_t rows_ = 0, dim_ = 0, row_offset_ = 0, total_rows_ = 0;
  cuvs::distance::DistanceType metric_ = cuvs::distance::DistanceType::L2Expanded;
  int device_ = 0;
};

// Builds an index over `dataset` (host or device, fp32) on resources.device().
index<float> build(const raft::resources& res,
                   raft::device_matrix_view<const float, std::int64_t> dataset,
                   cuvs::distance::DistanceType metric = cuvs::distance::DistanceType::L2Expanded);
index<float> build(const raft::resources& res, const index_params& params,
                   raft::device_matrix_view<const float, std::int64_t> dataset);

// One row shard: rows [row_offset, row_offset + dataset.extent(0)) of a
// total_rows-row dataset; reported neighbour indices are global.
index<float> build_shard(const raft::resources& res,
                         raft::device_matrix_view<const float, std::int64_t> shard,
                         std::int64_t row_offset, std::int64_t total_rows,
                         cuvs::distance::DistanceType metric =
                             cuvs::distance::DistanceType::L2Expanded);

// Exact k-NN, k = neighbors.extent(1).  int64 neighbours follow upstream
// cuVS (missing neighbours are -1); uint32 neighbours follow the reference's
// cagra contract (missing = UINT32_MAX).  L2Expanded: distances are squared
// L2, ascending.  InnerProduct: distances are the inner products q.x,
// descending (largest first), ties by ascending index, missing = -inf.
void search(const raft::resources& res, const search_params& params, const index<float>& idx,
            raft::device_matrix_view<const float, std::int64_t> queries,
            raft::device_matrix_view<std::int64_t, std::int64_t> neighbors,
            raft::device_matrix_view<float, std::int64_t> distances);
void search(const raft::resources& res, const index<float>& idx,
            raft::device_matrix_view<const float, std::int64_t> queries,
            raft::device_matrix_view<std::int64_t, std::int64_t> neighbors,
            raft::device_matrix_view<float, std::int64_t> distances);
void search(const raft::resources& res, const index<float>& idx,
            raft::device_matrix_view<const float, std::int64_t> queries,
            raft::device_matrix_view<std::uint32_t, std::int64_t> neighbors,
            raft::device_matrix_view<float, std::int64_t> distances);

// Saves / loads an index in the reference's "CGRA" v1 container with graph
// degree 0 and the dataset present (src/cagra.cpp:268-366); the rows are
// written as fp32 (the fp16 device rows widen exactly) so the reference can
// read the file, and loading rebuilds the device copy.  The metric travels
// in flag bit 2 (set for InnerProduct).
void serialize(const raft::resources& res, const std::string& path, const index<float>& idx);
index<float> deserialize(const raft::resources& res, const std::string& path);

}  // namespace cuvs::neighbors::brute_force
