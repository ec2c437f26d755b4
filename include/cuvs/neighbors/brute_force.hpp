// cuvs::neighbors::brute_force — exact k-NN index on B200.
//
// No counterpart header exists in the reference (ysys143/cuvs-silicon has
// only cagra.hpp; its exact path is cagra::search on a graph-less index).
// This adds the cuVS brute-force entry points with the caching semantics of
// the reference's MetalContext (src/metal_context.mm:22-55,155-175) moved
// into the index: the index owns the device fp16 rows and the fp32 row norms
// (d_norms), filled at build time, instead of a process-wide cache keyed on
// the dataset pointer.  An index built with a raft::resources that lists
// several devices holds one contiguous row shard per device of this process
// and merges their results on the first device.  An index may also hold one
// row shard of a dataset split across processes (one per GPU), searched
// through an NCCL communicator (include/cuvs_b200.h, knn_index_attach_comm).
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include <cuvs/distance/distance.hpp>
#include <raft/core/resources.hpp>

struct knn_index;  // include/cuvs_b200.h

namespace cuvs::neighbors::brute_force {

struct index_params {
  cuvs::distance::DistanceType metric = cuvs::distance::DistanceType::L2Expanded;
};

struct search_params {};

// One shard's device cache: the fp16 rows (bit patterns, row r starting at
// data + r * ld; the first dim values of a row are its values, the rest
// zero) and, beside it, the fp32 squared norms of those fp16 rows.
struct device_rows_view {
  const std::uint16_t* data = nullptr;
  std::int64_t rows = 0, dim = 0, ld = 0;
};

namespace detail {
struct multi_device_scratch;  // per-index search buffers of a multi-device index
}

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
  int device() const noexcept { return shards_.empty() ? 0 : shards_.front().device; }
  // The first shard's engine handle (the only one for a single-device index).
  knn_index* handle() const noexcept {
    return shards_.empty() ? nullptr : shards_.front().handle.get();
  }

  // Shards: one per device of the resources the index was built with.
  int n_shards() const noexcept { return static_cast<int>(shards_.size()); }
  knn_index* shard_handle(int s) const noexcept { return shards_.at(s).handle.get(); }
  int shard_device(int s) const { return shards_.at(s).device; }
  std::int64_t shard_row_offset(int s) const { return shards_.at(s).row_offset; }
  std::int64_t shard_rows(int s) const { return shards_.at(s).rows; }

  // The device cache the reference's MetalContext keeps per dataset
  // (src/metal_context.mm:38-54,155-175), owned by the index: shard s's
  // fp16 rows and their norms (d_norms), in device memory of
  // shard_device(s).  Valid while the index lives; read only.
  device_rows_view dataset(int s = 0) const;
  raft::device_vector_view<const float, std::int64_t> norms(int s = 0) const;

  // Library-internal: adopt a built engine handle as the next shard.
  void adopt(knn_index* h, std::int64_t rows, std::int64_t dim, std::int64_t row_offset,
             std::int64_t total_rows, cuvs::distance::DistanceType metric, int device);
  detail::multi_device_scratch& scratch() const;

 private:
  struct closer {
    void operator()(knn_index* h) const noexcept;
  };
  struct shard {
    std::unique_ptr<knn_index, closer> handle;
    int device = 0;
    std::int64_t row_offset = 0, rows = 0;
  };
  // Declared before the shards so that it is destroyed after them: it owns
  // the streams the shards' searches ran on.  Created where the type is
  // complete (the library), so this header needs only its declaration.
  mutable std::shared_ptr<detail::multi_device_scratch> scratch_;
  std::vector<shard> shards_;
  std::int64_t rows_ = 0, dim_ = 0, row_offset_ = 0, total_rows_ = 0;
  cuvs::distance::DistanceType metric_ = cuvs::distance::DistanceType::L2Expanded;
};

// Builds an index over `dataset` (host or device, fp32) on resources.device(),
// or, when the resources list several devices, one contiguous row shard
// (knn_shard_range) per device; neighbour indices are global either way.
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
// degree 0 (src/cagra.cpp:268-366).  The metric travels in flag bit 2 (set
// for InnerProduct).  Payloads:
//   fp32 (default): flag bit 0, the rows as fp32 (the fp16 device rows
//     widen exactly), so the reference's own load_index reads the file;
//     loading converts them to fp16 and computes the norms again.
//   fp16_with_norms: flag bit 3 instead of bit 0, the fp16 rows (n x dim x 2
//     bytes) followed by their fp32 norms (n x 4 bytes): half the size, and
//     loading copies both into HBM without converting anything.  The
//     reference's loader sees no dataset block in such a file.
enum class payload { fp32, fp16_with_norms };
void serialize(const raft::resources& res, const std::string& path, const index<float>& idx,
               payload format = payload::fp32);
index<float> deserialize(const raft::resources& res, const std::string& path);

}  // namespace cuvs::neighbors::brute_force
