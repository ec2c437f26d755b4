// raft::resources and raft::device_matrix_view for the B200 exact k-NN engine.
//
// Source-compatible with the shim the reference ships
// (include/raft/core/resources.hpp:8-45 of ysys143/cuvs-silicon): the same
// class and function names, constructors and accessors, so code written
// against the reference compiles unchanged.  Differences: `resources` also
// carries a CUDA device ordinal (or a list of devices for an index sharded
// across the GPUs of one process) and an optional caller-owned cudaStream_t
// (held as void* so this header needs no CUDA include), and sync_stream()
// really waits for that stream.  A device_matrix_view is still a raw
// pointer plus extents; the pointer may be host or device memory.
#pragma once

#include <cstddef>
#include <cstdint>
#include <utility>
#include <vector>

namespace raft {

class resources {
 public:
  resources() = default;
  explicit resources(int device, void* cuda_stream = nullptr) noexcept
      : device_(device), stream_(cuda_stream) {}
  // Several CUDA devices of this process: a brute_force index built with
  // these resources holds one contiguous row shard per device, and its
  // searches run on all of them and merge on the first.  device() is the
  // first of the list.
  explicit resources(std::vector<int> devices)
      : device_(devices.empty() ? 0 : devices.front()), devices_(std::move(devices)) {}

  int device() const noexcept { return device_; }
  // The devices an index built with these resources spans ({device()} when
  // no list was given).
  std::vector<int> devices() const {
    return devices_.empty() ? std::vector<int>{device_} : devices_;
  }
  void* cuda_stream() const noexcept { return stream_; }
  void set_device(int device) noexcept {
    device_ = device;
    devices_.clear();
  }
  void set_cuda_stream(void* stream) noexcept { stream_ = stream; }

  // Waits for the work queued on this handle's stream (no-op without one).
  void sync_stream() const;

 private:
  int device_ = 0;
  void* stream_ = nullptr;
  std::vector<int> devices_;
};

// A raw pointer and a length (the 1-D counterpart of device_matrix_view).
template <typename ElementType, typename IndexType = std::int64_t>
class device_vector_view {
 public:
  using element_type = ElementType;
  using index_type = IndexType;
  constexpr device_vector_view(ElementType* data, IndexType n) noexcept : ptr_(data), n_(n) {}
  constexpr ElementType* data_handle() const noexcept { return ptr_; }
  constexpr IndexType extent(std::size_t) const noexcept { return n_; }
  constexpr IndexType size() const noexcept { return n_; }

 private:
  ElementType* ptr_;
  IndexType n_;
};

template <typename ElementType, typename IndexType = std::int64_t>
class device_matrix_view {
 public:
  using element_type = ElementType;
  using index_type = IndexType;

  constexpr device_matrix_view(ElementType* data, IndexType rows, IndexType cols) noexcept
      : ptr_(data), rows_(rows), cols_(cols) {}

  constexpr ElementType* data_handle() const noexcept { return ptr_; }
  constexpr ElementType* data() const noexcept { return ptr_; }
  constexpr IndexType extent(std::size_t axis) const noexcept {
    return axis == 0 ? rows_ : cols_;
  }
  constexpr IndexType size() const noexcept { return rows_ * cols_; }

 private:
  ElementType* ptr_;
  IndexType rows_;
  IndexType cols_;
};

template <typename ElementType, typename IndexType>
constexpr device_matrix_view<ElementType, IndexType> make_device_matrix_view(
    ElementType* data, IndexType rows, IndexType cols) noexcept {
  return device_matrix_view<ElementType, IndexType>(data, rows, cols);
}

}  // namespace raft
