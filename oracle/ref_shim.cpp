// ref_shim.cpp -- C entry points over the reference's OWN exact search.
//
// TEST INFRASTRUCTURE ONLY.  Compiled together with the unmodified reference
// sources (src/cagra.cpp, src/distance.cpp of ysys143/cuvs-silicon) into
// oracle/_ref/libref_cagra.so by oracle/Makefile.  On a non-Apple host the
// reference's cuvs::neighbors::cagra::search is exactly its CPU exact path
// (src/cagra.cpp:211-252), so these functions run the reference itself.
// The product library never loads this file.
#include <cstdint>
#include <stdexcept>
#include <string>

#include <cuvs/neighbors/cagra.hpp>
#include <cuvs_silicon/distance.hpp>

namespace {
thread_local std::string g_err;
}

extern "C" {

// Runs cagra::build (src/cagra.cpp:20-88, graph_degree ignored off-Apple)
// and cagra::search (src/cagra.cpp:90-253) through the reference's public
// API.  Returns 0 on success, 1 for std::invalid_argument, 2 for any other
// exception (message in ref_last_error()).
int ref_cagra_knn(const float* base, std::int64_t n, std::int64_t dim,
                  const float* queries, std::int64_t nq, std::int64_t k,
                  std::uint32_t* out_idx, float* out_dist,
                  int attach_dataset) {
  try {
    raft::resources res;
    cuvs::neighbors::cagra::index_params ip;
    ip.metric = cuvs::distance::DistanceType::L2Expanded;
    ip.graph_degree = 0;
    ip.attach_dataset_on_build = attach_dataset != 0;
    auto idx = cuvs::neighbors::cagra::build(
        res, ip,
        raft::make_device_matrix_view<const float, std::int64_t>(base, n, dim));
    cuvs::neighbors::cagra::search_params sp;
    cuvs::neighbors::cagra::search(
        res, sp, idx,
        raft::make_device_matrix_view<const float, std::int64_t>(queries, nq, dim),
        raft::make_device_matrix_view<std::uint32_t, std::int64_t>(out_idx, nq, k),
        raft::make_device_matrix_view<float, std::int64_t>(out_dist, nq, k));
    return 0;
  } catch (const std::invalid_argument& e) {
    g_err = e.what();
    return 1;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 2;
  }
}

// The reference's metric-validation behaviour: build with a non-L2 metric.
int ref_cagra_build_inner_product(const float* base, std::int64_t n,
                                  std::int64_t dim) {
  try {
    raft::resources res;
    cuvs::neighbors::cagra::index_params ip;
    ip.metric = cuvs::distance::DistanceType::InnerProduct;
    auto idx = cuvs::neighbors::cagra::build(
        res, ip,
        raft::make_device_matrix_view<const float, std::int64_t>(base, n, dim));
    (void)idx;
    return 0;
  } catch (const std::invalid_argument& e) {
    g_err = e.what();
    return 1;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 2;
  }
}

// The reference's own container code (src/cagra.cpp:268-366): cagra::build
// with the dataset attached, then cagra::save_index(path).  Used to check
// that files written by either side load on the other.
int ref_cagra_save_index(const float* base, std::int64_t n, std::int64_t dim,
                         const char* path) {
  try {
    raft::resources res;
    cuvs::neighbors::cagra::index_params ip;
    ip.metric = cuvs::distance::DistanceType::L2Expanded;
    ip.graph_degree = 0;
    auto idx = cuvs::neighbors::cagra::build(
        res, ip,
        raft::make_device_matrix_view<const float, std::int64_t>(base, n, dim));
    cuvs::neighbors::cagra::save_index(idx, path);
    return 0;
  } catch (const std::invalid_argument& e) {
    g_err = e.what();
    return 1;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 2;
  }
}

// cagra::load_index(path) and the reference's search on the loaded index;
// *rows / *dim receive the loaded shape.
int ref_cagra_load_search(const char* path, const float* queries, std::int64_t nq,
                          std::int64_t k, std::uint32_t* out_idx, float* out_dist,
                          std::int64_t* rows, std::int64_t* dim) {
  try {
    raft::resources res;
    auto idx = cuvs::neighbors::cagra::load_index(path);
    *rows = idx.rows();
    *dim = idx.cols();
    cuvs::neighbors::cagra::search_params sp;
    cuvs::neighbors::cagra::search(
        res, sp, idx,
        raft::make_device_matrix_view<const float, std::int64_t>(queries, nq, idx.cols()),
        raft::make_device_matrix_view<std::uint32_t, std::int64_t>(out_idx, nq, k),
        raft::make_device_matrix_view<float, std::int64_t>(out_dist, nq, k));
    return 0;
  } catch (const std::invalid_argument& e) {
    g_err = e.what();
    return 1;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 2;
  }
}

// src/distance.cpp:8-20.
float ref_squared_l2_distance_128(const float* a, const float* b) {
  return cuvs_silicon::squared_l2_distance_128(a, b);
}

const char* ref_last_error() { return g_err.c_str(); }

}  // extern "C"
