// The call pattern of the reference's benchmark CLI
// (tests/test_cohere_wiki_validation.cpp:40-155), against this library:
// headered .bin matrices loaded with cuvs_silicon::load_bin_*, a graph-less
// cagra index built through the cuVS API, saved and loaded in the "CGRA"
// container, searched with the CLI's beam-search knobs (accepted, ignored),
// warm-up then timed iterations, recall@k with the CLI's rule (a returned
// index counts when it appears anywhere in the ground-truth row), and the
// dispatch spy.  The data and the float64 exhaustive ground truth are made
// here (the Cohere files are not available).  argv[1]: a scratch directory.
#include <cuvs/neighbors/cagra.hpp>
#include <cuvs_silicon/sift_loader.hpp>
#include <raft/core/resources.hpp>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <fstream>
#include <numeric>
#include <random>
#include <string>
#include <vector>

namespace cg = cuvs::neighbors::cagra;

template <typename T>
static void write_bin(const std::string& path, std::int32_t rows, std::int32_t cols,
                      const std::vector<T>& v) {
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char*>(&rows), 4);
  f.write(reinterpret_cast<const char*>(&cols), 4);
  f.write(reinterpret_cast<const char*>(v.data()), static_cast<std::streamsize>(v.size() * 4));
}

static double recall(const std::vector<std::uint32_t>& got, const std::vector<std::uint32_t>& gt,
                     std::int64_t q, std::int64_t k) {
  std::int64_t hits = 0;
  for (std::int64_t i = 0; i < q; ++i)
    for (std::int64_t r = 0; r < k; ++r)
      for (std::int64_t g = 0; g < k; ++g)
        if (got[static_cast<size_t>(i * k + r)] == gt[static_cast<size_t>(i * k + g)]) {
          ++hits;
          break;
        }
  return static_cast<double>(hits) / static_cast<double>(q * k);
}

int main(int argc, char** argv) {
  const std::string dir = argc > 1 ? argv[1] : "/tmp";
  const std::int64_t n = 20000, d = 128, q = 200, k = 10;
  std::mt19937 gen(7);
  std::normal_distribution<float> nd(0.0f, 1.0f);
  std::vector<float> base(static_cast<size_t>(n * d)), queries(static_cast<size_t>(q * d));
  for (auto& v : base) v = nd(gen);
  for (auto& v : queries) v = nd(gen);
  // float64 exhaustive ground truth, ties by index
  std::vector<std::int32_t> gt(static_cast<size_t>(q * k));
  std::vector<double> dist(static_cast<size_t>(n));
  std::vector<std::int32_t> order(static_cast<size_t>(n));
  for (std::int64_t i = 0; i < q; ++i) {
    for (std::int64_t r = 0; r < n; ++r) {
      double s = 0.0;
      for (std::int64_t c = 0; c < d; ++c) {
        const double t = static_cast<double>(queries[i * d + c]) - base[r * d + c];
        s += t * t;
      }
      dist[static_cast<size_t>(r)] = s;
    }
    std::iota(order.begin(), order.end(), 0);
    std::partial_sort(order.begin(), order.begin() + k, order.end(), [&](int a, int b) {
      return dist[a] < dist[b] || (dist[a] == dist[b] && a < b);
    });
    std::copy(order.begin(), order.begin() + k, gt.begin() + i * k);
  }
  write_bin(dir + "/base.bin", n, d, base);
  write_bin(dir + "/queries.bin", q, d, queries);
  write_bin(dir + "/gt.bin", q, k, gt);

  // the CLI's sequence
  const auto b = cuvs_silicon::load_bin_f32(dir + "/base.bin");
  const auto qs = cuvs_silicon::load_bin_f32(dir + "/queries.bin");
  const auto g = cuvs_silicon::load_bin_i32(dir + "/gt.bin");
  raft::resources res;
  cg::index_params ip;
  ip.graph_degree = 0;
  auto built = cg::build(res, ip,
                         raft::device_matrix_view<const float, std::int64_t>(
                             b.values.data(), static_cast<std::int64_t>(b.rows),
                             static_cast<std::int64_t>(b.cols)));
  const std::string saved = dir + "/index.cgra";
  cg::save_index(built, saved);
  auto idx = cg::load_index(saved);
  cg::search_params sp;
  sp.itopk_size = 512;
  sp.max_iterations = 600;
  std::vector<std::uint32_t> nbr(static_cast<size_t>(q * k));
  std::vector<float> dst(static_cast<size_t>(q * k));
  auto do_search = [&]() {
    cg::search(res, sp, idx,
               raft::device_matrix_view<const float, std::int64_t>(qs.values.data(), q, d),
               raft::device_matrix_view<std::uint32_t, std::int64_t>(nbr.data(), q, k),
               raft::device_matrix_view<float, std::int64_t>(dst.data(), q, k));
  };
  for (int i = 0; i < 3; ++i) do_search();
  cg::reset_metal_dispatch_count();
  std::vector<double> ms;
  for (int i = 0; i < 20; ++i) {
    const auto t0 = std::chrono::high_resolution_clock::now();
    do_search();
    ms.push_back(std::chrono::duration<double, std::milli>(
                     std::chrono::high_resolution_clock::now() - t0)
                     .count());
  }
  std::sort(ms.begin(), ms.end());
  const double r = recall(nbr, g.neighbors, q, k);
  const auto dispatched = cg::metal_dispatch_count();
  std::printf("cli_test: recall@%lld %.4f  p50 %.3f ms  p99 %.3f ms  dispatches %llu\n",
              static_cast<long long>(k), r, ms[ms.size() / 2], ms.back(),
              static_cast<unsigned long long>(dispatched));
  // fp16 storage may swap exact near-ties at the k-th place only
  if (r < 0.99 || dispatched == 0 || idx.graph_degree() != 0) {
    std::fprintf(stderr, "cli_test: FAILED\n");
    return 1;
  }
  return 0;
}
