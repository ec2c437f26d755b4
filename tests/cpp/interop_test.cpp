// interop_test.cpp -- container files between this library and the
// reference's own code (src/cagra.cpp:268-366, compiled as a test oracle).
//
//   interop_test write <index.bin> <rows.f32> <n> <d>
//       brute_force::build + brute_force::serialize (fp32 payload): a file
//       the reference's cagra::load_index must read.
//   interop_test read <index.bin> <queries.f32> <nq> <k> <out.u32> <out.f32>
//       a file the reference's cagra::save_index wrote: loaded here with
//       cagra::load_index + cagra::search and with brute_force::deserialize +
//       search; both results must agree; the first is written out.
// Raw files are row-major little-endian arrays.  Exit code 0 = success.
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <string>
#include <vector>

#include <cuvs/neighbors/brute_force.hpp>
#include <cuvs/neighbors/cagra.hpp>
#include <raft/core/resources.hpp>

namespace cg = cuvs::neighbors::cagra;
namespace bf = cuvs::neighbors::brute_force;

template <typename T>
static std::vector<T> read_raw(const std::string& path, std::size_t count) {
  std::vector<T> v(count);
  std::ifstream f(path, std::ios::binary);
  f.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(count * sizeof(T)));
  if (!f) {
    std::fprintf(stderr, "cannot read %zu values from %s\n", count, path.c_str());
    std::exit(2);
  }
  return v;
}

template <typename T>
static void write_raw(const std::string& path, const std::vector<T>& v) {
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char*>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(T)));
  if (!f) std::exit(2);
}

int main(int argc, char** argv) {
  if (argc < 2) return 2;
  const std::string mode = argv[1];
  raft::resources res;
  try {
    if (mode == "write" && argc == 6) {
      const std::int64_t n = std::atoll(argv[4]), d = std::atoll(argv[5]);
      const auto rows = read_raw<float>(argv[3], static_cast<std::size_t>(n * d));
      auto idx = bf::build(res, raft::make_device_matrix_view<const float, std::int64_t>(rows.data(), n, d));
      bf::serialize(res, argv[2], idx);
      std::printf("wrote %lld x %lld\n", static_cast<long long>(n), static_cast<long long>(d));
      return 0;
    }
    if (mode == "read" && argc == 8) {
      const std::int64_t nq = std::atoll(argv[4]), k = std::atoll(argv[5]);
      auto ci = cg::load_index(argv[2]);
      const std::int64_t d = ci.cols();
      const auto qs = read_raw<float>(argv[3], static_cast<std::size_t>(nq * d));
      std::vector<std::uint32_t> i1(static_cast<std::size_t>(nq * k)), i2(i1.size());
      std::vector<float> d1(i1.size()), d2(i1.size());
      cg::search(res, cg::search_params{}, ci,
                 raft::make_device_matrix_view<const float, std::int64_t>(qs.data(), nq, d),
                 raft::make_device_matrix_view<std::uint32_t, std::int64_t>(i1.data(), nq, k),
                 raft::make_device_matrix_view<float, std::int64_t>(d1.data(), nq, k));
      auto bi = bf::deserialize(res, argv[2]);
      bf::search(res, bi, raft::make_device_matrix_view<const float, std::int64_t>(qs.data(), nq, d),
                 raft::make_device_matrix_view<std::uint32_t, std::int64_t>(i2.data(), nq, k),
                 raft::make_device_matrix_view<float, std::int64_t>(d2.data(), nq, k));
      if (i1 != i2 || d1 != d2) {
        std::fprintf(stderr, "cagra::load_index and brute_force::deserialize disagree\n");
        return 1;
      }
      write_raw(argv[6], i1);
      write_raw(argv[7], d1);
      std::printf("read %lld x %lld\n", static_cast<long long>(ci.rows()), static_cast<long long>(d));
      return 0;
    }
  } catch (const std::exception& e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 1;
  }
  return 2;
}
