// Loader checks that need no GPU: the .bin matrices of the Cohere-wiki
// benchmark (int32 rows, int32 cols, payload; the format read by the
// reference's tests/test_cohere_wiki_validation.cpp:40-52) and fvecs error
// reporting of this implementation.  argv[1]: a scratch directory.
#include <cuvs_silicon/sift_loader.hpp>

#include <cstdint>
#include <cstdio>
#include <fstream>
#include <functional>
#include <string>
#include <vector>

static int g_failures = 0;
#define EXPECT(c)                                                         \
  do {                                                                    \
    if (!(c)) {                                                           \
      std::fprintf(stderr, "%s:%d: expectation failed: %s\n", __FILE__, __LINE__, #c); \
      ++g_failures;                                                       \
    }                                                                     \
  } while (0)

static bool load_error(const std::function<void()>& f, const char* needle) {
  try {
    f();
  } catch (const cuvs_silicon::SiftLoadError& e) {
    return std::string(e.what()).find(needle) != std::string::npos;
  }
  return false;
}

template <typename T>
static void write_bin(const std::string& path, std::int32_t rows, std::int32_t cols,
                      const std::vector<T>& v, int extra = 0) {
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char*>(&rows), 4);
  f.write(reinterpret_cast<const char*>(&cols), 4);
  f.write(reinterpret_cast<const char*>(v.data()), static_cast<std::streamsize>(v.size() * 4));
  for (int i = 0; i < extra; ++i) f.put('\0');
}

int main(int argc, char** argv) {
  const std::string dir = argc > 1 ? argv[1] : "/tmp";
  const std::string p = dir + "/m.bin";
  std::vector<float> vals(3 * 5);
  for (std::size_t i = 0; i < vals.size(); ++i) vals[i] = 0.5f * static_cast<float>(i) - 2.0f;
  write_bin(p, 3, 5, vals);
  const auto ds = cuvs_silicon::load_bin_f32(p);
  EXPECT(ds.rows == 3 && ds.cols == 5 && ds.values == vals);

  write_bin(p, 3, 5, vals, 4);
  EXPECT(load_error([&] { cuvs_silicon::load_bin_f32(p); }, "after its payload"));
  write_bin(p, 4, 5, vals);
  EXPECT(load_error([&] { cuvs_silicon::load_bin_f32(p); }, "truncated"));
  write_bin(p, -1, 5, vals);
  EXPECT(load_error([&] { cuvs_silicon::load_bin_f32(p); }, "negative shape"));
  EXPECT(load_error([&] { cuvs_silicon::load_bin_f32(dir + "/missing.bin"); }, "cannot open"));

  const std::vector<std::int32_t> gt = {0, 7, 3, 2, 9, 1};
  write_bin(p, 2, 3, gt);
  const auto g = cuvs_silicon::load_bin_i32(p);
  EXPECT(g.query_count == 2 && g.neighbor_count == 3);
  EXPECT((g.neighbors == std::vector<std::uint32_t>{0, 7, 3, 2, 9, 1}));
  write_bin(p, 2, 3, std::vector<std::int32_t>{0, 7, -3, 2, 9, 1});
  EXPECT(load_error([&] { cuvs_silicon::load_bin_i32(p); }, "negative id"));

  // fvecs spanning several read blocks (64 MiB): 40,000 rows of 512 floats
  const std::string fv = dir + "/big.fvecs";
  {
    std::ofstream f(fv, std::ios::binary);
    std::vector<float> row(512);
    const std::int32_t w = 512;
    for (int r = 0; r < 40000; ++r) {
      for (int c = 0; c < 512; ++c) row[c] = static_cast<float>(r) + c * 1e-3f;
      f.write(reinterpret_cast<const char*>(&w), 4);
      f.write(reinterpret_cast<const char*>(row.data()), 512 * 4);
    }
  }
  const auto big = cuvs_silicon::load_fvecs(fv, 40000, 512);
  EXPECT(big.values.size() == 40000u * 512u);
  EXPECT(big.values[39999u * 512u + 7] == 39999.0f + 7 * 1e-3f);
  EXPECT(big.values[33000u * 512u] == 33000.0f);
  EXPECT(load_error([&] { cuvs_silicon::load_fvecs(fv, 40001, 512); }, "before the width header"));
  EXPECT(load_error([&] { cuvs_silicon::load_fvecs(fv, 39999, 512); }, "bytes after"));
  EXPECT(load_error([&] { cuvs_silicon::load_fvecs(fv, 40000, 511); }, "has width 512"));
  cuvs_silicon::validate_fvecs_shape(fv, 40000, 512);
  std::remove(fv.c_str());
  std::remove(p.c_str());

  if (g_failures) {
    std::fprintf(stderr, "%d expectation(s) failed\n", g_failures);
    return 1;
  }
  std::printf("loader_test: all expectations passed\n");
  return 0;
}
