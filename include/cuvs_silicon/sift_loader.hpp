// cuvs_silicon SIFT / fvecs / ivecs loaders.
//
// Same declarations as the reference's include/cuvs_silicon/sift_loader.hpp
// (names, structs, constants and the SiftLoadError exception type), so
// callers and the reference's own tests/test_sift_loader.cpp compile against
// this library unchanged.  The implementation (src/loaders.cpp) is this
// repository's: files are read in large blocks and every record header is
// checked while the payload is compacted, instead of one stream read per
// field.
//
// Formats (the TEXMEX corpus layout):
//   fvecs: per row, int32 d then d float32;
//   ivecs: per row, int32 d then d int32 (ground-truth neighbour ids, >= 0).
// Every loader checks the exact shape it is asked for: the row count, every
// row's width, and that the file ends where the last expected row ends; any
// mismatch, a negative neighbour id or an I/O failure throws SiftLoadError.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace cuvs_silicon {

constexpr std::size_t kSift1MBaseVectorCount = 1'000'000;
constexpr std::size_t kSift1MQueryVectorCount = 10'000;
constexpr std::size_t kSift1MVectorDimension = 128;
constexpr std::size_t kSift1MGroundTruthNeighborCount = 100;

class SiftLoadError : public std::runtime_error {
 public:
  explicit SiftLoadError(const std::string& message);
};

struct FloatVectorDataset {
  std::size_t rows = 0;
  std::size_t cols = 0;
  std::vector<float> values;  // rows x cols, row-major, contiguous
};

struct GroundTruthDataset {
  std::size_t query_count = 0;
  std::size_t neighbor_count = 0;
  std::vector<std::uint32_t> neighbors;  // query_count x neighbor_count
};

struct SiftDataset {
  FloatVectorDataset base;
  FloatVectorDataset queries;
  GroundTruthDataset groundtruth;
};

FloatVectorDataset load_fvecs(const std::string& path, std::size_t expected_rows,
                              std::size_t expected_cols);

// Checks the record headers and the file length without keeping the payload.
void validate_fvecs_shape(const std::string& path, std::size_t expected_rows,
                          std::size_t expected_cols);

GroundTruthDataset load_ivecs(const std::string& path, std::size_t expected_rows,
                              std::size_t expected_cols);

// Loads base, queries and ground truth and checks that they fit together:
// equal dimensions, one ground-truth row per query, every neighbour id a
// base row ("outside base rows" otherwise).
SiftDataset load_sift_dataset(const std::string& base_path, const std::string& query_path,
                              const std::string& groundtruth_path,
                              std::size_t expected_base_rows, std::size_t expected_query_rows,
                              std::size_t expected_cols,
                              std::size_t expected_groundtruth_cols);

FloatVectorDataset load_sift1m_base(const std::string& path);
void validate_sift1m_base_shape(const std::string& path);
FloatVectorDataset load_sift1m_queries(const std::string& path);
GroundTruthDataset load_sift1m_groundtruth(const std::string& path);
SiftDataset load_sift1m_dataset(const std::string& base_path, const std::string& query_path,
                                const std::string& groundtruth_path);

// ---------------------------------------------------------------- .bin
// The headered binary matrices of the reference's Cohere-wiki benchmark
// (tests/test_cohere_wiki_validation.cpp:40-52, written by
// scripts/download_cohere_wiki.py): int32 rows, int32 cols, then rows x cols
// values (float32 vectors, or int32 ground-truth ids).  Not part of the
// reference's loader header; the benchmark reads them with a file-local
// helper.  Throws SiftLoadError on a negative or truncated shape, a short
// payload or trailing bytes.
FloatVectorDataset load_bin_f32(const std::string& path);
GroundTruthDataset load_bin_i32(const std::string& path);

}  // namespace cuvs_silicon
