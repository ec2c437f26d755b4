// Dataset file loaders: the cuvs_silicon fvecs / ivecs / SIFT API
// (include/cuvs_silicon/sift_loader.hpp; behaviour of the reference's
// src/sift_loader.cpp:21-215) and the headered .bin matrices of the
// Cohere-wiki benchmark.
//
// Records are read in blocks of whole records (up to 64 MiB) with POSIX
// read(); each block's record headers are checked and the payloads copied
// into the contiguous result, so a 1M x 128 file takes a few dozen system
// calls instead of millions of stream reads.
#include <cuvs_silicon/sift_loader.hpp>

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <limits>
#include <string>
#include <vector>

namespace cuvs_silicon {

SiftLoadError::SiftLoadError(const std::string& message) : std::runtime_error(message) {}

namespace {

std::size_t mul_checked(std::size_t a, std::size_t b, const char* what) {
  if (b != 0 && a > std::numeric_limits<std::size_t>::max() / b)
    throw SiftLoadError(std::string(what) + ": shape overflows size_t");
  return a * b;
}

// Owns a read-only file descriptor.
class File {
 public:
  File(const std::string& path, const char* kind) : path_(path) {
    fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd_ < 0)
      throw SiftLoadError(std::string("cannot open ") + kind + " file " + path + ": " +
                          std::strerror(errno));
    struct stat st;
    if (::fstat(fd_, &st) != 0) {
      ::close(fd_);
      throw SiftLoadError("cannot stat " + path);
    }
    size_ = static_cast<std::size_t>(st.st_size);
  }
  ~File() { ::close(fd_); }
  File(const File&) = delete;
  File& operator=(const File&) = delete;

  std::size_t size() const { return size_; }

  // Reads exactly n bytes at the current position (n may be 0).
  void read_exact(void* dst, std::size_t n) {
    auto* p = static_cast<char*>(dst);
    while (n > 0) {
      const ssize_t r = ::read(fd_, p, n);
      if (r < 0 && errno == EINTR) continue;
      if (r <= 0) throw SiftLoadError("read failed on " + path_);
      p += r;
      n -= static_cast<std::size_t>(r);
    }
  }

 private:
  std::string path_;
  int fd_ = -1;
  std::size_t size_ = 0;
};

// Walks a "vecs" file (per record: int32 width, then width 4-byte values)
// expecting `rows` records of width `cols`.  For every block of whole
// records, `sink(block_bytes, first_row, n_rows)` receives the raw records
// (headers already checked).  Errors name what was wrong, in the order a
// sequential reader meets them: a short header, a wrong width, a short
// payload, then bytes after the last expected record.
template <typename Sink>
void walk_vecs(const std::string& path, const char* kind, std::size_t rows, std::size_t cols,
               Sink&& sink) {
  File f(path, kind);
  const std::size_t rec = mul_checked(cols, 4, kind) + 4;
  const std::size_t want = mul_checked(rec, rows, kind);
  constexpr std::size_t kBlock = std::size_t(64) << 20;
  const std::size_t per_block = rec >= kBlock ? 1 : kBlock / rec;
  std::vector<char> buf(std::min(per_block, std::max<std::size_t>(rows, 1)) * rec);
  const std::size_t avail = f.size();
  std::size_t row = 0;
  while (row < rows) {
    const std::size_t nr = std::min(per_block, rows - row);
    const std::size_t start = row * rec;
    // records of this block that are complete in the file
    const std::size_t have = avail > start ? (avail - start) : 0;
    const std::size_t full = std::min(nr, have / rec);
    const std::size_t take = full * rec + (full < nr ? std::min(have - full * rec, rec) : 0);
    f.read_exact(buf.data(), take);
    for (std::size_t r = 0; r < nr; ++r) {
      const char* h = buf.data() + r * rec;
      const std::size_t left = take - std::min(take, r * rec);
      if (left < 4)
        throw SiftLoadError(std::string(kind) + " file ended before the width header of row " +
                            std::to_string(row + r) + " (" + path + ")");
      std::int32_t width;
      std::memcpy(&width, h, 4);
      if (width < 0 || static_cast<std::size_t>(width) != cols)
        throw SiftLoadError(std::string(kind) + " row " + std::to_string(row + r) +
                            " has width " + std::to_string(width) + ", expected " +
                            std::to_string(cols) + " (" + path + ")");
      if (left < rec)
        throw SiftLoadError(std::string(kind) + " file ended inside the payload of row " +
                            std::to_string(row + r) + " (" + path + ")");
    }
    sink(buf.data(), row, nr);
    row += nr;
  }
  if (avail > want)
    throw SiftLoadError(std::string(kind) + " file has " + std::to_string(avail - want) +
                        " bytes after the expected " + std::to_string(rows) + " rows (" + path +
                        ")");
}

}  // namespace

FloatVectorDataset load_fvecs(const std::string& path, std::size_t expected_rows,
                              std::size_t expected_cols) {
  FloatVectorDataset ds;
  ds.rows = expected_rows;
  ds.cols = expected_cols;
  ds.values.resize(mul_checked(expected_rows, expected_cols, "fvecs"));
  const std::size_t rec = expected_cols * 4 + 4;
  walk_vecs(path, "fvecs", expected_rows, expected_cols,
            [&](const char* block, std::size_t row0, std::size_t n) {
              for (std::size_t r = 0; r < n; ++r)
                std::memcpy(ds.values.data() + (row0 + r) * expected_cols, block + r * rec + 4,
                            expected_cols * 4);
            });
  return ds;
}

void validate_fvecs_shape(const std::string& path, std::size_t expected_rows,
                          std::size_t expected_cols) {
  walk_vecs(path, "fvecs", expected_rows, expected_cols,
            [](const char*, std::size_t, std::size_t) {});
}

GroundTruthDataset load_ivecs(const std::string& path, std::size_t expected_rows,
                              std::size_t expected_cols) {
  GroundTruthDataset ds;
  ds.query_count = expected_rows;
  ds.neighbor_count = expected_cols;
  ds.neighbors.resize(mul_checked(expected_rows, expected_cols, "ivecs"));
  const std::size_t rec = expected_cols * 4 + 4;
  walk_vecs(path, "ivecs", expected_rows, expected_cols,
            [&](const char* block, std::size_t row0, std::size_t n) {
              for (std::size_t r = 0; r < n; ++r) {
                const char* src = block + r * rec + 4;
                std::uint32_t* dst = ds.neighbors.data() + (row0 + r) * expected_cols;
                for (std::size_t c = 0; c < expected_cols; ++c) {
                  std::int32_t v;
                  std::memcpy(&v, src + c * 4, 4);
                  if (v < 0)
                    throw SiftLoadError("ivecs row " + std::to_string(row0 + r) +
                                        " holds the negative neighbour id " +
                                        std::to_string(v) + " (" + path + ")");
                  dst[c] = static_cast<std::uint32_t>(v);
                }
              }
            });
  return ds;
}

SiftDataset load_sift_dataset(const std::string& base_path, const std::string& query_path,
                              const std::string& groundtruth_path,
                              std::size_t expected_base_rows, std::size_t expected_query_rows,
                              std::size_t expected_cols,
                              std::size_t expected_groundtruth_cols) {
  SiftDataset ds;
  ds.base = load_fvecs(base_path, expected_base_rows, expected_cols);
  ds.queries = load_fvecs(query_path, expected_query_rows, expected_cols);
  ds.groundtruth = load_ivecs(groundtruth_path, expected_query_rows, expected_groundtruth_cols);
  if (ds.base.cols != ds.queries.cols)
    throw SiftLoadError("base and query vectors have different dimensions");
  if (ds.groundtruth.query_count != ds.queries.rows)
    throw SiftLoadError("ground truth has a different number of rows than the queries");
  for (std::size_t i = 0; i < ds.groundtruth.neighbors.size(); ++i) {
    if (ds.groundtruth.neighbors[i] >= ds.base.rows)
      throw SiftLoadError("ground-truth neighbour " + std::to_string(ds.groundtruth.neighbors[i]) +
                          " of query " + std::to_string(i / ds.groundtruth.neighbor_count) +
                          " is outside base rows (" + std::to_string(ds.base.rows) + ")");
  }
  return ds;
}

FloatVectorDataset load_sift1m_base(const std::string& path) {
  return load_fvecs(path, kSift1MBaseVectorCount, kSift1MVectorDimension);
}

void validate_sift1m_base_shape(const std::string& path) {
  validate_fvecs_shape(path, kSift1MBaseVectorCount, kSift1MVectorDimension);
}

FloatVectorDataset load_sift1m_queries(const std::string& path) {
  return load_fvecs(path, kSift1MQueryVectorCount, kSift1MVectorDimension);
}

GroundTruthDataset load_sift1m_groundtruth(const std::string& path) {
  return load_ivecs(path, kSift1MQueryVectorCount, kSift1MGroundTruthNeighborCount);
}

SiftDataset load_sift1m_dataset(const std::string& base_path, const std::string& query_path,
                                const std::string& groundtruth_path) {
  return load_sift_dataset(base_path, query_path, groundtruth_path, kSift1MBaseVectorCount,
                           kSift1MQueryVectorCount, kSift1MVectorDimension,
                           kSift1MGroundTruthNeighborCount);
}

namespace {

// Reads the .bin header and checks that the payload of rows x cols values
// of 4 bytes is exactly what follows it.
void open_bin(File& f, const std::string& path, std::size_t& rows, std::size_t& cols) {
  if (f.size() < 8) throw SiftLoadError("bin file shorter than its 8-byte header: " + path);
  std::int32_t hdr[2];
  f.read_exact(hdr, 8);
  if (hdr[0] < 0 || hdr[1] < 0)
    throw SiftLoadError("bin file has a negative shape (" + std::to_string(hdr[0]) + " x " +
                        std::to_string(hdr[1]) + "): " + path);
  rows = static_cast<std::size_t>(hdr[0]);
  cols = static_cast<std::size_t>(hdr[1]);
  const std::size_t want = mul_checked(mul_checked(rows, cols, "bin"), 4, "bin") + 8;
  if (f.size() < want)
    throw SiftLoadError("bin file is truncated: " + std::to_string(f.size()) + " bytes, " +
                        std::to_string(want) + " expected: " + path);
  if (f.size() > want)
    throw SiftLoadError("bin file has " + std::to_string(f.size() - want) +
                        " bytes after its payload: " + path);
}

}  // namespace

FloatVectorDataset load_bin_f32(const std::string& path) {
  File f(path, "bin");
  FloatVectorDataset ds;
  open_bin(f, path, ds.rows, ds.cols);
  ds.values.resize(ds.rows * ds.cols);
  f.read_exact(ds.values.data(), ds.values.size() * 4);
  return ds;
}

GroundTruthDataset load_bin_i32(const std::string& path) {
  File f(path, "bin");
  GroundTruthDataset ds;
  open_bin(f, path, ds.query_count, ds.neighbor_count);
  ds.neighbors.resize(ds.query_count * ds.neighbor_count);
  f.read_exact(ds.neighbors.data(), ds.neighbors.size() * 4);
  for (std::size_t i = 0; i < ds.neighbors.size(); ++i) {
    if (static_cast<std::int32_t>(ds.neighbors[i]) < 0)
      throw SiftLoadError("bin ground truth holds the negative id " +
                          std::to_string(static_cast<std::int32_t>(ds.neighbors[i])) + ": " + path);
  }
  return ds;
}

}  // namespace cuvs_silicon
