// api_test.cpp -- the cuVS-compatible C++ API on the B200 engine.
//
// Re-creates the call patterns the reference's own tests use on its exact
// path and asserts the values those tests assert:
//   * a FAISS-facing adapter that rebuilds the index on every add and maps
//     UINT32_MAX to -1 (tests/faiss_v1_8_cagra_runtime_smoke.cpp:129-224,
//     values :299-396), written here without FAISS;
//   * the dispatch spy (tests/test_metal_search.cpp:16-58);
//   * attach_dataset_on_build = false (faiss smoke :247-261);
// plus save/load round trips, brute_force (its device cache views, the fp16
// + norms container payload, an index sharded over the devices of a
// raft::resources), and the validation errors of src/cagra.cpp:26-32,100-111.
// Exit code 0 = all passed.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <functional>
#include <limits>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuvs/neighbors/brute_force.hpp>
#include <cuvs/neighbors/cagra.hpp>
#include <raft/core/device_mdspan.hpp>
#include <raft/core/resources.hpp>

namespace cg = cuvs::neighbors::cagra;
namespace bf = cuvs::neighbors::brute_force;

static int g_failures = 0;
#define EXPECT(cond)                                                          \
  do {                                                                        \
    if (!(cond)) {                                                            \
      std::fprintf(stderr, "%s:%d: expectation failed: %s\n", __FILE__, __LINE__, #cond); \
      ++g_failures;                                                           \
    }                                                                         \
  } while (0)

template <typename E>
static bool throws(const std::function<void()>& f, const char* needle = nullptr) {
  try {
    f();
  } catch (const E& e) {
    return needle == nullptr || std::string(e.what()).find(needle) != std::string::npos;
  } catch (...) {
    return false;
  }
  return false;
}

// The adapter pattern of the reference's FAISS smoke test, without FAISS.
class FaissLikeIndex {
 public:
  explicit FaissLikeIndex(std::int64_t dim) : dim_(dim) {}
  void add(std::int64_t n, const float* x) {
    rows_.insert(rows_.end(), x, x + n * dim_);
    ntotal_ += n;
    cg::index_params ip;
    ip.metric = cuvs::distance::DistanceType::L2Expanded;
    index_ = cg::build(res_, ip,
                       raft::make_device_matrix_view<const float, std::int64_t>(rows_.data(),
                                                                                ntotal_, dim_));
  }
  void search(std::int64_t nq, const float* q, std::int64_t k, float* dist,
              std::int64_t* labels) const {
    if (!(k > 0)) throw std::invalid_argument("Error: 'k > 0' failed");
    cg::search_params sp;
    sp.itopk_size = static_cast<std::uint64_t>(k);
    std::vector<std::uint32_t> lab(static_cast<std::size_t>(nq * k));
    cg::search(res_, sp, index_,
               raft::make_device_matrix_view<const float, std::int64_t>(q, nq, dim_),
               raft::make_device_matrix_view<std::uint32_t, std::int64_t>(lab.data(), nq, k),
               raft::make_device_matrix_view<float, std::int64_t>(dist, nq, k));
    for (std::int64_t i = 0; i < nq * k; ++i)
      labels[i] = lab[i] == std::numeric_limits<std::uint32_t>::max()
                      ? -1
                      : static_cast<std::int64_t>(lab[i]);
  }
  std::int64_t ntotal() const { return ntotal_; }
  const cg::index<float, std::uint32_t>& index() const { return index_; }

 private:
  std::int64_t dim_, ntotal_ = 0;
  raft::resources res_;
  std::vector<float> rows_;
  cg::index<float, std::uint32_t> index_;
};

static void test_faiss_adapter_values() {
  const std::vector<float> db{0, 0, 10, 0, 0, 10, 2, 2};
  const std::vector<float> q{0, 0, 9, 1};
  FaissLikeIndex idx(2);
  idx.add(2, db.data());
  idx.add(2, db.data() + 4);
  EXPECT(idx.ntotal() == 4 && idx.index().rows() == 4);

  std::vector<float> d(4);
  std::vector<std::int64_t> l(4);
  idx.search(2, q.data(), 2, d.data(), l.data());
  EXPECT(l[0] == 0 && d[0] == 0.0F);
  EXPECT(l[1] == 3 && d[1] == 8.0F);
  EXPECT(l[2] == 1 && d[2] == 2.0F);
  EXPECT(l[3] == 3 && d[3] == 50.0F);

  std::vector<float> od(4, -7.0F);
  std::vector<std::int64_t> ol(4, -7);
  idx.search(1, q.data(), 4, od.data(), ol.data());
  EXPECT(ol[0] == 0 && od[0] == 0.0F);
  EXPECT(ol[1] == 3 && od[1] == 8.0F);
  EXPECT(ol[2] == 1 && od[2] == 100.0F);  // tie at 100: lower label first
  EXPECT(ol[3] == 2 && od[3] == 100.0F);

  std::vector<float> sd(5, -7.0F);
  std::vector<std::int64_t> sl(5, -7);
  idx.search(1, q.data(), 5, sd.data(), sl.data());
  EXPECT(sl[0] == 0 && sd[0] == 0.0F);
  EXPECT(sl[4] == -1 && std::isinf(sd[4]));

  std::vector<float> bd(10, -7.0F);
  std::vector<std::int64_t> bl(10, -7);
  idx.search(2, q.data(), 5, bd.data(), bl.data());
  EXPECT(bl[0] == 0 && bd[0] == 0.0F);
  EXPECT(bl[4] == -1 && std::isinf(bd[4]));
  EXPECT(bl[9] == -1 && std::isinf(bd[9]));

  std::vector<float> zd(2);
  std::vector<std::int64_t> zl(2);
  EXPECT(throws<std::invalid_argument>([&] { idx.search(2, q.data(), 0, zd.data(), zl.data()); },
                                       "k > 0"));
}

static void test_dispatch_spy() {
  constexpr int N = 64, Q = 4, D = 8, K = 4;
  std::vector<float> base(N * D, 0.0F), queries(Q * D, 0.0F);
  for (int i = 0; i < N; ++i) base[i * D + (i % D)] = static_cast<float>(i);
  for (int j = 0; j < Q; ++j) queries[j * D + (j % D)] = 1.0F;
  std::vector<std::uint32_t> nb(Q * K);
  std::vector<float> ds(Q * K);
  raft::resources res;
  cg::index_params ip;
  cg::search_params sp;
  auto idx = cg::build(res, ip,
                       raft::device_matrix_view<const float, std::int64_t>(base.data(), N, D));
  cg::reset_metal_dispatch_count();
  cg::search(res, sp, idx,
             raft::device_matrix_view<const float, std::int64_t>(queries.data(), Q, D),
             raft::device_matrix_view<std::uint32_t, std::int64_t>(nb.data(), Q, K),
             raft::device_matrix_view<float, std::int64_t>(ds.data(), Q, K));
  EXPECT(cg::metal_dispatch_count() > 0);
  // query 0 = e0: row 0 (the zero vector) is at distance 1
  EXPECT(nb[0] == 0 && ds[0] == 1.0F);
  cg::increment_metal_dispatch_count();
  const auto c = cg::metal_dispatch_count();
  cg::reset_metal_dispatch_count();
  EXPECT(c > 0 && cg::metal_dispatch_count() == 0);
}

static void test_lifecycle_and_validation() {
  const std::vector<float> db{0, 0, 10, 0, 0, 10, 2, 2};
  raft::resources res;
  cg::index_params ip;
  ip.attach_dataset_on_build = false;
  auto idx = cg::build(res, ip, raft::make_device_matrix_view<const float, std::int64_t>(
                                    db.data(), 4, 2));
  EXPECT(idx.rows() == 4 && idx.cols() == 2 && idx.dataset().empty());
  std::vector<float> q{0, 0};
  std::vector<std::uint32_t> nb(1);
  std::vector<float> ds(1);
  cg::search_params sp;
  auto qv = raft::make_device_matrix_view<const float, std::int64_t>(q.data(), 1, 2);
  auto nv = raft::make_device_matrix_view<std::uint32_t, std::int64_t>(nb.data(), 1, 1);
  auto dv = raft::make_device_matrix_view<float, std::int64_t>(ds.data(), 1, 1);
  EXPECT(throws<std::invalid_argument>([&] { cg::search(res, sp, idx, qv, nv, dv); }));

  cg::index_params ipl2;
  ipl2.metric = cuvs::distance::DistanceType::InnerProduct;
  EXPECT(throws<std::invalid_argument>([&] {
    cg::build(res, ipl2, raft::make_device_matrix_view<const float, std::int64_t>(db.data(), 4, 2));
  }, "L2Expanded"));
  EXPECT(throws<std::invalid_argument>([&] {
    cg::build(res, cg::index_params{},
              raft::make_device_matrix_view<const float, std::int64_t>(nullptr, 4, 2));
  }, "non-empty"));

  auto full = cg::build(res, cg::index_params{},
                        raft::make_device_matrix_view<const float, std::int64_t>(db.data(), 4, 2));
  std::vector<float> q3{0, 0, 0};
  EXPECT(throws<std::invalid_argument>([&] {
    cg::search(res, sp, full,
               raft::make_device_matrix_view<const float, std::int64_t>(q3.data(), 1, 3), nv, dv);
  }, "dimension"));
  std::vector<std::uint32_t> nb2(2);
  EXPECT(throws<std::invalid_argument>([&] {
    cg::search(res, sp, full, qv,
               raft::make_device_matrix_view<std::uint32_t, std::int64_t>(nb2.data(), 1, 2), dv);
  }, "shape"));
  EXPECT(throws<std::invalid_argument>([&] {
    cg::search(res, sp, full, qv,
               raft::make_device_matrix_view<std::uint32_t, std::int64_t>(nullptr, 1, 1), dv);
  }, "valid buffers"));
}

static std::vector<float> random_rows(std::int64_t n, std::int64_t d, unsigned seed) {
  std::vector<float> v(static_cast<std::size_t>(n * d));
  std::uint64_t s = seed * 6364136223846793005ULL + 1442695040888963407ULL;
  for (auto& x : v) {
    s = s * 6364136223846793005ULL + 1442695040888963407ULL;
    x = static_cast<float>(static_cast<std::int64_t>(s >> 40) % 2001 - 1000) / 1000.0F;
  }
  return v;
}

static void test_save_load_and_brute_force(const std::string& tmpdir) {
  const std::int64_t n = 5000, d = 96, q = 7, k = 12;
  const auto base = random_rows(n, d, 1);
  const auto qs = random_rows(q, d, 2);
  raft::resources res;
  auto ci = cg::build(res, cg::index_params{},
                      raft::make_device_matrix_view<const float, std::int64_t>(base.data(), n, d));
  std::vector<std::uint32_t> n1(q * k), n2(q * k);
  std::vector<float> d1(q * k), d2(q * k);
  cg::search(res, cg::search_params{}, ci,
             raft::make_device_matrix_view<const float, std::int64_t>(qs.data(), q, d),
             raft::make_device_matrix_view<std::uint32_t, std::int64_t>(n1.data(), q, k),
             raft::make_device_matrix_view<float, std::int64_t>(d1.data(), q, k));
  const std::string path = tmpdir + "/cagra_index.bin";
  cg::save_index(ci, path);
  auto loaded = cg::load_index(path);
  EXPECT(loaded.rows() == n && loaded.cols() == d && loaded.graph_degree() == 0);
  cg::search(res, cg::search_params{}, loaded,
             raft::make_device_matrix_view<const float, std::int64_t>(qs.data(), q, d),
             raft::make_device_matrix_view<std::uint32_t, std::int64_t>(n2.data(), q, k),
             raft::make_device_matrix_view<float, std::int64_t>(d2.data(), q, k));
  EXPECT(n1 == n2 && d1 == d2);

  // brute_force: int64 and uint32 neighbours agree with cagra
  auto bi = bf::build(res, raft::make_device_matrix_view<const float, std::int64_t>(base.data(), n, d));
  EXPECT(bi.size() == n && bi.dim() == d);
  std::vector<std::int64_t> l64(q * k);
  std::vector<float> d3(q * k);
  bf::search(res, bi, raft::make_device_matrix_view<const float, std::int64_t>(qs.data(), q, d),
             raft::make_device_matrix_view<std::int64_t, std::int64_t>(l64.data(), q, k),
             raft::make_device_matrix_view<float, std::int64_t>(d3.data(), q, k));
  for (std::int64_t i = 0; i < q * k; ++i) EXPECT(l64[i] == static_cast<std::int64_t>(n1[i]));
  EXPECT(d3 == d1);

  const std::string bpath = tmpdir + "/bf_index.bin";
  bf::serialize(res, bpath, bi);
  auto bl = bf::deserialize(res, bpath);
  std::vector<std::uint32_t> n4(q * k);
  std::vector<float> d4(q * k);
  bf::search(res, bl, raft::make_device_matrix_view<const float, std::int64_t>(qs.data(), q, d),
             raft::make_device_matrix_view<std::uint32_t, std::int64_t>(n4.data(), q, k),
             raft::make_device_matrix_view<float, std::int64_t>(d4.data(), q, k));
  EXPECT(n4 == n1 && d4 == d1);
  // a brute_force file is a valid reference container: cagra::load_index reads it
  auto as_cagra = cg::load_index(bpath);
  EXPECT(as_cagra.rows() == n && as_cagra.dataset().size() == static_cast<std::size_t>(n * d));

  // InnerProduct (rejected by cagra::build, src/cagra.cpp:26-28; accepted by
  // brute_force): integer vectors, so the scores are exact.  Database rows
  // (1,0) (0,1) (2,2) (-1,3), query (3,1): scores 3, 1, 8, 0 -> rows
  // 2, 0, 1, 3, then padding (-1, -inf).
  const std::vector<float> ipdb = {1, 0, 0, 1, 2, 2, -1, 3};
  const std::vector<float> ipq = {3, 1};
  auto ipi = bf::build(res, raft::make_device_matrix_view<const float, std::int64_t>(ipdb.data(), 4, 2),
                       cuvs::distance::DistanceType::InnerProduct);
  EXPECT(ipi.metric() == cuvs::distance::DistanceType::InnerProduct);
  std::vector<std::int64_t> ipl(5);
  std::vector<float> ips(5);
  bf::search(res, ipi, raft::make_device_matrix_view<const float, std::int64_t>(ipq.data(), 1, 2),
             raft::make_device_matrix_view<std::int64_t, std::int64_t>(ipl.data(), 1, 5),
             raft::make_device_matrix_view<float, std::int64_t>(ips.data(), 1, 5));
  EXPECT((ipl == std::vector<std::int64_t>{2, 0, 1, 3, -1}));
  EXPECT(ips[0] == 8.0f && ips[1] == 3.0f && ips[2] == 1.0f && ips[3] == 0.0f &&
         std::isinf(ips[4]) && ips[4] < 0);
  // the metric survives serialisation (flag bit 2 of the container)
  const std::string ippath = tmpdir + "/bf_ip_index.bin";
  bf::serialize(res, ippath, ipi);
  auto ipl2 = bf::deserialize(res, ippath);
  EXPECT(ipl2.metric() == cuvs::distance::DistanceType::InnerProduct);
  std::vector<std::int64_t> ipl3(5);
  std::vector<float> ips3(5);
  bf::search(res, ipl2, raft::make_device_matrix_view<const float, std::int64_t>(ipq.data(), 1, 2),
             raft::make_device_matrix_view<std::int64_t, std::int64_t>(ipl3.data(), 1, 5),
             raft::make_device_matrix_view<float, std::int64_t>(ips3.data(), 1, 5));
  EXPECT(ipl3 == ipl && ips3 == ips);
  cg::index_params ipp;
  ipp.metric = cuvs::distance::DistanceType::InnerProduct;
  EXPECT(throws<std::invalid_argument>([&] {
    cg::build(res, ipp, raft::make_device_matrix_view<const float, std::int64_t>(base.data(), n, d));
  }));
}

// IEEE binary16 bits -> float (exact), for checking the device cache.
static float half_bits_to_float(std::uint16_t h) {
  const int e = (h >> 10) & 31, m = h & 1023;
  const float sign = (h & 0x8000) ? -1.0f : 1.0f;
  if (e == 0) return sign * std::ldexp(static_cast<float>(m), -24);
  if (e == 31) return m ? std::numeric_limits<float>::quiet_NaN()
                        : sign * std::numeric_limits<float>::infinity();
  return sign * std::ldexp(static_cast<float>(m + 1024), e - 25);
}

// The index's device cache (the reference's fp16 dataset + d_norms,
// src/metal_context.mm:38-54,155-175) through dataset()/norms(), and the
// fp16 + norms container payload that reloads without conversion.
static void test_device_cache_and_fp16_payload(const std::string& tmpdir) {
  const std::int64_t n = 3001, d = 70, q = 5, k = 9;
  const auto base = random_rows(n, d, 3);
  const auto qs = random_rows(q, d, 4);
  raft::resources res;
  auto bi = bf::build(res, raft::make_device_matrix_view<const float, std::int64_t>(base.data(), n, d));
  const auto rows = bi.dataset();
  const auto norms = bi.norms();
  EXPECT(rows.rows == n && rows.dim == d && rows.ld >= d && rows.ld % 8 == 0);
  EXPECT(norms.size() == n);
  std::vector<std::uint16_t> h16(static_cast<std::size_t>(n * rows.ld));
  std::vector<float> hn(static_cast<std::size_t>(n));
  EXPECT(cudaMemcpy(h16.data(), rows.data, h16.size() * 2, cudaMemcpyDeviceToHost) == cudaSuccess);
  EXPECT(cudaMemcpy(hn.data(), norms.data_handle(), hn.size() * 4, cudaMemcpyDeviceToHost) ==
         cudaSuccess);
  int bad_rows = 0, bad_norms = 0;
  for (std::int64_t r = 0; r < n; ++r) {
    double acc = 0.0;
    for (std::int64_t c = 0; c < rows.ld; ++c) {
      const float v = half_bits_to_float(h16[static_cast<std::size_t>(r * rows.ld + c)]);
      if (c < d) {
        // round-to-nearest-even fp16 of the input: within half an fp16 ulp
        const float x = base[static_cast<std::size_t>(r * d + c)];
        if (std::fabs(v - x) > std::ldexp(std::fabs(x), -11) + 1e-7f) ++bad_rows;
        acc += static_cast<double>(v) * v;
      } else if (v != 0.0f) {
        ++bad_rows;  // padding columns are zero
      }
    }
    if (std::fabs(hn[static_cast<std::size_t>(r)] - acc) > 1e-5 * (acc + 1e-6)) ++bad_norms;
  }
  EXPECT(bad_rows == 0 && bad_norms == 0);

  std::vector<std::int64_t> l1(q * k), l2(q * k);
  std::vector<float> d1(q * k), d2(q * k);
  bf::search(res, bi, raft::make_device_matrix_view<const float, std::int64_t>(qs.data(), q, d),
             raft::make_device_matrix_view<std::int64_t, std::int64_t>(l1.data(), q, k),
             raft::make_device_matrix_view<float, std::int64_t>(d1.data(), q, k));
  const std::string path = tmpdir + "/bf_fp16.bin";
  bf::serialize(res, path, bi, bf::payload::fp16_with_norms);
  {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    EXPECT(static_cast<std::int64_t>(f.tellg()) == 32 + n * d * 2 + n * 4);
  }
  auto bl = bf::deserialize(res, path);
  EXPECT(bl.size() == n && bl.dim() == d);
  bf::search(res, bl, raft::make_device_matrix_view<const float, std::int64_t>(qs.data(), q, d),
             raft::make_device_matrix_view<std::int64_t, std::int64_t>(l2.data(), q, k),
             raft::make_device_matrix_view<float, std::int64_t>(d2.data(), q, k));
  EXPECT(l1 == l2 && d1 == d2);
  // the reloaded cache holds the same norms, bit for bit
  std::vector<float> hn2(static_cast<std::size_t>(n));
  EXPECT(cudaMemcpy(hn2.data(), bl.norms().data_handle(), hn2.size() * 4,
                    cudaMemcpyDeviceToHost) == cudaSuccess);
  EXPECT(hn2 == hn);
  // the reference's loader sees no fp32 dataset block in an fp16 file
  auto as_cagra = cg::load_index(path);
  EXPECT(as_cagra.rows() == n && as_cagra.dataset().empty());
}

// A raft::resources with several devices shards the index across them; the
// merged result equals the single-device index's byte for byte.  With one
// GPU the device list {0, 0} still runs two shards, streams, the gather and
// the device merge.
static void test_multi_device_index(const std::string& tmpdir) {
  int count = 0;
  cudaGetDeviceCount(&count);
  const std::vector<int> devs = count >= 2 ? std::vector<int>{0, 1} : std::vector<int>{0, 0};
  const std::int64_t n = 20011, d = 72, q = 37, k = 10;
  const auto base = random_rows(n, d, 5);
  const auto qs = random_rows(q, d, 6);
  raft::resources one;
  raft::resources multi(devs);
  EXPECT(multi.devices().size() == 2 && multi.device() == 0);
  for (auto metric : {cuvs::distance::DistanceType::L2Expanded,
                      cuvs::distance::DistanceType::InnerProduct}) {
    auto single = bf::build(one, raft::make_device_matrix_view<const float, std::int64_t>(base.data(), n, d), metric);
    auto sharded = bf::build(multi, raft::make_device_matrix_view<const float, std::int64_t>(base.data(), n, d), metric);
    EXPECT(sharded.n_shards() == 2 && sharded.size() == n);
    EXPECT(sharded.shard_row_offset(1) == sharded.shard_rows(0));
    EXPECT(sharded.shard_device(1) == devs[1]);
    for (std::int64_t kk : {std::int64_t(1), k, std::int64_t(100)}) {
      std::vector<std::int64_t> l1(q * kk), l2(q * kk);
      std::vector<std::uint32_t> u2(q * kk);
      std::vector<float> d1(q * kk), d2(q * kk), e2(q * kk);
      auto qv = raft::make_device_matrix_view<const float, std::int64_t>(qs.data(), q, d);
      bf::search(one, single, qv, raft::make_device_matrix_view<std::int64_t, std::int64_t>(l1.data(), q, kk),
                 raft::make_device_matrix_view<float, std::int64_t>(d1.data(), q, kk));
      bf::search(multi, sharded, qv, raft::make_device_matrix_view<std::int64_t, std::int64_t>(l2.data(), q, kk),
                 raft::make_device_matrix_view<float, std::int64_t>(d2.data(), q, kk));
      bf::search(multi, sharded, qv, raft::make_device_matrix_view<std::uint32_t, std::int64_t>(u2.data(), q, kk),
                 raft::make_device_matrix_view<float, std::int64_t>(e2.data(), q, kk));
      EXPECT(l1 == l2 && d1 == d2 && d1 == e2);
      for (std::int64_t i = 0; i < q * kk; ++i) EXPECT(static_cast<std::int64_t>(u2[i]) == l1[i]);
    }
  }
  // device-resident queries and outputs, and a sharded fp16 round trip
  auto sharded = bf::build(multi, raft::make_device_matrix_view<const float, std::int64_t>(base.data(), n, d));
  float* dq = nullptr;
  std::int64_t* dl = nullptr;
  float* dd = nullptr;
  cudaSetDevice(0);
  EXPECT(cudaMalloc(&dq, q * d * 4) == cudaSuccess && cudaMalloc(&dl, q * k * 8) == cudaSuccess &&
         cudaMalloc(&dd, q * k * 4) == cudaSuccess);
  cudaMemcpy(dq, qs.data(), q * d * 4, cudaMemcpyHostToDevice);
  bf::search(multi, sharded, raft::make_device_matrix_view<const float, std::int64_t>(dq, q, d),
             raft::make_device_matrix_view<std::int64_t, std::int64_t>(dl, q, k),
             raft::make_device_matrix_view<float, std::int64_t>(dd, q, k));
  std::vector<std::int64_t> l3(q * k), l4(q * k);
  std::vector<float> d3(q * k), d4(q * k);
  cudaMemcpy(l3.data(), dl, q * k * 8, cudaMemcpyDeviceToHost);
  cudaMemcpy(d3.data(), dd, q * k * 4, cudaMemcpyDeviceToHost);
  cudaFree(dq);
  cudaFree(dl);
  cudaFree(dd);
  const std::string path = tmpdir + "/bf_sharded.bin";
  bf::serialize(multi, path, sharded, bf::payload::fp16_with_norms);
  auto back = bf::deserialize(multi, path);
  EXPECT(back.n_shards() == 2);
  bf::search(multi, back, raft::make_device_matrix_view<const float, std::int64_t>(qs.data(), q, d),
             raft::make_device_matrix_view<std::int64_t, std::int64_t>(l4.data(), q, k),
             raft::make_device_matrix_view<float, std::int64_t>(d4.data(), q, k));
  EXPECT(l3 == l4 && d3 == d4);
}

int main(int argc, char** argv) {
  const std::string tmpdir = argc > 1 ? argv[1] : "/tmp";
  test_faiss_adapter_values();
  test_dispatch_spy();
  test_lifecycle_and_validation();
  test_save_load_and_brute_force(tmpdir);
  test_device_cache_and_fp16_payload(tmpdir);
  test_multi_device_index(tmpdir);
  if (g_failures) {
    std::fprintf(stderr, "%d expectation(s) failed\n", g_failures);
    return 1;
  }
  std::printf("api_test: all expectations passed\n");
  return 0;
}
