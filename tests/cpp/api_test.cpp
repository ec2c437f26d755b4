// api_test.cpp -- the cuVS-compatible C++ API on the B200 engine.
//
// Re-creates the call patterns the reference's own tests use on its exact
// path and asserts the values those tests assert:
//   * a FAISS-facing adapter that rebuilds the index on every add and maps
//     UINT32_MAX to -1 (tests/faiss_v1_8_cagra_runtime_smoke.cpp:129-224,
//     values :299-396), written here without FAISS;
//   * the dispatch spy (tests/test_metal_search.cpp:16-58);
//   * attach_dataset_on_build = false (faiss smoke :247-261);
// plus save/load round trips, brute_force, and the validation errors of
// src/cagra.cpp:26-32,100-111.  Exit code 0 = all passed.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
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

int main(int argc, char** argv) {
  const std::string tmpdir = argc > 1 ? argv[1] : "/tmp";
  test_faiss_adapter_values();
  test_dispatch_spy();
  test_lifecycle_and_validation();
  test_save_load_and_brute_force(tmpdir);
  if (g_failures) {
    std::fprintf(stderr, "%d expectation(s) failed\n", g_failures);
    return 1;
  }
  std::printf("api_test: all expectations passed\n");
  return 0;
}
