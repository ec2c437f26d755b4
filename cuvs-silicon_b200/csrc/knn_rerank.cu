// knn_rerank.cu -- exact fp32 re-ranking of the fp16 scan's candidates.
//
// The reference's API takes fp32 rows and queries, and its portable exact
// search computes every distance in fp32 from the unrounded vectors:
// dist = sum over d, in order, of (q[d] - x[d])^2 (src/cagra.cpp:218-226),
// ordered by (distance, index) (src/cagra.cpp:229-238).  The scan kernel
// works on fp16-rounded rows, so its order can differ from that one where
// distances are closer than the rounding.  This kernel takes the scan's top
// kc candidates per query (kc > k), recomputes each candidate's distance
// from the fp32 rows with exactly the reference's arithmetic (sequential
// over d, fp32, every operation rounded on its own: __fsub_rn / __fmul_rn /
// __fadd_rn, so no fused multiply-add), and keeps the k best by
// (distance, index).  The distances it reports are bit-identical to the
// reference's for the same rows.
//
// Certificate.  The result is the exact fp32 top-k whenever no row outside
// the candidates can beat the k-th re-ranked distance r_k.  A row y outside
// the candidates has scan distance d16(y) >= t, the kc-th candidate's scan
// distance.  With delta an upper bound of |d16(y) - d32(y)| over every row
// that could beat r_k, r_k + delta < t proves that no such row exists.
// delta follows a rounding model stated in full in bound_l2 / bound_ip
// (fp16 rounding of every coordinate, fp32 norms, tensor-core accumulation
// losing at most two units in the last place per addition, fp32 sequential
// sums of the reference).  A query that fails the test is counted in
// *uncertified; its result is still the best re-ranked candidates.
//
// Inner product: the same procedure on score = sum q[d] * x[d] (fp32,
// sequential), ordered by (-score, index); the reported value is the score.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "knn_internal.h"

namespace knn {

namespace {

constexpr int kRerankThreads = 256;  // >= the largest candidate count (kMaxK)
static_assert(kRerankThreads >= kMaxK, "one thread per candidate");

__device__ __forceinline__ bool less_pair(float da, uint32_t ia, float db, uint32_t ib) {
  return da < db || (da == db && ia < ib);
}

// Exact fp32 distance of the reference (or minus the exact fp32 inner
// product), every operation rounded separately and in index order.
template <int kMetric>
__device__ float exact_dist(const float* __restrict__ q, const float* __restrict__ x,
                            int64_t dim, bool vec4) {
  float acc = 0.0f;
  if (vec4) {
    const float4* q4 = reinterpret_cast<const float4*>(q);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int64_t j = 0; j < dim / 4; ++j) {
      const float4 a = __ldg(q4 + j);
      const float4 b = __ldg(x4 + j);
      if constexpr (kMetric == KNN_METRIC_INNER_PRODUCT) {
        acc = __fadd_rn(acc, __fmul_rn(a.x, b.x));
        acc = __fadd_rn(acc, __fmul_rn(a.y, b.y));
        acc = __fadd_rn(acc, __fmul_rn(a.z, b.z));
        acc = __fadd_rn(acc, __fmul_rn(a.w, b.w));
      } else {
        float t;
        t = __fsub_rn(a.x, b.x);
        acc = __fadd_rn(acc, __fmul_rn(t, t));
        t = __fsub_rn(a.y, b.y);
        acc = __fadd_rn(acc, __fmul_rn(t, t));
        t = __fsub_rn(a.z, b.z);
        acc = __fadd_rn(acc, __fmul_rn(t, t));
        t = __fsub_rn(a.w, b.w);
        acc = __fadd_rn(acc, __fmul_rn(t, t));
      }
    }
  } else {
    for (int64_t j = 0; j < dim; ++j) {
      const float a = __ldg(q + j), b = __ldg(x + j);
      if constexpr (kMetric == KNN_METRIC_INNER_PRODUCT) {
        acc = __fadd_rn(acc, __fmul_rn(a, b));
      } else {
        const float t = __fsub_rn(a, b);
        acc = __fadd_rn(acc, __fmul_rn(t, t));
      }
    }
  }
  if constexpr (kMetric == KNN_METRIC_INNER_PRODUCT) {
    return acc == 0.0f ? 0.0f : -acc;  // never -0 (order of equal keys)
  } else {
    return acc;
  }
}

// Cooperative path (dim % 4 == 0, 16-byte aligned rows and queries): the
// block copies the candidate rows into shared memory chunk by chunk with
// cp.async (kRerankStages chunks in flight, coalesced 16-byte copies; rows
// padded by one float4 so 8 consecutive lanes read distinct banks), and
// thread t sums candidate t's chunk from there.  Every thread still adds
// the dimensions of its row in index order, so the values equal
// exact_dist's.
constexpr int kRerankStages = 4;
constexpr int kRerankStageBytes = 40960;

// float4 per row per chunk for kc candidates (at most 64, at least 1).
inline int rerank_chunk_f4(int kc, int64_t dim) {
  int cw = kRerankStageBytes / (16 * kc) - 1;
  if (cw > 64) cw = 64;
  if (cw > dim / 4) cw = static_cast<int>(dim / 4);
  return cw < 1 ? 1 : cw;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t sa = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Called by every thread of the block; returns candidate t's distance for
// t < kc with a valid row (s_i[t] != kNoIndex), +inf otherwise.
template <int kMetric>
__device__ float staged_dist(const float* __restrict__ qv, const float* __restrict__ rows,
                             int64_t dim, const uint32_t* s_i, int kc, int cw, float4* buf) {
  const int t = threadIdx.x;
  const int64_t d4 = dim / 4;
  const int nch = static_cast<int>((d4 + cw - 1) / cw);
  const int rs = cw + 1;
  const int stage_f4 = kc * rs;
  auto issue = [&](int c) {
    if (c < nch) {
      float4* dst = buf + (c % kRerankStages) * stage_f4;
      const int64_t w0 = static_cast<int64_t>(c) * cw;
      const int wn = static_cast<int>(d4 - w0 < cw ? d4 - w0 : cw);
      for (int e = t; e < kc * wn; e += blockDim.x) {
        const int r = e / wn;
        const int w = e - r * wn;
        const uint32_t row = s_i[r];
        if (row != kNoIndex)
          cp_async16(dst + r * rs + w, rows + static_cast<int64_t>(row) * dim + (w0 + w) * 4);
      }
    }
    cp_async_commit();  // one group per call, empty or not: uniform counting
  };
  for (int c = 0; c < kRerankStages - 1; ++c) issue(c);
  const bool mine = t < kc && s_i[t] != kNoIndex;
  const float4* q4 = reinterpret_cast<const float4*>(qv);
  float acc = 0.0f;
  for (int c = 0; c < nch; ++c) {
    cp_async_wait<kRerankStages - 2>();  // this thread's copies of chunk c
    __syncthreads();                     // everyone's
    if (mine) {
      const float4* src = buf + (c % kRerankStages) * stage_f4 + t * rs;
      const int64_t w0 = static_cast<int64_t>(c) * cw;
      const int wn = static_cast<int>(d4 - w0 < cw ? d4 - w0 : cw);
      for (int w = 0; w < wn; ++w) {
        const float4 a = __ldg(q4 + w0 + w);
        const float4 b = src[w];
        if constexpr (kMetric == KNN_METRIC_INNER_PRODUCT) {
          acc = __fadd_rn(acc, __fmul_rn(a.x, b.x));
          acc = __fadd_rn(acc, __fmul_rn(a.y, b.y));
          acc = __fadd_rn(acc, __fmul_rn(a.z, b.z));
          acc = __fadd_rn(acc, __fmul_rn(a.w, b.w));
        } else {
          float u;
          u = __fsub_rn(a.x, b.x);
          acc = __fadd_rn(acc, __fmul_rn(u, u));
          u = __fsub_rn(a.y, b.y);
          acc = __fadd_rn(acc, __fmul_rn(u, u));
          u = __fsub_rn(a.z, b.z);
          acc = __fadd_rn(acc, __fmul_rn(u, u));
          u = __fsub_rn(a.w, b.w);
          acc = __fadd_rn(acc, __fmul_rn(u, u));
        }
      }
    }
    __syncthreads();                     // chunk c's stage may be refilled
    issue(c + kRerankStages - 1);
  }
  cp_async_wait<0>();
  if (!mine) return __int_as_float(0x7f800000);
  if constexpr (kMetric == KNN_METRIC_INNER_PRODUCT) {
    return acc == 0.0f ? 0.0f : -acc;
  } else {
    return acc;
  }
}

// Bound of |d16(y) - d32(y)| for squared L2 over rows y with d32(y) <= r.
// qn = |q| of the fp32 query, xn >= |x| of every fp32 row, D = dim,
// u = 2^-24 (fp32 unit roundoff):
//   e  = |(q16 - q) - (x16 - x)| <= 2^-11 (qn + xn) + 2 sqrt(D) 2^-25
//        (fp16 round-to-nearest: relative 2^-11 per coordinate, absolute
//        2^-25 in the subnormal range);
//   |d(q16, x16) - d(q, x)| <= 2 sqrt(d) e + e^2 (d = exact squared L2);
//   scan arithmetic: norms (fp32 sums of D terms) D u (qn^2 + xn^2), the
//        tensor-core dot product 4 D u qn xn (each addition loses at most
//        two units in the last place), the final fma and add 2u (qn + xn)^2;
//   the reference's own sum: |d32 - d| <= (D + 3) u d, so d <= r / (1 - g).
// A 1.25 factor covers the rounding of this bound itself.
__host__ __device__ double bound_l2(double r, double qn, double xn, int64_t dim) {
  const double u = 5.9604644775390625e-08;  // 2^-24
  const double D = static_cast<double>(dim);
  const double g = (D + 3.0) * u;
  const double d = fmax(r, 0.0) / (1.0 - g);
  const double e = 4.8828125e-04 * (qn + xn) + 2.0 * sqrt(D) * 2.98023223876953125e-08;
  const double scan = D * u * (qn * qn + xn * xn) + 4.0 * D * u * qn * xn +
                      2.0 * u * (qn + xn) * (qn + xn);
  return 1.25 * (g * d + 2.0 * sqrt(d) * e + e * e + scan);
}

// Same for the inner product (d = -score):
//   |q16.x16 - q.x| <= |q16 - q| |x16| + |q| |x16 - x| <= 2^-10 qn xn + subnormal terms;
//   tensor-core dot 4 D u qn xn; the reference's sum (D + 1) u qn xn.
__host__ __device__ double bound_ip(double qn, double xn, int64_t dim) {
  const double u = 5.9604644775390625e-08;
  const double D = static_cast<double>(dim);
  const double sub = sqrt(D) * 2.98023223876953125e-08;
  return 1.25 * ((9.765625e-04 + 4.0 * D * u + (D + 1.0) * u) * qn * xn +
                 sub * (qn + xn) * (1.0 + 4.8828125e-04) + sub * sub);
}

template <int kMetric, typename OutIdx>
__global__ void __launch_bounds__(kRerankThreads)
    rerank_kernel(const float* __restrict__ queries, const float* __restrict__ rows,
                  int64_t dim, const float* __restrict__ cand_d,
                  const uint32_t* __restrict__ cand_i, int kc, int k,
                  const float* __restrict__ max_norm2, int64_t index_offset,
                  float* __restrict__ out_d, OutIdx* __restrict__ out_i, float sign,
                  int* __restrict__ uncertified, int cw) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float s_d[kRerankThreads];
  __shared__ uint32_t s_i[kRerankThreads];
  __shared__ double s_red[kRerankThreads / 32];
  __shared__ int s_valid;
  __shared__ float s_rk;

  const int64_t q = blockIdx.x;
  const int t = threadIdx.x;
  const float* qv = queries + q * dim;
  const bool vec4 = (dim % 4) == 0 && (reinterpret_cast<uintptr_t>(queries) % 16) == 0 &&
                    (reinterpret_cast<uintptr_t>(rows) % 16) == 0;
  if (t == 0) s_valid = 0;
  __syncthreads();

  // |q|^2 of the fp32 query, in float64 (for the certificate only)
  double part = 0.0;
  for (int64_t j = t; j < dim; j += blockDim.x) {
    const double v = qv[j];
    part += v * v;
  }
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if ((t & 31) == 0) s_red[t >> 5] = part;

  uint32_t idx = kNoIndex;
  if (t < kc) idx = cand_i[q * kc + t];
  s_i[t] = idx;
  if (idx != kNoIndex) atomicAdd(&s_valid, 1);
  __syncthreads();
  float d = __int_as_float(0x7f800000);
  if (cw > 0) {  // uniform: the launcher picks the path
    extern __shared__ float4 rr_buf[];
    d = staged_dist<kMetric>(qv, rows, dim, s_i, kc, cw, rr_buf);
  } else if (idx != kNoIndex) {
    d = exact_dist<kMetric>(qv, rows + static_cast<int64_t>(idx) * dim, dim, vec4);
  }
  s_d[t] = d;
  __syncthreads();
  const int valid = s_valid;

  // rank counting over the candidates (distinct rows; padding after them)
  if (t < kc && idx != kNoIndex) {
    int rank = 0;
    for (int u = 0; u < kc; ++u) rank += less_pair(s_d[u], s_i[u], d, idx) ? 1 : 0;
    if (rank < k) {
      out_d[q * k + rank] = sign * d + 0.0f;
      if constexpr (sizeof(OutIdx) == 8) {
        out_i[q * k + rank] = static_cast<OutIdx>(idx) + index_offset;
      } else {
        out_i[q * k + rank] = static_cast<uint32_t>(idx + index_offset);
      }
    }
    if (rank == k - 1) s_rk = d;
  }
  for (int r = valid + t; r < k; r += blockDim.x) {
    out_d[q * k + r] = sign * __int_as_float(0x7f800000);
    if constexpr (sizeof(OutIdx) == 8) {
      out_i[q * k + r] = OutIdx(-1);
    } else {
      out_i[q * k + r] = kNoIndex;
    }
  }
  __syncthreads();

  if (t == 0) {
    // fewer than kc candidates: every row of the shard is a candidate
    bool certified = valid < kc;
    if (!certified && valid >= k) {
      double qn2 = 0.0;
      for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) qn2 += s_red[w];
      const double qn = sqrt(qn2);
      const double D = static_cast<double>(dim);
      // |x| <= (|x16| + sqrt(D) 2^-25) / (1 - 2^-11) for every row
      const double xn =
          (sqrt(static_cast<double>(*max_norm2)) + sqrt(D) * 2.98023223876953125e-08) /
          (1.0 - 4.8828125e-04);
      const double rk = s_rk;
      const double tk = cand_d[q * kc + kc - 1];
      const double delta = kMetric == KNN_METRIC_INNER_PRODUCT ? bound_ip(qn, xn, dim)
                                                               : bound_l2(rk, qn, xn, dim);
      certified = isfinite(delta) && isfinite(rk) && rk + delta < tk;
    }
    if (!certified) atomicAdd(uncertified, 1);
  }
}

template <int kMetric, typename OutIdx>
cudaError_t launch_t(const float* queries, const float* rows, int64_t dim,
                     const float* cand_d, const uint32_t* cand_i, int kc, int k,
                     int64_t n_queries, const float* max_norm2, int64_t index_offset,
                     float* out_d, OutIdx* out_i, float sign, int* uncertified,
                     cudaStream_t stream) {
  // cooperative staging when rows and queries allow 16-byte copies
  const bool vec4 = (dim % 4) == 0 && (reinterpret_cast<uintptr_t>(queries) % 16) == 0 &&
                    (reinterpret_cast<uintptr_t>(rows) % 16) == 0;
  const int cw = vec4 ? rerank_chunk_f4(kc, dim) : 0;
  const size_t smem =
      vec4 ? static_cast<size_t>(kRerankStages) * kc * (cw + 1) * 16 : size_t(0);
  static std::atomic<bool> configured[64] = {};  // set once; idempotent
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(rerank_kernel<kMetric, OutIdx>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kRerankStages * kRerankStageBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(n_queries));
  cfg.blockDim = dim3(kRerankThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, rerank_kernel<kMetric, OutIdx>, queries, rows, dim, cand_d,
                            cand_i, kc, k, max_norm2, index_offset, out_d, out_i, sign,
                            uncertified, cw);
}

// Largest |x16|^2 over the rows (norms are >= 0 or NaN/inf, so their bit
// patterns order like the values under a signed-integer maximum).
__global__ void max_norm_kernel(const float* __restrict__ norms, int64_t n,
                                int* __restrict__ out_bits) {
  int m = 0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    m = max(m, __float_as_int(norms[i]));
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out_bits, m);
}

}  // namespace

cudaError_t launch_rerank(const float* queries, const float* rows, int64_t dim,
                          const float* cand_d, const uint32_t* cand_i, int kc, int k,
                          int64_t n_queries, int metric, const float* max_norm2,
                          int64_t index_offset, float* out_d, void* out_i, bool out_i64,
                          bool negate_out, int* uncertified, cudaStream_t stream) {
  if (n_queries <= 0 || k <= 0) return cudaSuccess;
  if (kc < k || kc > kRerankThreads || n_queries > 0x7fffffff) return cudaErrorInvalidValue;
  const float sign = negate_out ? -1.0f : 1.0f;
  const bool ip = metric == KNN_METRIC_INNER_PRODUCT;
  if (ip && out_i64)
    return launch_t<KNN_METRIC_INNER_PRODUCT, int64_t>(
        queries, rows, dim, cand_d, cand_i, kc, k, n_queries, max_norm2, index_offset, out_d,
        static_cast<int64_t*>(out_i), sign, uncertified, stream);
  if (ip)
    return launch_t<KNN_METRIC_INNER_PRODUCT, uint32_t>(
        queries, rows, dim, cand_d, cand_i, kc, k, n_queries, max_norm2, index_offset, out_d,
        static_cast<uint32_t*>(out_i), sign, uncertified, stream);
  if (out_i64)
    return launch_t<KNN_METRIC_L2_EXPANDED, int64_t>(
        queries, rows, dim, cand_d, cand_i, kc, k, n_queries, max_norm2, index_offset, out_d,
        static_cast<int64_t*>(out_i), sign, uncertified, stream);
  return launch_t<KNN_METRIC_L2_EXPANDED, uint32_t>(
      queries, rows, dim, cand_d, cand_i, kc, k, n_queries, max_norm2, index_offset, out_d,
      static_cast<uint32_t*>(out_i), sign, uncertified, stream);
}

double rerank_bound(int metric, double r, double qn, double xn, int64_t dim) {
  return metric == KNN_METRIC_INNER_PRODUCT ? bound_ip(qn, xn, dim) : bound_l2(r, qn, xn, dim);
}

cudaError_t launch_max_norm(const float* norms, int64_t n, float* out, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float), stream);
  if (e != cudaSuccess || n <= 0) return e;
  int blocks = static_cast<int>((n + 255) / 256);
  if (blocks > 1184) blocks = 1184;
  max_norm_kernel<<<blocks, 256, 0, stream>>>(norms, n, reinterpret_cast<int*>(out));
  return cudaGetLastError();
}

}  // namespace knn
