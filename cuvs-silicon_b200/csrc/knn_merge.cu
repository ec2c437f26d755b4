// knn_merge.cu -- merge of sorted per-unit (or per-rank) top-k lists.
//
// The reference selects its final top-k with a serial pass of thread 0 over
// 128 per-thread lists followed by an insertion sort
// (shaders/cagra_kernels.metal:636-649).  Here one CTA of 8 warps owns one
// query: each warp keeps a sorted list of K2 = 32 * E entries in registers
// (E per lane, element e = r * 32 + lane) and folds in one input list at a
// time with a bitonic merge:
//   C[e] = min(A[e], B[K2 - 1 - e])      (the K2 smallest of A u B, bitonic)
//   then log2(K2) compare-exchange stages (register swaps for strides >= 32,
//   warp shuffles below).
// A list whose best entry is not better than the running k-th entry is
// skipped after one compare.  The 8 warp lists are then folded by warp 0
// through shared memory.  Order is (distance, index), as
// src/cagra.cpp:229-238; missing entries stay (+inf, UINT32_MAX), the
// padding of src/cagra.cpp:245-250.
#include <cuda_runtime.h>

#include <cstdint>

#include "knn_internal.h"

namespace knn {

namespace {

constexpr int kMergeWarps = 8;

__device__ __forceinline__ bool less_pair(float da, uint32_t ia, float db, uint32_t ib) {
  return da < db || (da == db && ia < ib);
}

template <int E>
struct List {
  float d[E];
  uint32_t i[E];
};

template <int E>
__device__ __forceinline__ void fill_inf(List<E>& l) {
#pragma unroll
  for (int r = 0; r < E; ++r) {
    l.d[r] = __int_as_float(0x7f800000);
    l.i[r] = kNoIndex;
  }
}

// Loads a sorted list of k entries (padded to K2 with +inf).
template <int E>
__device__ __forceinline__ void load_list(List<E>& l, const float* d, const uint32_t* i, int k,
                                          int lane) {
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const int e = r * 32 + lane;
    if (e < k) {
      l.d[r] = d[e];
      l.i[r] = i[e];
    } else {
      l.d[r] = __int_as_float(0x7f800000);
      l.i[r] = kNoIndex;
    }
  }
}

// a <- the K2 smallest of (a, b), sorted ascending; both inputs sorted.
template <int E>
__device__ __forceinline__ void merge_into(List<E>& a, const List<E>& b, int lane) {
  // reverse b and take the element-wise minimum -> bitonic sequence
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const float bd = __shfl_sync(0xffffffffu, b.d[E - 1 - r], 31 - lane);
    const uint32_t bi = __shfl_sync(0xffffffffu, b.i[E - 1 - r], 31 - lane);
    if (less_pair(bd, bi, a.d[r], a.i[r])) {
      a.d[r] = bd;
      a.i[r] = bi;
    }
  }
  // bitonic merge, strides K2/2 ... 32 inside the thread
#pragma unroll
  for (int rs = E / 2; rs >= 1; rs >>= 1) {
#pragma unroll
    for (int r = 0; r < E; ++r) {
      if ((r & rs) == 0) {
        const int p = r | rs;
        if (less_pair(a.d[p], a.i[p], a.d[r], a.i[r])) {
          const float td = a.d[r];
          const uint32_t ti = a.i[r];
          a.d[r] = a.d[p];
          a.i[r] = a.i[p];
          a.d[p] = td;
          a.i[p] = ti;
        }
      }
    }
  }
  // strides 16 ... 1 across lanes
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int r = 0; r < E; ++r) {
      const float od = __shfl_xor_sync(0xffffffffu, a.d[r], s);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, a.i[r], s);
      const bool other_less = less_pair(od, oi, a.d[r], a.i[r]);
      // lower lane keeps the minimum, upper lane the maximum
      if (other_less != upper) {
        a.d[r] = od;
        a.i[r] = oi;
      }
    }
  }
}

// Entry e of the warp list, broadcast to all lanes.
template <int E>
__device__ __forceinline__ void get_entry(const List<E>& l, int e, float& d, uint32_t& i) {
  const int r = e >> 5;
  float dv = l.d[0];
  uint32_t iv = l.i[0];
#pragma unroll
  for (int rr = 1; rr < E; ++rr) {
    if (rr == r) {
      dv = l.d[rr];
      iv = l.i[rr];
    }
  }
  d = __shfl_sync(0xffffffffu, dv, e & 31);
  i = __shfl_sync(0xffffffffu, iv, e & 31);
}

template <int E, typename OutIdx>
__global__ void __launch_bounds__(kMergeWarps * 32)
    merge_kernel(const float* __restrict__ in_d, const uint32_t* __restrict__ in_i,
                 int64_t stride_list, int64_t stride_query, int n_lists, int k,
                 int64_t index_offset, float* __restrict__ out_d, OutIdx* __restrict__ out_i) {
  extern __shared__ uint8_t smem_raw[];
  constexpr int K2 = 32 * E;
  float* sd = reinterpret_cast<float*>(smem_raw);
  uint32_t* si = reinterpret_cast<uint32_t*>(sd + kMergeWarps * K2);

  const int64_t q = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const float* qd = in_d + q * stride_query;
  const uint32_t* qi = in_i + q * stride_query;

  List<E> acc;
  fill_inf(acc);
  for (int l = warp; l < n_lists; l += kMergeWarps) {
    const float* ld = qd + l * stride_list;
    const uint32_t* li = qi + l * stride_list;
    // skip lists that cannot improve the current k-th entry
    float kd;
    uint32_t ki;
    get_entry(acc, k - 1, kd, ki);
    const float b0d = ld[0];
    const uint32_t b0i = li[0];
    if (!less_pair(b0d, b0i, kd, ki)) continue;
    List<E> b;
    load_list(b, ld, li, k, lane);
    merge_into(acc, b, lane);
  }
  if (warp > 0) {
#pragma unroll
    for (int r = 0; r < E; ++r) {
      sd[warp * K2 + r * 32 + lane] = acc.d[r];
      si[warp * K2 + r * 32 + lane] = acc.i[r];
    }
  }
  __syncthreads();
  if (warp != 0) return;
  for (int w = 1; w < kMergeWarps && w < n_lists; ++w) {
    List<E> b;
#pragma unroll
    for (int r = 0; r < E; ++r) {
      b.d[r] = sd[w * K2 + r * 32 + lane];
      b.i[r] = si[w * K2 + r * 32 + lane];
    }
    merge_into(acc, b, lane);
  }
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const int e = r * 32 + lane;
    if (e < k) {
      const uint32_t idx = acc.i[r];
      out_d[q * k + e] = acc.d[r];
      if constexpr (sizeof(OutIdx) == 8) {
        out_i[q * k + e] = idx == kNoIndex ? OutIdx(-1)
                                           : static_cast<OutIdx>(idx) + index_offset;
      } else {
        out_i[q * k + e] =
            idx == kNoIndex ? kNoIndex : static_cast<uint32_t>(idx + index_offset);
      }
    }
  }
}

template <int E>
cudaError_t launch_e(const float* in_d, const uint32_t* in_i, int64_t stride_list,
                     int64_t stride_query, int n_lists, int k, int64_t n_queries,
                     int64_t index_offset, float* out_d, void* out_i, bool out_i64,
                     cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(kMergeWarps) * 32 * E * 8;
  if (smem > 48 * 1024) {
    cudaError_t e = out_i64
                        ? cudaFuncSetAttribute(merge_kernel<E, int64_t>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem))
                        : cudaFuncSetAttribute(merge_kernel<E, uint32_t>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const unsigned grid = static_cast<unsigned>(n_queries);
  if (out_i64) {
    merge_kernel<E, int64_t><<<grid, kMergeWarps * 32, smem, stream>>>(
        in_d, in_i, stride_list, stride_query, n_lists, k, index_offset, out_d,
        static_cast<int64_t*>(out_i));
  } else {
    merge_kernel<E, uint32_t><<<grid, kMergeWarps * 32, smem, stream>>>(
        in_d, in_i, stride_list, stride_query, n_lists, k, index_offset, out_d,
        static_cast<uint32_t*>(out_i));
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_merge(const float* in_d, const uint32_t* in_i, int64_t stride_list,
                         int64_t stride_query, int n_lists, int k, int64_t n_queries,
                         int64_t index_offset, float* out_d, void* out_i, bool out_i64,
                         cudaStream_t stream) {
  if (n_queries <= 0 || k <= 0) return cudaSuccess;
  if (n_queries > 0x7fffffff) return cudaErrorInvalidValue;
  if (k <= 32)
    return launch_e<1>(in_d, in_i, stride_list, stride_query, n_lists, k, n_queries,
                       index_offset, out_d, out_i, out_i64, stream);
  if (k <= 64)
    return launch_e<2>(in_d, in_i, stride_list, stride_query, n_lists, k, n_queries,
                       index_offset, out_d, out_i, out_i64, stream);
  if (k <= 128)
    return launch_e<4>(in_d, in_i, stride_list, stride_query, n_lists, k, n_queries,
                       index_offset, out_d, out_i, out_i64, stream);
  if (k <= 256)
    return launch_e<8>(in_d, in_i, stride_list, stride_query, n_lists, k, n_queries,
                       index_offset, out_d, out_i, out_i64, stream);
  if (k <= 512)
    return launch_e<16>(in_d, in_i, stride_list, stride_query, n_lists, k, n_queries,
                        index_offset, out_d, out_i, out_i64, stream);
  return cudaErrorInvalidValue;
}

}  // namespace knn
