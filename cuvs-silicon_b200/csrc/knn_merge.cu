// knn_merge.cu -- merge of sorted per-unit (or per-rank) top-k lists.
//
// The reference selects its final top-k with a serial pass of thread 0 over
// 128 per-thread lists followed by an insertion sort
// (shaders/cagra_kernels.metal:636-649).  Here one CTA of 8 warps owns one
// query and the order is (distance, index), as src/cagra.cpp:229-238;
// missing entries are (+inf, UINT32_MAX), the padding of
// src/cagra.cpp:245-250.
//
// Threshold path (default).  The input lists are sorted.  With S lists and
// j = ceil(k / S), let tau be the ceil(k / j)-th smallest of the lists' j-th
// entries (lexicographic (distance, index)): ceil(k / j) lists then hold j
// entries each that are <= tau, so the merged k-th entry is <= tau and only
// entries <= tau can be in the result.  (For k <= S, tau is the k-th
// smallest list head.)  The CTA finds tau with a small shared-memory sort,
// filters the entries <= tau into a candidate array and sorts that with one
// block-wide bitonic sort; typically about k entries pass.
//
// Fold path (fallback when more than kCandCap entries pass, e.g. massive
// exact ties).  Lists are staged in shared memory in batches; each warp
// keeps a sorted list of K2 = 32 * E entries in registers (element
// e = r * 32 + lane) and folds lists in with a bitonic merge:
//   C[e] = min(A[e], B[K2 - 1 - e])   (the K2 smallest of A u B, bitonic)
//   then log2(K2) compare-exchange stages (register swaps for strides >= 32,
//   warp shuffles below); the 8 warp lists are folded last by warp 0.
//
// The kernel is launched as a programmatic dependent of the kernel before it
// in the stream and waits (griddepcontrol.wait) before reading its input.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "knn_internal.h"
#include "ptx.cuh"

namespace knn {

namespace {

constexpr int kMergeWarps = 8;
constexpr int kStageEntries = 6144;  // 48 KiB of (fp32, uint32) entries (fold path)
constexpr int kSelCap = 2048;        // lists' j-th entries (threshold path)
constexpr int kCandCap = 4096;       // threshold-path candidates
constexpr int kRankPlaceMax = 1024;  // candidates ordered by rank counting (4 per thread)
// Lists longer than this: prefix lengths by binary search, candidates copied
// by the whole block, and rank counting only up to kRankPlaceLong of them
// (it is quadratic; the block-wide sort takes over above).
constexpr int kLongList = 128;
constexpr int kRankPlaceLong = 256;
// Entries per list in the fallback threshold sample (see merge_query).
constexpr int kSampleJ = 8;
static_assert(kSelCap + kCandCap <= kStageEntries, "threshold arrays share the stage");

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
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const float bd = __shfl_sync(0xffffffffu, b.d[E - 1 - r], 31 - lane);
    const uint32_t bi = __shfl_sync(0xffffffffu, b.i[E - 1 - r], 31 - lane);
    if (less_pair(bd, bi, a.d[r], a.i[r])) {
      a.d[r] = bd;
      a.i[r] = bi;
    }
  }
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

template <typename OutIdx>
__device__ __forceinline__ void store_out(float* out_d, OutIdx* out_i, int64_t at, float d,
                                          uint32_t idx, int64_t index_offset, float sign) {
  out_d[at] = sign * d + 0.0f;  // + 0 maps -0 to +0
  if constexpr (sizeof(OutIdx) == 8) {
    out_i[at] = idx == kNoIndex ? OutIdx(-1) : static_cast<OutIdx>(idx) + index_offset;
  } else {
    out_i[at] = idx == kNoIndex ? kNoIndex : static_cast<uint32_t>(idx + index_offset);
  }
}

// Block-wide ascending bitonic sort of p2 (a power of two) entries in
// shared memory.  All threads of the block call it.
__device__ __forceinline__ void block_sort(float* d, uint32_t* i, int p2) {
  for (int size = 2; size <= p2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int a = threadIdx.x; a < p2 / 2; a += blockDim.x) {
        const int lo = 2 * a - (a & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const float dl = d[lo], dh = d[hi];
        const uint32_t il = i[lo], ih = i[hi];
        if (less_pair(dh, ih, dl, il) == up) {
          d[lo] = dh;
          i[lo] = ih;
          d[hi] = dl;
          i[hi] = il;
        }
      }
      __syncthreads();
    }
  }
}

// Order-preserving 32-bit image of a distance (-0 counted as +0, which the
// (distance, index) order treats as equal).
__device__ __forceinline__ uint32_t order_key(float d) {
  const uint32_t u = __float_as_uint(d == 0.0f ? 0.0f : d);
  return u ^ ((u >> 31) ? 0xFFFFFFFFu : 0x80000000u);
}

// Inverse of order_key.
__device__ __forceinline__ float key_float(uint32_t b) {
  return __uint_as_float(b ^ ((b >> 31) ? 0x80000000u : 0xFFFFFFFFu));
}

// The image (order_key) of the k-th smallest of d[0..n), 1 <= k <= n, by a
// radix select: four passes over the 8-bit digits from the top, each a
// shared-memory histogram of the entries that match the digits chosen so far
// and a block scan that finds the digit holding the k-th.  blockDim.x ==
// 256 (one histogram bin per thread); hist: 256 ints, misc: 10 ints.
// Called by every thread; ends with a block barrier.
__device__ uint32_t block_select_kth(const float* d, int n, int k, int* hist, int* misc) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t prefix = 0, mask = 0;
  int want = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    hist[tid] = 0;
    __syncthreads();
    for (int e = tid; e < n; e += blockDim.x) {
      const uint32_t key = order_key(d[e]);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1);
    }
    __syncthreads();
    const int h = hist[tid];
    int incl = h;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) misc[warp] = incl;
    __syncthreads();
    for (int w = 0; w < warp; ++w) incl += misc[w];
    if (incl - h < want && want <= incl) {  // exactly one bin
      misc[8] = tid;
      misc[9] = incl - h;
    }
    __syncthreads();
    want -= misc[9];
    prefix |= static_cast<uint32_t>(misc[8]) << shift;
    mask |= 255u << shift;
    __syncthreads();
  }
  return prefix;
}

// Sorts n <= blockDim.x entries by rank counting: thread t takes entry t,
// counts the entries ordered before it (one broadcast shared-memory read per
// entry, no barrier in between) and stores it at that rank in out_d/out_i,
// which must not alias in_d/in_i.  Keys are distinct except for padding
// entries, which land on the positions their rank gives (all padding values
// are equal, so any of them may fill those slots); only ranks < limit are
// stored.  Called by every thread; ends with a block barrier.
__device__ __forceinline__ void rank_place(const float* in_d, const uint32_t* in_i, int n,
                                           float* out_d, uint32_t* out_i, int limit) {
  // n <= kRankPlaceMax: thread t ranks entries t, t + blockDim.x, ...
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    const float d = in_d[t];
    const uint32_t i = in_i[t];
    int rank = 0;
    for (int u = 0; u < n; ++u) rank += less_pair(in_d[u], in_i[u], d, i) ? 1 : 0;
    if (rank < limit) {
      out_d[rank] = d;
      out_i[rank] = i;
    }
  }
  __syncthreads();
}

// Fold path: folds every list of the query; leaves the first k entries of
// the result in res_d / res_i (shared memory, read after a block barrier).
template <int E>
__device__ void fold_merge(float* sd, uint32_t* si, const float* qd, const uint32_t* qi,
                           int64_t stride_list, int n_lists, int k, float* res_d,
                           uint32_t* res_i) {
  constexpr int K2 = 32 * E;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  List<E> acc;
  fill_inf(acc);
  const int batch = kStageEntries / k < n_lists ? kStageEntries / k : n_lists;
  for (int l0 = 0; l0 < n_lists; l0 += batch) {
    const int nb = n_lists - l0 < batch ? n_lists - l0 : batch;
    for (int e = threadIdx.x; e < nb * k; e += blockDim.x) {
      const int l = e / k;
      const int r = e - l * k;
      const int64_t at = static_cast<int64_t>(l0 + l) * stride_list + r;
      sd[e] = qd[at];
      si[e] = qi[at];
    }
    __syncthreads();
    for (int l = warp; l < nb; l += kMergeWarps) {
      float kd;
      uint32_t ki;
      get_entry(acc, k - 1, kd, ki);
      if (!less_pair(sd[l * k], si[l * k], kd, ki)) continue;  // cannot improve
      List<E> b;
      load_list(b, sd + l * k, si + l * k, k, lane);
      merge_into(acc, b, lane);
    }
    __syncthreads();
  }
  if (warp > 0) {
#pragma unroll
    for (int r = 0; r < E; ++r) {
      sd[warp * K2 + r * 32 + lane] = acc.d[r];
      si[warp * K2 + r * 32 + lane] = acc.i[r];
    }
  }
  __syncthreads();
  if (warp == 0) {
  for (int w = 1; w < kMergeWarps && w < n_lists; ++w) {
    List<E> b;
#pragma unroll
    for (int r = 0; r < E; ++r) {
      b.d[r] = sd[w * K2 + r * 32 + lane];
      b.i[r] = si[w * K2 + r * 32 + lane];
    }
    merge_into(acc, b, lane);
  }
  }
  __syncthreads();  // every warp is done reading the staged lists
  if (warp == 0) {
#pragma unroll
    for (int r = 0; r < E; ++r) {
      const int e = r * 32 + lane;
      if (e < k) {
        res_d[e] = acc.d[r];
        res_i[e] = acc.i[r];
      }
    }
  }
}

__device__ __forceinline__ void ld_relaxed_sys_v2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_v2(uint64_t* p, uint64_t a, uint64_t b) {
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}

// Mode 2: the block collects every rank's list for query q from this
// rank's exchange buffer, waiting (bounded by ex.wait_ns) until both words of
// each entry carry this search's epoch, and decodes them to ex.dec_d/dec_i.
// Returns false (for the whole block) after recording kErrTimeoutPeer when an
// entry never arrives, or as soon as another block has recorded an error
// (so a missing peer costs one bound, not one bound per wave of blocks).
__device__ bool receive_lists(const Exchange& ex, uint32_t epoch, int64_t q, int k,
                              int* s_abort) {
  if (threadIdx.x == 0) *s_abort = 0;
  __syncthreads();
  const uint64_t* own = reinterpret_cast<const uint64_t*>(ex.base[ex.rank]);
  const int parity = static_cast<int>(epoch & 1u);
  const int total = ex.n_ranks * k;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int r = i / k;
    const int e = i - r * k;
    const uint64_t* src =
        own + ((static_cast<int64_t>(parity) * ex.n_ranks + r) * ex.cap_qk + q * k + e) * 2;
    uint64_t a, b;
    uint64_t t0 = 0;
    uint32_t spins = 0;
    bool ok = true;
    while (true) {
      ld_relaxed_sys_v2(src, a, b);
      if (static_cast<uint32_t>(a >> 32) == epoch && static_cast<uint32_t>(b >> 32) == epoch)
        break;
      if (*reinterpret_cast<volatile int*>(s_abort)) {
        ok = false;
        break;
      }
      if ((++spins & 31u) == 0 && *reinterpret_cast<volatile int*>(ex.err) != 0) {
        *reinterpret_cast<volatile int*>(s_abort) = 1;
        ok = false;
        break;
      }
      uint64_t now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (t0 == 0) t0 = now;
      if (now - t0 > ex.wait_ns) {
        atomicCAS(ex.err, 0, kErrTimeoutPeer);
        *reinterpret_cast<volatile int*>(s_abort) = 1;
        ok = false;
        break;
      }
    }
    if (!ok) break;
    ex.dec_d[q * total + i] = __uint_as_float(static_cast<uint32_t>(a));
    ex.dec_i[q * total + i] = static_cast<uint32_t>(b);
  }
  __syncthreads();
  return *reinterpret_cast<volatile int*>(s_abort) == 0;
}

// Writes the query's first k result entries (the first `count` valid, the
// rest padding) to the output, or in mode 1 to every rank's exchange buffer
// as epoch-tagged words.  Called by every thread of the block.
template <typename OutIdx>
__device__ void emit_result(const Exchange& ex, bool push, uint32_t epoch, int64_t q, int k,
                            const float* rd, const uint32_t* ri, int count,
                            int64_t index_offset, float* out_d, OutIdx* out_i, float sign) {
  const float kInf = __int_as_float(0x7f800000);
  if (!push) {
    for (int e = threadIdx.x; e < k; e += blockDim.x) {
      const bool have = e < count;
      store_out(out_d, out_i, q * k + e, have ? rd[e] : kInf, have ? ri[e] : kNoIndex,
                index_offset, sign);
    }
    return;
  }
  const uint64_t tag = static_cast<uint64_t>(epoch) << 32;
  const int64_t parity = static_cast<int64_t>(epoch & 1u);
  const int64_t at = ((parity * ex.n_ranks + ex.rank) * ex.cap_qk + q * k);
  for (int e = threadIdx.x; e < k; e += blockDim.x) {
    const bool have = e < count;
    const uint32_t idx = have ? ri[e] : kNoIndex;
    const uint32_t gidx = idx == kNoIndex ? kNoIndex : static_cast<uint32_t>(idx + index_offset);
    const uint64_t wd = tag | __float_as_uint(have ? rd[e] : kInf);
    const uint64_t wi = tag | gidx;
    for (int r = 0; r < ex.n_ranks; ++r)
      st_relaxed_sys_v2(reinterpret_cast<uint64_t*>(ex.base[r]) + (at + e) * 2, wd, wi);
  }
}

// Merges the lists of query blockIdx.x (every thread of the block).
template <int E, typename OutIdx>
__device__ __forceinline__ void merge_query(const float* __restrict__ in_d,
                                            const uint32_t* __restrict__ in_i,
                                            int64_t stride_list, int64_t stride_query,
                                            int n_lists, int k, int64_t index_offset,
                                            float* __restrict__ out_d,
                                            OutIdx* __restrict__ out_i, const Exchange& ex,
                                            bool push, uint32_t epoch, float sign) {
  extern __shared__ uint8_t smem_raw[];
  float* sd = reinterpret_cast<float*>(smem_raw);
  uint32_t* si = reinterpret_cast<uint32_t*>(sd + kStageEntries);
  __shared__ int s_count;
  __shared__ int s_hist[kMergeWarps * 32];  // radix selects
  __shared__ int s_misc[10];

  const int64_t q = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const float* qd = in_d + q * stride_query;
  const uint32_t* qi = in_i + q * stride_query;
  const float kInf = __int_as_float(0x7f800000);

  // tau: the r-th smallest of the lists' j-th entries
  const int j = (k + n_lists - 1) / n_lists;  // >= 1
  const int r = (k + j - 1) / j;               // <= n_lists
  float* seld = sd;
  uint32_t* seli = si;
  float* cd = sd + kSelCap;
  uint32_t* ci = si + kSelCap;
  if (n_lists > kSelCap) {
    fold_merge<E>(sd, si, qd, qi, stride_list, n_lists, k, sd + kSelCap, si + kSelCap);
    __syncthreads();
    emit_result(ex, push, epoch, q, k, sd + kSelCap, si + kSelCap, k, index_offset, out_d, out_i, sign);
    return;
  }
  int p2 = 1;
  while (p2 < n_lists) p2 <<= 1;
  for (int l = tid; l < p2; l += blockDim.x) {
    if (l < n_lists) {
      const int64_t at = static_cast<int64_t>(l) * stride_list + (j - 1);
      seld[l] = qd[at];
      seli[l] = qi[at];
    } else {
      seld[l] = kInf;
      seli[l] = kNoIndex;
    }
  }
  if (tid == 0) s_count = 0;
  __syncthreads();
  float td;
  uint32_t ti;
  if (n_lists <= static_cast<int>(blockDim.x)) {
    // rank counting: the entry of rank r - 1 is tau (cd/ci are free here)
    if (tid == 0) {
      cd[0] = kInf;
      ci[0] = kNoIndex;
    }
    __syncthreads();
    if (tid < n_lists) {
      const float d = seld[tid];
      const uint32_t i = seli[tid];
      int rank = 0;
      for (int u = 0; u < n_lists; ++u) rank += less_pair(seld[u], seli[u], d, i) ? 1 : 0;
      if (rank == r - 1) {
        cd[0] = d;
        ci[0] = i;
      }
    }
    __syncthreads();
    td = cd[0];
    ti = ci[0];
    __syncthreads();
  } else {
    block_sort(seld, seli, p2);
    td = seld[r - 1];
    ti = seli[r - 1];
  }

  // Fewer than r lists hold j entries (the scan's shared bound leaves many
  // unit lists short), so tau is the padding.  The first kSampleJ entries
  // of every list then give a bound instead: if at least k of them are
  // valid, their k-th smallest distance D has k entries at or below it, so
  // (D, any index) bounds the merged k-th entry; with short lists D is
  // close to it.  (Without this, thousands of candidates went to the fold.)
  if (ti == kNoIndex && n_lists * kSampleJ <= kSelCap && k <= n_lists * kSampleJ) {
    __syncthreads();  // every thread has read tau from the selection array
    const int ns = n_lists * kSampleJ;
    for (int e = tid; e < ns; e += blockDim.x) {
      const int l = e / kSampleJ, rr = e - l * kSampleJ;
      float dv = kInf;
      if (rr < k) {
        const int64_t at = static_cast<int64_t>(l) * stride_list + rr;
        if (qi[at] != kNoIndex) dv = qd[at];
      }
      seld[e] = dv;
    }
    __syncthreads();
    const uint32_t kth = block_select_kth(seld, ns, k, s_hist, s_misc);
    if (kth != order_key(kInf)) {
      td = key_float(kth);
      ti = kNoIndex - 1u;  // every entry at distance D is kept
    }
  }

  // candidates: every valid entry (d, i) <= tau (every valid entry when
  // tau is the padding, i.e. when fewer than r lists have j entries)
  const int total = n_lists * k;
  constexpr int kPer = 8;  // entries per thread per round, loaded before use
  if (n_lists <= static_cast<int>(blockDim.x) && k > kLongList) {
    // Long lists: the length of each list's prefix <= tau, found by the
    // warps: warp w takes lists w, w + 8, ... in batches of kPrefixBatch,
    // lane e reading entry e of every list of the batch (independent loads,
    // one memory round per batch); a list's prefix length is the popcount
    // of the ballot of its entries <= tau, extended 32 entries at a time in
    // the rare case that all 32 pass.  A block scan then turns the lengths
    // into offsets and all threads copy the candidates together.  The
    // offsets reuse the selection array (tau is already in registers).
    int* off = reinterpret_cast<int*>(seli);  // [n_lists + 1]
    constexpr int kPrefixBatch = 8;
    const int warp = tid >> 5;
    auto passes = [&](float dm, uint32_t im) {
      return im != kNoIndex && (dm < td || (dm == td && im <= ti));
    };
    for (int l0 = warp; l0 < n_lists; l0 += kMergeWarps * kPrefixBatch) {
      float dv[kPrefixBatch];
      uint32_t iv[kPrefixBatch];
#pragma unroll
      for (int b = 0; b < kPrefixBatch; ++b) {
        const int l = l0 + b * kMergeWarps;
        dv[b] = 0.0f;
        iv[b] = kNoIndex;
        if (l < n_lists && lane < k) {
          const int64_t at = static_cast<int64_t>(l) * stride_list + lane;
          iv[b] = qi[at];
          dv[b] = qd[at];
        }
      }
#pragma unroll
      for (int b = 0; b < kPrefixBatch; ++b) {
        const int l = l0 + b * kMergeWarps;  // warp-uniform
        if (l >= n_lists) continue;
        unsigned m = __ballot_sync(0xffffffffu, passes(dv[b], iv[b]));
        int len = __popc(m);
        for (int e0 = 32; m == 0xffffffffu && e0 < k; e0 += 32) {
          const int e = e0 + lane;
          const int64_t at = static_cast<int64_t>(l) * stride_list + e;
          const bool p = e < k && passes(qd[at], qi[at]);
          m = __ballot_sync(0xffffffffu, p);
          len += __popc(m);
        }
        if (lane == 0) off[l] = len;
      }
    }
    __syncthreads();
    const int len = tid < n_lists ? off[tid] : 0;
    // exclusive scan of the lengths: warp scans, then the warp totals
    __shared__ int s_warp[kMergeWarps];
    int incl = len;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) s_warp[tid >> 5] = incl;
    __syncthreads();
    int base = 0;
    for (int w = 0; w < (tid >> 5); ++w) base += s_warp[w];
    if (tid < n_lists) off[tid] = base + incl - len;
    if (tid == static_cast<int>(blockDim.x) - 1) s_count = base + incl;
    __syncthreads();
    const int cnt = s_count < kCandCap ? s_count : kCandCap;
    for (int c = tid; c < cnt; c += blockDim.x) {
      // list of candidate c: the last l with off[l] <= c
      int a = 0, b = n_lists - 1;
      while (a < b) {
        const int m = (a + b + 1) >> 1;
        if (off[m] <= c) a = m;
        else b = m - 1;
      }
      const int64_t at = static_cast<int64_t>(a) * stride_list + (c - off[a]);
      cd[c] = qd[at];
      ci[c] = qi[at];
    }
  } else if (n_lists <= static_cast<int>(blockDim.x)) {
    // The lists are sorted, so a list's candidates are a prefix of it:
    // thread l reads list l four entries at a time (independent loads) and
    // stops at the first entry above tau or at the padding.
    if (tid < n_lists) {
      const float* lsd = qd + static_cast<int64_t>(tid) * stride_list;
      const uint32_t* lsi = qi + static_cast<int64_t>(tid) * stride_list;
      bool more = true;
      for (int e0 = 0; e0 < k && more; e0 += 4) {
        float dv[4];
        uint32_t iv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = e0 + u;
          dv[u] = e < k ? lsd[e] : kInf;
          iv[u] = e < k ? lsi[e] : kNoIndex;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          more = more && iv[u] != kNoIndex && (dv[u] < td || (dv[u] == td && iv[u] <= ti));
          if (more) {
            const int pos = atomicAdd(&s_count, 1);
            if (pos < kCandCap) {
              cd[pos] = dv[u];
              ci[pos] = iv[u];
            }
          }
        }
      }
    }
  } else {
  for (int e0 = 0; e0 < total; e0 += kPer * kMergeWarps * 32) {
    float dv[kPer];
    uint32_t iv[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int e = e0 + u * kMergeWarps * 32 + tid;
      iv[u] = kNoIndex;
      dv[u] = kInf;
      if (e < total) {
        const int l = e / k;
        const int rr = e - l * k;
        const int64_t at = static_cast<int64_t>(l) * stride_list + rr;
        iv[u] = qi[at];
        dv[u] = qd[at];
      }
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const bool take = iv[u] != kNoIndex && (dv[u] < td || (dv[u] == td && iv[u] <= ti));
      // warp-aggregated append: one shared atomic per warp
      const unsigned ballot = __ballot_sync(0xffffffffu, take);
      if (ballot) {
        int base = 0;
        if (lane == 0) base = atomicAdd(&s_count, __popc(ballot));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (take) {
          const int pos = base + __popc(ballot & ((1u << lane) - 1u));
          if (pos < kCandCap) {
            cd[pos] = dv[u];
            ci[pos] = iv[u];
          }
        }
      }
    }
  }
  }
  __syncthreads();
  const int count = s_count;
  if (count > kCandCap) {  // block-uniform
    __syncthreads();
    fold_merge<E>(sd, si, qd, qi, stride_list, n_lists, k, cd, ci);
    __syncthreads();
    emit_result(ex, push, epoch, q, k, cd, ci, k, index_offset, out_d, out_i, sign);
    return;
  }
  if (count <= (k > kLongList ? kRankPlaceLong : kRankPlaceMax)) {
    // candidates are distinct (distinct row indices): rank counting places
    // the first k of them, sorted, in front of the selection array
    rank_place(cd, ci, count, seld, seli, k);
    emit_result(ex, push, epoch, q, k, seld, seli, count, index_offset, out_d, out_i, sign);
    return;
  }
  if (count > 2 * kRankPlaceLong) {
    // Many candidates (a loose tau, or none when fewer than r lists hold j
    // entries): the k-th smallest distance D by a radix select, then only
    // the entries at or below D (k of them, more only with ties at D) are
    // ordered, by rank counting.  Up to 512 candidates the block-wide sort
    // is as fast (same-box A/B: K = 200, ~340 candidates, 20.5 us sorted
    // against 22.5 us selected; K = 256, ~570 candidates, 26.6 -> 24.4 us).
    // With ~3,800 candidates (tau the padding) a traced search spent 88 to
    // 160 us per query block in the 4096-entry sort; with the select the
    // whole search (125k rows, Q = 16, K = 256) went 130.7 -> 116.1 us.
    const uint32_t kth = block_select_kth(cd, count, k, s_hist, s_misc);
    if (tid == 0) s_count = 0;
    __syncthreads();
    for (int e = tid; e < count; e += blockDim.x) {
      if (order_key(cd[e]) <= kth) {
        const int pos = atomicAdd(&s_count, 1);
        if (pos < kSelCap) {
          seld[pos] = cd[e];
          seli[pos] = ci[e];
        }
      }
    }
    __syncthreads();
    const int m = s_count;  // >= k
    if (m <= kSelCap && m <= kRankPlaceLong) {
      rank_place(seld, seli, m, cd, ci, k);
      emit_result(ex, push, epoch, q, k, cd, ci, k, index_offset, out_d, out_i, sign);
      return;
    }
  }
  // at most 512 candidates, or more than 256 ties at the k-th distance:
  // sort every candidate
  int c2 = 1;
  while (c2 < count) c2 <<= 1;
  for (int e = count + tid; e < c2; e += blockDim.x) {
    cd[e] = kInf;
    ci[e] = kNoIndex;
  }
  __syncthreads();
  block_sort(cd, ci, c2);
  emit_result(ex, push, epoch, q, k, cd, ci, count, index_offset, out_d, out_i, sign);
}

template <int E, typename OutIdx>
__global__ void __launch_bounds__(kMergeWarps * 32, 4)
    merge_kernel(const float* __restrict__ in_d, const uint32_t* __restrict__ in_i,
                 int64_t stride_list, int64_t stride_query, int n_lists, int k,
                 int64_t index_offset, float* __restrict__ out_d, OutIdx* __restrict__ out_i,
                 const __grid_constant__ Exchange ex, float sign) {
  // The next kernel may be scheduled now; it waits for this one to finish
  // before it reads anything this kernel writes.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ int s_abort;
  const int64_t q = blockIdx.x;
  // Everything this kernel reads was written by kernels before it in the
  // stream; in particular the exchange epoch, which the query conversion
  // that opened this search incremented.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // debug builds: every list this block reads (and, with an exchange, every
  // slot it writes or polls) lies inside its buffer
  const int64_t last_in = q * stride_query + static_cast<int64_t>(n_lists - 1) * stride_list + k;
  if (!in_bounds(ex.in_len <= 0 || last_in <= ex.in_len, ex.err)) return;
  if (ex.mode != 0 && !in_bounds((q + 1) * k <= ex.cap_qk && ex.n_ranks <= kMaxRanks, ex.err))
    return;
  const uint32_t epoch = ex.mode != 0 ? *reinterpret_cast<const volatile uint32_t*>(ex.epoch) : 0u;
  if (ex.mode == 1) {
    // Exchange, one block per query from end to end: merge this rank's
    // per-unit lists and push the result into every rank's exchange buffer
    // (NVLink stores), then collect every rank's list for the same query
    // from this rank's own buffer (bounded wait), decode and merge them.
    // No block waits for another block of this GPU, only for the block of
    // the same query on each peer.
    merge_query<E, OutIdx>(in_d, in_i, stride_list, stride_query, n_lists, k, index_offset,
                           nullptr, nullptr, ex, true, epoch, 1.0f);
    if (receive_lists(ex, epoch, q, k, &s_abort))
      merge_query<E, OutIdx>(ex.dec_d, ex.dec_i, k, static_cast<int64_t>(ex.n_ranks) * k,
                             ex.n_ranks, k, 0, out_d, out_i, ex, false, epoch, sign);
    return;
  }
  merge_query<E, OutIdx>(in_d, in_i, stride_list, stride_query, n_lists, k, index_offset, out_d,
                         out_i, ex, false, epoch, sign);
}

template <int E>
cudaError_t launch_e(const float* in_d, const uint32_t* in_i, int64_t stride_list,
                     int64_t stride_query, int n_lists, int k, int64_t n_queries,
                     int64_t index_offset, float* out_d, void* out_i, bool out_i64,
                     cudaStream_t stream, bool overlap, const Exchange& ex, float sign) {
  static_assert(kMergeWarps * 32 * E <= kStageEntries, "warp lists fit the staging area");
  static_assert(kCandCap <= kStageEntries, "candidates fit the staging area");
  constexpr size_t smem = static_cast<size_t>(kStageEntries) * 8;
  // opt in to more than 48 KiB of dynamic shared memory once per device
  static std::atomic<bool> configured[64][2] = {};  // set once; idempotent
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const int w = out_i64 ? 1 : 0;
  if (dev < 0 || dev >= 64 || !configured[dev][w]) {
    e = out_i64 ? cudaFuncSetAttribute(merge_kernel<E, int64_t>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem))
                : cudaFuncSetAttribute(merge_kernel<E, uint32_t>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    // same shared-memory carve-out as the scan kernel: no SM reconfiguration
    // between the two
    e = out_i64 ? cudaFuncSetAttribute(merge_kernel<E, int64_t>,
                                       cudaFuncAttributePreferredSharedMemoryCarveout, 100)
                : cudaFuncSetAttribute(merge_kernel<E, uint32_t>,
                                       cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev][w] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(n_queries));
  cfg.blockDim = dim3(kMergeWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = overlap ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (out_i64) {
    return cudaLaunchKernelEx(&cfg, merge_kernel<E, int64_t>, in_d, in_i, stride_list,
                              stride_query, n_lists, k, index_offset, out_d,
                              static_cast<int64_t*>(out_i), ex, sign);
  }
  return cudaLaunchKernelEx(&cfg, merge_kernel<E, uint32_t>, in_d, in_i, stride_list,
                            stride_query, n_lists, k, index_offset, out_d,
                            static_cast<uint32_t*>(out_i), ex, sign);
}

}  // namespace

cudaError_t launch_merge(const float* in_d, const uint32_t* in_i, int64_t stride_list,
                         int64_t stride_query, int n_lists, int k, int64_t n_queries,
                         int64_t index_offset, float* out_d, void* out_i, bool out_i64,
                         cudaStream_t stream, bool overlap, const Exchange* ex_opt,
                         bool negate_out, int* err, int64_t in_len) {
  if (n_queries <= 0 || k <= 0) return cudaSuccess;
  const float sign = negate_out ? -1.0f : 1.0f;
  Exchange none = {};
  none.err = err;
  none.in_len = in_len;
  const Exchange& ex = ex_opt ? *ex_opt : none;
  if (n_queries > 0x7fffffff) return cudaErrorInvalidValue;
  if (k <= 32)
    return launch_e<1>(in_d, in_i, stride_list, stride_query, n_lists, k, n_queries,
                       index_offset, out_d, out_i, out_i64, stream, overlap, ex, sign);
  if (k <= 64)
    return launch_e<2>(in_d, in_i, stride_list, stride_query, n_lists, k, n_queries,
                       index_offset, out_d, out_i, out_i64, stream, overlap, ex, sign);
  if (k <= 128)
    return launch_e<4>(in_d, in_i, stride_list, stride_query, n_lists, k, n_queries,
                       index_offset, out_d, out_i, out_i64, stream, overlap, ex, sign);
  if (k <= 256)
    return launch_e<8>(in_d, in_i, stride_list, stride_query, n_lists, k, n_queries,
                       index_offset, out_d, out_i, out_i64, stream, overlap, ex, sign);
  return cudaErrorInvalidValue;
}

}  // namespace knn
