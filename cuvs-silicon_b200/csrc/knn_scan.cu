// knn_scan.cu -- the fused exact-L2 scan kernel for sm_100a.
//
// Replaces the reference's two passes, MPS fp16 GEMM into a Q x N fp32
// `cross` buffer (src/metal_context.mm:202-225) followed by the
// l2_topk_from_cross kernel (shaders/cagra_kernels.metal:604-653), with one
// kernel in which the Q x N matrix never leaves the SM:
//
//   warp 0  (1 thread)  TMA producer: per 64-wide slice of the dimension, a
//                       128-row query slab and a 256-row dataset slab, both
//                       128-byte swizzled, into a ring of shared-memory stages.
//   warp 1  (1 thread)  tcgen05.mma issuer: 128 x 256 x 16 fp16 MMAs into an
//                       fp32 accumulator in tensor memory (TMEM); two
//                       accumulators of 256 columns alternate so the
//                       epilogue of one tile overlaps the MMAs of the next.
//   warps 2-5           epilogue: thread t owns query row t of the tile
//                       (TMEM lane t).  tcgen05.ld brings 32 dataset columns
//                       at a time into registers; d = |q|^2 + |x|^2 - 2 q.x
//                       (squared L2, the expanded form of
//                       shaders/cagra_kernels.metal:624, clamped at 0); a
//                       per-thread threshold rejects almost every candidate
//                       with one compare; survivors are buffered per query
//                       and merged into the query's shared-memory max-heap
//                       by warp-uniform flushes (see epilogue()).
//
// Work is split into units (query tile m, contiguous row range s).  Row
// ranges are cut in 32-row granules, so every unit of a query tile holds the
// same number of rows to within one granule: a unit is a run of full
// 256-row tiles and one narrower last tile (its MMAs use N = its width and
// its rows arrive as 32-row TMA boxes).  A persistent CTA walks units
// blockIdx.x, +gridDim.x, ...; at the end of a unit each query's top-k is
// sorted and written as list s of that query:
// part[(q * splits + s) * k + r].  The merge kernel (knn_merge.cu) reduces
// the lists to the final top-k, ordered by (distance, index) like
// src/cagra.cpp:229-238.
//
// Variants chosen by plan_search (same results, different speed):
//   * CTA pairs (kPair): clusters of two CTAs issue cta_group::2 MMAs with
//     M = 256, each CTA loading its 128 queries and half of every dataset
//     tile, for more than 128 queries;
//   * register top-k (kReg, k <= 16), shared-memory heaps of 8-byte keys,
//     or compact heaps of 6-byte entries (kC);
//   * spread 32-query blocks (ScanParams::spread): the queries sit in all
//     four TMEM lane quadrants, so every epilogue warp owns some;
//   * heaps sized to the batch's rows when there is one query tile.
//
// Every TMA load lands in the issuing CTA only (the same code runs under multi-GPU
// sharding).  Every mbarrier wait is bounded (ptx.cuh).
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "knn_internal.h"
#include "ptx.cuh"

namespace knn {

namespace {

// A (distance, index) pair as one 64-bit key: an order-preserving image of
// the distance's bits above, the index below, so comparing keys as unsigned
// integers is exactly the (distance, index) lexicographic order of
// src/cagra.cpp:233-238.
//   L2: distances are >= 0 (clamped, never -0) or +inf, whose IEEE bit
//       patterns already order like the values: the image is the bits.
//   Inner product (signed values): the image flips every bit of a negative
//       float and only the sign bit of a non-negative one (-inf < ... < -0 <
//       +0 < ... < +inf < NaN); the distance function never produces -0,
//       so equal values have equal images.
template <int kMetric>
__device__ __forceinline__ uint64_t make_key(float d, uint32_t i) {
  uint32_t u = __float_as_uint(d);
  if constexpr (kMetric == KNN_METRIC_INNER_PRODUCT)
    u ^= static_cast<uint32_t>(static_cast<int32_t>(u) >> 31) | 0x80000000u;  // branch-free
  return (static_cast<uint64_t>(u) << 32) | i;
}
template <int kMetric>
__device__ __forceinline__ float key_dist(uint64_t key) {
  uint32_t b = static_cast<uint32_t>(key >> 32);
  if constexpr (kMetric == KNN_METRIC_INNER_PRODUCT)
    b ^= ~static_cast<uint32_t>(static_cast<int32_t>(b) >> 31) | 0x80000000u;
  return __uint_as_float(b);
}
// (+inf, no index)
template <int kMetric>
__host__ __device__ constexpr uint64_t empty_key() {
  return (static_cast<uint64_t>(kMetric == KNN_METRIC_INNER_PRODUCT ? 0xFF800000u : 0x7f800000u)
          << 32) |
         0xFFFFFFFFull;
}

// Heap storage.  Full keys (64 bits), or compact entries: the distance's
// order image in a 32-bit word and the row's offset from the unit's first
// row in a 16-bit word, 6 bytes an entry (a unit then spans at most
// kCompactMaxRows rows).  A compact entry reads back as the 64-bit key
// (image << 32 | offset), which orders like the full key of the same row
// because every row of the unit has the same first row.
template <bool kC>
struct HeapStore {
  uint64_t* h;
  __device__ __forceinline__ uint64_t get(int i) const { return h[i]; }
  __device__ __forceinline__ void set(int i, uint64_t v) const { h[i] = v; }
};
template <>
struct HeapStore<true> {
  uint32_t* hi;
  uint16_t* lo;
  __device__ __forceinline__ uint64_t get(int i) const {
    return (static_cast<uint64_t>(hi[i]) << 32) | lo[i];
  }
  __device__ __forceinline__ void set(int i, uint64_t v) const {
    hi[i] = static_cast<uint32_t>(v >> 32);
    lo[i] = static_cast<uint16_t>(v);
  }
};

// Max-heap of keys stored column-wise: entry `pos` of query row `row` lives
// at [pos * stride + row], so the 32 threads of a warp always touch 32
// consecutive words whatever positions they visit.
template <typename H>
__device__ __forceinline__ void heap_sift_down(const H& h, int size, int stride, int row, int pos,
                                               uint64_t key, int cap, int* err) {
  if (!in_bounds(size <= cap && pos < cap && row < stride, err)) return;
  while (true) {
    int c = 2 * pos + 1;
    if (c >= size) break;
    uint64_t ck = h.get(c * stride + row);
    if (c + 1 < size) {
      const uint64_t rk = h.get((c + 1) * stride + row);
      if (rk > ck) {
        c += 1;
        ck = rk;
      }
    }
    if (ck <= key) break;
    h.set(pos * stride + row, ck);
    pos = c;
  }
  h.set(pos * stride + row, key);
}

// Adds `key` at position pos (= the heap's current size) of a max-heap.
template <typename H>
__device__ __forceinline__ void heap_sift_up(const H& h, int stride, int row, int pos,
                                             uint64_t key, int cap, int* err) {
  if (!in_bounds(pos < cap && row < stride, err)) return;
  while (pos > 0) {
    const int parent = (pos - 1) >> 1;
    const uint64_t pk = h.get(parent * stride + row);
    if (pk >= key) break;
    h.set(pos * stride + row, pk);
    pos = parent;
  }
  h.set(pos * stride + row, key);
}

struct Smem {
  uint8_t* stages;
  uint64_t* heap;  // [k][query_block] keys (full keys)
  uint32_t* heap_hi;  // [k][query_block] distance images (compact heaps)
  uint16_t* heap_lo;  // [k][query_block] row offsets in the unit (compact heaps)
  uint64_t* buf;   // [kRowBuf][query_block] buffered survivor keys
  float* norm_stage;  // [4 epilogue warps][kAccCols] row norms of the current tile
  uint64_t* full;
  uint64_t* empty;
  uint64_t* acc_full;
  uint64_t* acc_empty;
  uint64_t* drain;
  uint64_t* epi_bar;  // the 4 epilogue warps meet here around a unit's list sort
  uint32_t* tmem_slot;
};

// Bytes of one pipeline stage: the query slab and the dataset slab (the
// whole tile's, or with CTA pairs this CTA's half of it).
__host__ __device__ __forceinline__ int stage_bytes(int pair) {
  return kStageA + (pair ? kTileRows / 2 : kTileRows) * kKChunk * 2;
}

__device__ __forceinline__ Smem carve(uint8_t* raw, const ScanParams& p) {
  Smem s;
  const uint32_t base = smem_addr(raw);
  const uint32_t pad = (1024u - (base & 1023u)) & 1023u;
  s.stages = raw + pad;
  uint8_t* const heap0 = s.stages + static_cast<size_t>(p.stages) * stage_bytes(p.pair);
  const size_t entries = static_cast<size_t>(p.k) * p.heap_rows;
  s.heap = reinterpret_cast<uint64_t*>(heap0);
  s.heap_hi = reinterpret_cast<uint32_t*>(heap0);
  s.heap_lo = reinterpret_cast<uint16_t*>(s.heap_hi + entries);
  // heap_rows is a multiple of 8, so the compact arrays end 16-byte aligned
  // (as do the survivor buffers, ahead of the float4 norm staging)
  s.buf = p.compact ? reinterpret_cast<uint64_t*>(s.heap_lo + entries) : s.heap + entries;
  s.norm_stage = reinterpret_cast<float*>(s.buf + static_cast<size_t>(kRowBuf) * p.heap_rows);
  uintptr_t b = reinterpret_cast<uintptr_t>(s.norm_stage + 4 * kAccCols);
  b = (b + 7) & ~static_cast<uintptr_t>(7);
  uint64_t* bars = reinterpret_cast<uint64_t*>(b);
  s.full = bars;
  s.empty = bars + p.stages;
  s.acc_full = bars + 2 * p.stages;
  s.acc_empty = s.acc_full + 2;
  s.drain = s.acc_empty + 2;
  s.epi_bar = s.drain + 1;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.epi_bar + 1);
  return s;
}

// Unit u: query tile m and rows [r0, r_end), whole granules.  At the end of
// the dataset r_end may pass n_rows by less than a granule: TMA fills those
// rows with zeros and the epilogue masks them (row norm +inf).  The pilot
// pass keeps only the unit's first tile.
struct Unit {
  int m;
  int64_t r0, r_end;
};
__device__ __forceinline__ Unit unit_of(const ScanParams& p, int u) {
  Unit x;
  x.m = u % p.query_tiles;
  const int64_t s = u / p.query_tiles;
  x.r0 = s * p.n_gran / p.splits * p.gran_rows;
  x.r_end = (s + 1) * p.n_gran / p.splits * p.gran_rows;
  if (p.pilot && x.r_end > x.r0 + kTileRows) x.r_end = x.r0 + kTileRows;
  return x;
}
// Width (rows, a multiple of kGranRows) of the tile starting at row rs.
__device__ __forceinline__ int tile_width(int64_t rs, int64_t r_end) {
  const int64_t w = r_end - rs;
  return w < kTileRows ? static_cast<int>(w) : kTileRows;
}

// Bounded wait used while unwinding after an error: ignores the error word,
// gives up after ~10 ms.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > 10000000ull) break;
  }
}

// TMA producer.  The kernel is launched as a programmatic dependent of the
// query conversion, so it may start before that kernel's writes are
// visible.  The dataset rows are not written while a search runs (a build
// synchronises before it returns), so the dataset slabs of the first
// stages are requested before griddepcontrol.wait and only the query slabs
// wait for it: the first tile's load overlaps the kernels before this one.
// A full tile's slab is one 256-row box; a narrower tile's slab is w / 32
// boxes of 32 rows placed one after the other, which gives the same
// shared-memory layout for its first w rows (every box starts on a 1024-byte
// swizzle atom).
template <bool kPair>
__device__ void producer(const CUtensorMap* qmap, const CUtensorMap* xmap,
                         const CUtensorMap* xmap_tail, const CUtensorMap* xmap_half,
                         const ScanParams& p, const Smem& sm) {
  const uint64_t pol_q = policy_evict_last();
  const uint64_t pol_x = p.dataset_evict_first ? policy_evict_first() : policy_evict_normal();
  const uint32_t crank = kPair ? cluster_ctarank() : 0u;
  const int first = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int step = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int sbytes = stage_bytes(kPair);
  // With pairs, a tile of w rows is split in two halves of w / 2 rows
  // (multiples of 32: the granule is 64 rows), this CTA loading half crank;
  // the loads count on the first CTA's full barrier.
  auto half_rows = [&](int w) { return kPair ? w / 2 : w; };
  auto bar_of = [&](uint32_t slot) -> uint32_t {
    return kPair ? mapa_shared(&sm.full[slot], 0) : smem_addr(&sm.full[slot]);
  };
  auto expect = [&](uint32_t slot, uint32_t bytes) {
    if constexpr (kPair) mbar_arrive_expect_tx_cluster(bar_of(slot), bytes);
    else mbar_arrive_expect_tx(&sm.full[slot], bytes);
  };
  auto load = [&](void* dst, const CUtensorMap* map, uint32_t slot, int32_t x, int32_t y,
                  uint64_t pol) {
    if constexpr (kPair) tma_load_2d_pair(dst, map, bar_of(slot), x, y, pol);
    else tma_load_2d(dst, map, &sm.full[slot], x, y, pol);
  };
  auto load_rows = [&](uint8_t* dst, uint32_t slot, int kc, int64_t rs, int w) {
    const int h = half_rows(w);
    const int64_t r0 = rs + (kPair ? static_cast<int64_t>(crank) * h : 0);
    // rows past n_rows (less than a granule) are TMA's zero fill
    if (!in_bounds(r0 >= 0 && r0 < p.n_rows + p.gran_rows && w > 0 && w <= kTileRows &&
                       h % kTailBox == 0 && kc * kKChunk < p.ld,
                   p.err))
      return;
    if (!kPair && w == kTileRows) {
      load(dst, xmap, slot, kc * kKChunk, static_cast<int32_t>(r0), pol_x);
    } else if (kPair && w == kTileRows) {
      load(dst, xmap_half, slot, kc * kKChunk, static_cast<int32_t>(r0), pol_x);
    } else {
      for (int j = 0; j < h; j += kTailBox)
        load(dst + j * (kKChunk * 2), xmap_tail, slot, kc * kKChunk,
             static_cast<int32_t>(r0 + j), pol_x);
    }
  };
  // phase 1: dataset slabs of the first p.stages loads (every stage is free)
  uint32_t pre = 0;
  for (int u = first; u < p.units && pre < static_cast<uint32_t>(p.stages); u += step) {
    const Unit un = unit_of(p, u);
    for (int64_t rs = un.r0; rs < un.r_end && pre < static_cast<uint32_t>(p.stages);
         rs += kTileRows) {
      const int w = tile_width(rs, un.r_end);
      for (int kc = 0; kc < p.k_chunks && pre < static_cast<uint32_t>(p.stages); ++kc) {
        uint8_t* st = sm.stages + static_cast<size_t>(pre) * sbytes;
        expect(pre, kStageA + half_rows(w) * (kKChunk * 2));
        load_rows(st + kStageA, pre, kc, rs, w);
        ++pre;
      }
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // phase 2: every load in order; the first `pre` only need their query slab
  uint32_t it = 0;
  bool failed = false;
  for (int u = first; u < p.units && !failed; u += step) {
    const Unit un = unit_of(p, u);
    // the unit's 128-row query slab (a spread block's slab is its own)
    const int32_t qy = p.spread ? un.m * kQueryRows
                                : un.m * p.unit_queries + static_cast<int32_t>(crank) * kQueryRows;
    if (!in_bounds(qy >= 0 && qy + kQueryRows <= p.q_rows, p.err)) {
      failed = true;
      break;
    }
    for (int64_t rs = un.r0; rs < un.r_end && !failed; rs += kTileRows) {
      const int w = tile_width(rs, un.r_end);
      for (int kc = 0; kc < p.k_chunks; ++kc) {
        const uint32_t slot = it % p.stages;
        uint8_t* st = sm.stages + static_cast<size_t>(slot) * sbytes;
        if (it < pre) {
          load(st, qmap, slot, kc * kKChunk, qy, pol_q);
          ++it;
          continue;
        }
        const uint32_t ph = (it / p.stages) & 1u;
        if (!mbar_wait(&sm.empty[slot], ph ^ 1u, p.err, kErrTimeoutEmpty)) {
          failed = true;
          break;
        }
        expect(slot, kStageA + half_rows(w) * (kKChunk * 2));
        load(st, qmap, slot, kc * kKChunk, qy, pol_q);
        load_rows(st + kStageA, slot, kc, rs, w);
        ++it;
      }
    }
  }
  if (failed && kPair) {
    // copies this CTA issued may still be landing in its shared memory:
    // give them time before the CTA can retire (bounded, 2 ms)
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 2000000ull) {
    }
  }
  if (failed && !kPair) {
    // Let the copies already issued land before the CTA can retire.  (With
    // pairs the copies complete on the first CTA's barrier; both CTAs wait
    // for each other at the end of the kernel, after bounded waits.)
    const uint32_t outstanding = it < static_cast<uint32_t>(p.stages) ? it : p.stages;
    for (uint32_t j = it - outstanding; j < it; ++j)
      drain_wait(&sm.full[j % p.stages], (j / p.stages) & 1u);
  }
}

template <bool kPair>
__device__ void mma_issuer(const ScanParams& p, const Smem& sm, uint32_t tmem_base) {
  // with pairs only the first CTA issues; the MMAs read both CTAs' slabs
  const int first = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int step = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int sbytes = stage_bytes(kPair);
  uint32_t it = 0, tc = 0;
  bool failed = false;
  for (int u = first; u < p.units && !failed; u += step) {
    const Unit un = unit_of(p, u);
    for (int64_t rs = un.r0; rs < un.r_end && !failed; rs += kTileRows) {
      // N = the tile's width: a narrower last tile multiplies only its rows
      const uint32_t idesc = idesc_f16_f32(kPair ? 2 * kQueryRows : kQueryRows,
                                           static_cast<uint32_t>(tile_width(rs, un.r_end)));
      const uint32_t b = tc & 1u;
      if (!mbar_wait(&sm.acc_empty[b], ((tc >> 1) & 1u) ^ 1u, p.err, kErrTimeoutAccEmpty)) {
        failed = true;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + b * kAccCols;
      for (int kc = 0; kc < p.k_chunks; ++kc) {
        const uint32_t slot = it % p.stages;
        if (!mbar_wait(&sm.full[slot], (it / p.stages) & 1u, p.err, kErrTimeoutFull)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_addr(sm.stages + static_cast<size_t>(slot) * sbytes);
        const uint32_t b0 = a0 + kStageA;
#pragma unroll
        for (int kk = 0; kk < kKChunk / 16; ++kk) {
          // advancing 16 fp16 (32 bytes) inside the 128-byte swizzle atom
          if constexpr (kPair) {
            umma_f16_ss_pair(d_tmem, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32),
                             idesc, (kc | kk) != 0 ? 1u : 0u);
          } else {
            umma_f16_ss(d_tmem, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32),
                        idesc, (kc | kk) != 0 ? 1u : 0u);
          }
        }
        if constexpr (kPair) umma_commit_pair_both(&sm.empty[slot]);
        else umma_commit(&sm.empty[slot]);
        ++it;
      }
      if (failed) break;
      if constexpr (kPair) umma_commit_pair_both(&sm.acc_full[b]);
      else umma_commit(&sm.acc_full[b]);
      ++tc;
    }
  }
  // All MMAs of this thread must be complete before TMEM is released.
  if constexpr (kPair) umma_commit_pair_own(sm.drain);
  else umma_commit(sm.drain);
  drain_wait(sm.drain, 0);
}

// The distance the scan orders by, from the fp32 dot product, per metric.
// Used by every pass over a tile so all passes see identical values.
//   L2:            |q|^2 + |x|^2 - 2 q.x, clamped at 0 (squared L2); xn is
//                  the row norm, +inf past the last row;
//   inner product: xn - q.x with xn = 0 for a row and +inf past the last
//                  row, so the ascending order is descending similarity
//                  (the final merge negates it back) and 0 - q.x is never -0.
// Both map -0 to +0 (key order); NaN stays NaN.
template <int kMetric>
__device__ __forceinline__ float dist_from_dot(uint32_t acc_bits, float qn, float xn) {
  if constexpr (kMetric == KNN_METRIC_INNER_PRODUCT) {
    return xn - __uint_as_float(acc_bits);
  } else {
    const float d = fmaf(-2.0f, __uint_as_float(acc_bits), qn + xn);
    return d <= 0.0f ? 0.0f : d;
  }
}

// Order-preserving 32-bit image of a distance (any sign) and its inverse;
// used for the per-query bound the CTAs share through atomicMin.
__device__ __forceinline__ uint32_t dist_order_bits(float d) {
  const uint32_t u = __float_as_uint(d);
  return u ^ ((u >> 31) ? 0xFFFFFFFFu : 0x80000000u);
}
__device__ __forceinline__ float dist_from_order_bits(uint32_t b) {
  return __uint_as_float(b ^ ((b >> 31) ? 0x80000000u : 0xFFFFFFFFu));
}

// Smallest float above a finite t (t is never -0 here).
__device__ __forceinline__ float next_up(float t) {
  const int b = __float_as_int(t);
  if (t == 0.0f) return __int_as_float(1);
  return __int_as_float(t > 0.0f ? b + 1 : b - 1);
}

// Ascending sort of 32 registers: bitonic network with every index a
// template constant, so the array stays in registers.
template <int Size, int Stride>
__device__ __forceinline__ void bitonic_pass(float (&g)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int j = i ^ Stride;
    if (j > i) {
      const float a = g[i], b = g[j];
      const bool up = (i & Size) == 0;
      g[i] = up ? fminf(a, b) : fmaxf(a, b);
      g[j] = up ? fmaxf(a, b) : fminf(a, b);
    }
  }
  if constexpr (Stride > 1) bitonic_pass<Size, Stride / 2>(g);
}

template <int Size>
__device__ __forceinline__ void bitonic_sort(float (&g)[32]) {
  bitonic_pass<Size, Size / 2>(g);
  if constexpr (Size < 32) bitonic_sort<Size * 2>(g);
}

__device__ __forceinline__ void sort32(float (&g)[32]) { bitonic_sort<2>(g); }

// k up to which each query row keeps its running top-k in registers (a
// sorted array of kRegK keys) instead of a shared-memory heap.
constexpr int kRegK = 16;

// Heap size from which a query block of 32 rows sorts its unit lists with
// all 4 epilogue warps (warp-wide bitonic sorts) instead of lane by lane.
constexpr int kCoopMinHeap = 64;

// Per query row (one epilogue lane): the filter threshold, the worst kept
// key (root), the number of buffered survivors and the top-k itself.
// kReg: top[] holds kRegK keys in ascending order, the first kRegK - k of
// them the sentinel 0 (below every real key, so they never leave the front)
// and the rest the row's k best keys, padded with the empty key; inserting a
// key drops the largest, so top[kRegK - 1] is the k-th best.  Otherwise the
// top-k lives in the shared-memory max-heap of the row.
template <bool kReg>
struct RowState {
  float thr;     // candidates with d < thr are kept
  uint64_t root; // worst kept key once the row holds k, else the empty key
  int cnt;       // survivors waiting in the row's buffer
  int size;      // entries in the heap (<= k; heap path only)
  uint32_t pub;  // bound this row last published (order bits)
  uint64_t top[kReg ? kRegK : 1];
};

// Inserts key x into the ascending register array a, dropping its largest
// key (x >= a[kRegK - 1] leaves it unchanged).  Branch-free: c[i] = x < a[i]
// for the original keys, then a[i] takes a[i - 1] (shifted up), x, or keeps
// its key.
__device__ __forceinline__ void topk_insert(uint64_t (&a)[kRegK], uint64_t x) {
  bool c[kRegK];
#pragma unroll
  for (int i = 0; i < kRegK; ++i) c[i] = x < a[i];
#pragma unroll
  for (int i = kRegK - 1; i > 0; --i) a[i] = c[i - 1] ? a[i - 1] : (c[i] ? x : a[i]);
  a[0] = c[0] ? x : a[0];
}

// Moves every lane's buffered survivors into its top-k.  Warp-uniform: all
// lanes run the same number of iterations (the warp's largest buffer), so
// the updates of the 32 query rows proceed in lock-step.  Heap path: the
// heap grows by sift-up until it holds k entries, then replaces its root.
// Compact heaps (kC) hold keys relative to the unit's first row `base`:
// a buffered key's index is rebased before it is compared or stored.
template <bool kC>
__device__ __forceinline__ HeapStore<kC> heap_of(const Smem& sm) {
  if constexpr (kC) return HeapStore<true>{sm.heap_hi, sm.heap_lo};
  else return HeapStore<false>{sm.heap};
}

template <int kMetric, bool kReg, bool kC>
__device__ __forceinline__ void flush_buffer(RowState<kReg>& st, const Smem& sm, int k,
                                             int stride, int row, uint32_t base, int* err) {
  const int maxc = __reduce_max_sync(0xffffffffu, st.cnt);
  if (!in_bounds(maxc <= kRowBuf, err)) return;
  if constexpr (kReg) {
    for (int b = 0; b < maxc; ++b) {
      if (b < st.cnt) {
        const uint64_t key = sm.buf[b * stride + row];
        if (key < st.top[kRegK - 1]) topk_insert(st.top, key);
      }
    }
    st.root = st.top[kRegK - 1];
  } else {
    const HeapStore<kC> heap = heap_of<kC>(sm);
    for (int b = 0; b < maxc; ++b) {
      if (b < st.cnt) {
        uint64_t key = sm.buf[b * stride + row];
        if constexpr (kC)
          key = (key & 0xFFFFFFFF00000000ull) | (static_cast<uint32_t>(key) - base);
        if (st.size < k) {
          heap_sift_up(heap, stride, row, st.size, key, k, err);
          if (++st.size == k) st.root = heap.get(row);
        } else if (key < st.root) {
          heap_sift_down(heap, k, stride, row, 0, key, k, err);
          st.root = heap.get(row);
        }
      }
    }
  }
  st.cnt = 0;
  st.thr = fminf(st.thr, key_dist<kMetric>(st.root));
}

// The 4 epilogue warps meet at sm.epi_bar (lane 0 of each arrives; every
// lane waits, bounded).  `use` counts this warp's meetings (the barrier's
// phase).  Returns false when the wait gave up (a warp that failed earlier
// never arrives; its error word ends the wait).
__device__ __forceinline__ bool epilogue_meet(const Smem& sm, uint32_t& use, int lane, int* err) {
  __syncwarp();
  if (lane == 0) mbar_arrive(sm.epi_bar);
  const bool ok = mbar_wait(sm.epi_bar, use & 1u, err, kErrTimeoutEpilogue);
  ++use;
  return !__any_sync(0xffffffffu, !ok);
}

// Ascending bitonic sort of 32 * E keys held by one warp: element e lives in
// register e / 32 of lane e % 32.  Strides of 32 and more compare registers
// of the same lane, smaller ones exchange with lane ^ stride.
template <int E>
__device__ __forceinline__ void warp_sort_keys(uint64_t (&v)[E], int lane) {
  constexpr int N = 32 * E;
#pragma unroll
  for (int size = 2; size <= N; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride >= 32) {
        const int rs = stride / 32;
#pragma unroll
        for (int j = 0; j < E; ++j) {
          if ((j & rs) == 0) {
            const bool up = ((j * 32 + lane) & size) == 0;
            const uint64_t a = v[j], b = v[j | rs];
            const bool swap = up ? (b < a) : (a < b);
            v[j] = swap ? b : a;
            v[j | rs] = swap ? a : b;
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < E; ++j) {
          const uint64_t o = __shfl_xor_sync(0xffffffffu, v[j], stride);
          const bool up = ((j * 32 + lane) & size) == 0;
          const bool lower = (lane & stride) == 0;
          // the lower element of an ascending pair keeps the minimum
          v[j] = (lower == up) ? (o < v[j] ? o : v[j]) : (o > v[j] ? o : v[j]);
        }
      }
    }
  }
}

// One query row's unit list from its heap: the warp loads the n heap
// entries (padding: the empty key, above every real key), sorts them and
// writes the first k as (distance, index), the index rebased for compact
// heaps.
template <int kMetric, bool kC, int E>
__device__ __forceinline__ void write_sorted_row(const HeapStore<kC>& heap, int stride, int row,
                                                 int n, int k, uint32_t base, float* od,
                                                 uint32_t* oi, int lane) {
  uint64_t v[E];
#pragma unroll
  for (int j = 0; j < E; ++j) {
    const int e = j * 32 + lane;
    v[j] = e < n ? heap.get(e * stride + row) : empty_key<kMetric>();
  }
  warp_sort_keys<E>(v, lane);
#pragma unroll
  for (int j = 0; j < E; ++j) {
    const int e = j * 32 + lane;
    if (e < k) {
      od[e] = key_dist<kMetric>(v[j]);
      oi[e] = e < n ? (kC ? base + static_cast<uint32_t>(v[j]) : static_cast<uint32_t>(v[j]))
                    : kNoIndex;
    }
  }
}

// The unit lists of a 32-row query block, row r sorted and written by
// epilogue warp r % 4 (write_sorted_row).  Kept out of line so that its
// registers do not weigh on the epilogue's tile loop.
// Heap size of slot r (r < 32) of a 32-query block, as its owner left it in
// its own norm-staging slice (warp w's slice is w - 2; the warp of TMEM lane
// quadrant c is (c + 2) & 3 slices in): slot r is lane r of quadrant 0, or
// in a spread block lane r / 4 of quadrant r % 4.
__device__ __forceinline__ int heap_size_of(const float* norm_stage, int r, bool spread) {
  const int quad = spread ? r % 4 : 0;
  const int lane = spread ? r / 4 : r;
  return reinterpret_cast<const int*>(norm_stage + ((quad + 2) & 3) * kAccCols)[lane];
}

template <int kMetric, bool kC>
__device__ __noinline__ void sort_rows_cooperative(const ScanParams& p, const HeapStore<kC> heap,
                                                   const float* norm_stage, int m, int s,
                                                   uint32_t base, int warp, int lane) {
  const int k = p.k;
  const int stride = p.heap_rows;
  for (int r = warp - 2; r < p.query_block; r += 4) {  // warp-uniform
    const int64_t qr = static_cast<int64_t>(m) * p.unit_queries + r;
    if (qr >= p.n_queries || !in_bounds(s < p.splits, p.err)) continue;
    const int n = heap_size_of(norm_stage, r, p.spread != 0);
    if (!in_bounds(n >= 0 && n <= k && r < stride, p.err)) continue;
    float* od = p.part_d + (static_cast<size_t>(qr) * p.splits + s) * k;
    uint32_t* oi = p.part_i + (static_cast<size_t>(qr) * p.splits + s) * k;
    if (k <= 32) write_sorted_row<kMetric, kC, 1>(heap, stride, r, n, k, base, od, oi, lane);
    else if (k <= 64) write_sorted_row<kMetric, kC, 2>(heap, stride, r, n, k, base, od, oi, lane);
    else if (k <= 128) write_sorted_row<kMetric, kC, 4>(heap, stride, r, n, k, base, od, oi, lane);
    else write_sorted_row<kMetric, kC, 8>(heap, stride, r, n, k, base, od, oi, lane);
  }
}

// Epilogue warp.  Lane `row` owns query row `row` of the unit's query block.
//
// Candidate handling per 32-column chunk of an accumulator tile:
//   * d for the 32 columns in registers; survivors are d < thr (one compare);
//   * survivors are appended to the row's shared-memory buffer (kRowBuf);
//   * when any lane's buffer could overflow, the whole warp flushes its
//     buffers into the heaps (flush_buffer) and tightens thr.
// Seeding: on the first tile of a unit (k <= 32) a first pass over the tile
// takes the minimum of each column position j over the 8 chunks (32 group
// minima, each the distance of a distinct row); the k-th smallest of them,
// t, has at least k rows of this unit at d <= t, so the unit's k-th best is
// <= t and filtering with d <= t drops no result.  This keeps the first
// tile from pushing all 256 columns through the heap.
// Pilot pass (p.pilot): only that first-tile pass runs, and each unit
// writes its 32 sorted group minima to p.pilot_out for
// pilot_threshold_kernel.  A main pass started with p.thr_init filters
// every tile from the first one with that per-query threshold.
// Shared bound (p.bound): once a row's heap holds k entries, its k-th
// distance R bounds the query's k-th distance over the whole shard (this
// unit alone has k rows at d <= R), so the CTA publishes R with atomicMin
// and every CTA filters with the smallest published R from its next tile
// on.  The seed threshold t of a unit's first tile bounds it the same way
// (k distinct rows of the unit lie at d <= t) and is published as soon as it
// is known, a tile before any top-k is full.  A row of the final top-k lies
// at d <= R and still passes in its own unit, whose best k then include it;
// units may end with fewer than k entries (padding), which the merge ignores.
// Survivors of a 16-column group are appended one per lane per round (the
// lowest remaining column first), so a group costs as many rounds as its
// busiest lane has survivors, usually one.
template <int kMetric, bool kReg, bool kC, bool kPair>
__device__ void epilogue(const ScanParams& p, const Smem& sm, uint32_t tmem_base, int warp,
                         int lane) {
  const uint32_t crank = kPair ? cluster_ctarank() : 0u;
  const int first = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int step = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int quad = warp & 3;              // TMEM lane quadrant this warp may access
  const int row = quad * 32 + lane;       // TMEM lane = row of the query slab
  // the row's query within the unit's block, which also indexes its heap and
  // survivor buffer: the row itself, or in a spread block query 4 * lane +
  // quad for lanes 0-7 (other lanes hold none: slot >= query_block)
  const int slot = p.spread ? (lane < 8 ? 4 * lane + quad : p.query_block + lane) : row;
  const bool warp_active = p.spread || quad * 32 < p.query_block;
  const int stride = p.heap_rows;
  const int k = p.k;
  const float kInf = __int_as_float(0x7f800000);
  uint32_t tc = 0;
  uint32_t meets = 0;  // epilogue_meet calls so far (the barrier's phase)
  bool failed = false;
  for (int u = first; u < p.units && !failed; u += step) {
    const Unit un = unit_of(p, u);
    const uint32_t base = static_cast<uint32_t>(un.r0);  // compact heaps' offsets start here
    // rows at or past row_lim are masked: the dataset's end, or (in a
    // narrower last tile) accumulator columns the tile's MMAs did not write
    const int64_t row_lim = un.r_end < p.n_rows ? un.r_end : p.n_rows;
    const int64_t q = static_cast<int64_t>(un.m) * p.unit_queries +
                      static_cast<int64_t>(crank) * kQueryRows + slot;
    const bool valid_q = warp_active && slot < p.query_block && q < p.n_queries;
    const float qn = valid_q ? p.query_norms[q] : 0.0f;
    RowState<kReg> st;
    st.thr = valid_q ? (p.thr_init ? p.thr_init[q] : kInf) : __int_as_float(0xff800000);
    st.root = empty_key<kMetric>();
    st.cnt = 0;
    st.size = 0;
    st.pub = 0xFFFFFFFFu;
    if constexpr (kReg) {
#pragma unroll
      for (int i = 0; i < kRegK; ++i) st.top[i] = i < kRegK - k ? 0ull : empty_key<kMetric>();
    }
    // Row norms are prefetched one tile ahead into registers, then staged in
    // this warp's slice of shared memory so the chunk loop reads them with
    // a shared-memory load instead of waiting on DRAM once per chunk (for
    // the inner product: 0 for a row, +inf past the last row).
    float* const ns = sm.norm_stage + (warp - 2) * kAccCols;
    float nx[kAccCols / 32];
    auto prefetch_norms = [&](int64_t rs) {
#pragma unroll
      for (int c = 0; c < kAccCols / 32; ++c) {
        const int64_t col = rs + c * 32 + lane;
        if constexpr (kMetric == KNN_METRIC_INNER_PRODUCT) {
          nx[c] = col < row_lim ? 0.0f : kInf;
        } else {
          nx[c] = col < row_lim && in_bounds(col < p.n_rows, p.err) ? __ldg(p.row_norms + col)
                                                                     : kInf;
        }
      }
    };
    if (warp_active) prefetch_norms(un.r0);
    for (int64_t rs = un.r0; rs < un.r_end; rs += kTileRows) {
      // 32-column chunks of this tile's accumulator, rounded up to a pair
      // (the TMEM loads go two chunks at a time; a chunk past the tile's
      // width holds stale columns, masked by their +inf norms)
      const int nch = ((tile_width(rs, un.r_end) / 32) + 1) & ~1;
      const uint32_t b = tc & 1u;
      // every lane waits; the warp leaves together if any lane gave up, so
      // the .sync.aligned TMEM loads below always see a converged warp
      const bool ok = mbar_wait(&sm.acc_full[b], (tc >> 1) & 1u, p.err, kErrTimeoutAccFull);
      if (__any_sync(0xffffffffu, !ok)) {
        failed = true;
        break;
      }
      tc_fence_after();
      uint32_t shared_b = 0xFFFFFFFFu;  // read now, applied before the chunk loop
      if (p.bound && valid_q && in_bounds(q < p.n_queries, p.err))
        shared_b = *reinterpret_cast<volatile const uint32_t*>(p.bound + q);
      if (warp_active) {
#pragma unroll
        for (int c = 0; c < kAccCols / 32; ++c) ns[c * 32 + lane] = nx[c];
        __syncwarp();
        if (rs + kTileRows < un.r_end) prefetch_norms(rs + kTileRows);
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + b * kAccCols;
        if (rs == un.r0 && (k <= 32 || p.pilot)) {
          float g[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) g[j] = kInf;
#pragma unroll 1
          for (int c = 0; c < nch; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tbase + c * 32, r);
            tmem_ld_wait_into(r);
            const float4* n4 = reinterpret_cast<const float4*>(ns + c * 32);
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 v = n4[j4];  // same address in every lane: broadcast
              g[4 * j4 + 0] = fminf(g[4 * j4 + 0], dist_from_dot<kMetric>(r[4 * j4 + 0], qn, v.x));
              g[4 * j4 + 1] = fminf(g[4 * j4 + 1], dist_from_dot<kMetric>(r[4 * j4 + 1], qn, v.y));
              g[4 * j4 + 2] = fminf(g[4 * j4 + 2], dist_from_dot<kMetric>(r[4 * j4 + 2], qn, v.z));
              g[4 * j4 + 3] = fminf(g[4 * j4 + 3], dist_from_dot<kMetric>(r[4 * j4 + 3], qn, v.w));
            }
          }
          sort32(g);
          if (p.pilot) {
            if (valid_q && in_bounds(q < p.n_queries && u / p.query_tiles < p.splits, p.err)) {
              float4* o = reinterpret_cast<float4*>(
                  p.pilot_out + (q * p.splits + u / p.query_tiles) * 32);
#pragma unroll
              for (int j4 = 0; j4 < 8; ++j4)
                o[j4] = make_float4(g[4 * j4], g[4 * j4 + 1], g[4 * j4 + 2], g[4 * j4 + 3]);
            }
          } else {
            // g is ascending, so g[k - 1] = max of g[0..k-1] (written without a
            // run-time register index; g[0] is the neutral filler for j >= k
            // because every g[j] >= g[0], whatever the sign of the distances)
            float tk = g[0];
#pragma unroll
            for (int j = 1; j < 32; ++j) tk = fmaxf(tk, j < k ? g[j] : g[0]);
            // keep d <= tk: the next float up
            if (valid_q && tk < kInf) {
              st.thr = fminf(st.thr, next_up(tk));
              // this unit holds k distinct rows at d <= tk, so tk bounds the
              // query's k-th distance over the shard: share it now
              const uint32_t bits = dist_order_bits(tk);
              if (p.bound && bits < st.pub && in_bounds(q < p.n_queries, p.err)) {
                // publish ours and take back the smallest bound published so
                // far: the units seed at about the same time, so the minimum
                // over those that already have is far tighter than our own
                const uint32_t seen = atomicMin(p.bound + q, bits);
                st.pub = bits;
                if (seen < bits) {
                  const float bnd = dist_from_order_bits(seen);
                  if (bnd < kInf) st.thr = fminf(st.thr, next_up(bnd));
                }
              }
            }
          }
        }
        // One 32-column chunk: distances, threshold filter, survivor buffer.
        auto process_chunk = [&](const uint32_t (&r)[32], int c) {
          float dv[32];
          const float4* n4 = reinterpret_cast<const float4*>(ns + c * 32);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 v = n4[j4];  // row norms of columns 4*j4.., broadcast
            dv[4 * j4 + 0] = dist_from_dot<kMetric>(r[4 * j4 + 0], qn, v.x);
            dv[4 * j4 + 1] = dist_from_dot<kMetric>(r[4 * j4 + 1], qn, v.y);
            dv[4 * j4 + 2] = dist_from_dot<kMetric>(r[4 * j4 + 2], qn, v.z);
            dv[4 * j4 + 3] = dist_from_dot<kMetric>(r[4 * j4 + 3], qn, v.w);
          }
          const uint32_t col0 = static_cast<uint32_t>(rs + c * 32);
#pragma unroll
          for (int h = 0; h < 32; h += kRowBuf) {
            uint32_t mask = 0;
#pragma unroll
            for (int j = 0; j < kRowBuf; ++j) mask |= (dv[h + j] < st.thr ? 1u : 0u) << j;
            if (__any_sync(0xffffffffu, mask != 0)) {
              if (__any_sync(0xffffffffu, st.cnt + __popc(mask) > kRowBuf)) {
                flush_buffer<kMetric, kReg, kC>(st, sm, k, stride, slot, base, p.err);
                mask = 0;
#pragma unroll
                for (int j = 0; j < kRowBuf; ++j) mask |= (dv[h + j] < st.thr ? 1u : 0u) << j;
              }
              // one survivor per lane per round, lowest column first; the
              // value is picked by an unrolled select chain (no local memory)
              uint32_t m = mask;
              while (__any_sync(0xffffffffu, m != 0)) {
                if (m != 0) {
                  const int j = __ffs(m) - 1;
                  float v = dv[h];
#pragma unroll
                  for (int jj = 1; jj < kRowBuf; ++jj) v = j == jj ? dv[h + jj] : v;
                  if (in_bounds(st.cnt < kRowBuf && slot < stride, p.err))
                    sm.buf[st.cnt * stride + slot] = make_key<kMetric>(v, col0 + h + j);
                  ++st.cnt;
                  m &= m - 1u;
                }
              }
            }
          }
        };
        // TMEM loads double-buffered: chunk c + 1 is in flight while chunk c
        // is processed.
        static_assert((kAccCols / 32) % 2 == 0, "chunk pairs");
        if (shared_b != 0xFFFFFFFFu) {
          const float bnd = dist_from_order_bits(shared_b);
          if (bnd < kInf) st.thr = fminf(st.thr, next_up(bnd));
        }
        if (!p.pilot) {  // uniform over the grid: the warp stays converged
          uint32_t ra[32], rb[32];
          tmem_ld_32x32b_x32(tbase, ra);
          tmem_ld_wait_into(ra);
#pragma unroll 1
          for (int c = 0; c < nch; c += 2) {
            tmem_ld_32x32b_x32(tbase + (c + 1) * 32, rb);
            process_chunk(ra, c);
            tmem_ld_wait_into(rb);
            if (c + 2 < nch) tmem_ld_32x32b_x32(tbase + (c + 2) * 32, ra);
            process_chunk(rb, c + 1);
            if (c + 2 < nch) tmem_ld_wait_into(ra);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        // with pairs the first CTA's MMAs wait for both CTAs' epilogues
        if constexpr (kPair) mbar_arrive_cluster(mapa_shared(&sm.acc_empty[b], 0));
        else mbar_arrive(&sm.acc_empty[b]);
      }
      ++tc;
      // survivors enter the heap at every tile end so thr tightens early (the
      // accumulator is already released; this overlaps the next tile's MMAs)
      if (warp_active && __any_sync(0xffffffffu, st.cnt > 0)) {
        flush_buffer<kMetric, kReg, kC>(st, sm, k, stride, slot, base, p.err);
        if (p.bound && valid_q && st.root != empty_key<kMetric>()) {
          const uint32_t bits = dist_order_bits(key_dist<kMetric>(st.root));
          if (bits < st.pub && in_bounds(q < p.n_queries, p.err)) {
            atomicMin(p.bound + q, bits);
            st.pub = bits;
          }
        }
      }
    }
    if (failed) break;
    if (p.pilot) continue;
    if (warp_active) flush_buffer<kMetric, kReg, kC>(st, sm, k, stride, slot, base, p.err);
    if (!kReg && p.query_block == kGranRows) {  // grid-uniform
      // Query blocks of 32 rows: one warp owns every row (up to 8 per warp
      // in a spread block) and would sort each row's heap alone, lane by
      // lane (a 256-entry heap sort costs tens of microseconds at the end
      // of the unit).  Each owner leaves
      // its row's heap size in its own norm-staging slice (free until its
      // next tile); once the warps have met, all of them read the sizes,
      // and if some heap holds kCoopMinHeap entries or more, row r is
      // sorted by warp r % 4 with a warp-wide bitonic sort (a heap is in
      // shared memory, so any warp can read it).  The warps meet again
      // afterwards, so no owner refills a heap that another warp still
      // reads.  Smaller heaps keep the per-lane sort below.
      if (warp_active) reinterpret_cast<int*>(ns)[lane] = valid_q ? st.size : 0;
      if (!epilogue_meet(sm, meets, lane, p.err)) {
        failed = true;
        break;
      }
      const bool coop =
          __reduce_max_sync(0xffffffffu, heap_size_of(sm.norm_stage, lane, p.spread != 0)) >=
          kCoopMinHeap;
      if (coop)
        sort_rows_cooperative<kMetric, kC>(p, heap_of<kC>(sm), sm.norm_stage, un.m, u / p.query_tiles,
                                           base, warp, lane);
      if (!epilogue_meet(sm, meets, lane, p.err)) {
        failed = true;
        break;
      }
      if (coop) continue;
    }
    const bool out_ok = !valid_q || in_bounds(q < p.n_queries && u / p.query_tiles < p.splits,
                                              p.err);
    if (kReg && valid_q && out_ok) {
      // the row's k best are top[kRegK - k ..], already ascending
      const int s = u / p.query_tiles;
      float* od = p.part_d + (static_cast<size_t>(q) * p.splits + s) * k;
      uint32_t* oi = p.part_i + (static_cast<size_t>(q) * p.splits + s) * k;
#pragma unroll
      for (int i = 0; i < (kReg ? kRegK : 0); ++i) {
        if (i >= kRegK - k) {
          od[i - (kRegK - k)] = key_dist<kMetric>(st.top[i]);
          oi[i - (kRegK - k)] = static_cast<uint32_t>(st.top[i]);
        }
      }
    } else if (valid_q && out_ok) {
      // heap sort of the st.size entries -> ascending (distance, index);
      // the rest of the list is padding
      const HeapStore<kC> heap = heap_of<kC>(sm);
      const int n = st.size;
      for (int end = n - 1; end > 0; --end) {
        const uint64_t top = heap.get(slot);
        const uint64_t last = heap.get(end * stride + slot);
        heap.set(end * stride + slot, top);
        heap_sift_down(heap, end, stride, slot, 0, last, k, p.err);
      }
      const int s = u / p.query_tiles;
      float* od = p.part_d + (static_cast<size_t>(q) * p.splits + s) * k;
      uint32_t* oi = p.part_i + (static_cast<size_t>(q) * p.splits + s) * k;
      for (int r = 0; r < k; ++r) {
        const uint64_t key = r < n ? heap.get(r * stride + slot) : empty_key<kMetric>();
        od[r] = key_dist<kMetric>(key);
        oi[r] = r < n && kC ? base + static_cast<uint32_t>(key) : static_cast<uint32_t>(key);
      }
    }
  }
}

template <int kMetric, bool kReg, bool kC, bool kPair>
__global__ void __launch_bounds__(kScanThreads, 1)
    knn_scan_kernel(const __grid_constant__ CUtensorMap qmap,
                    const __grid_constant__ CUtensorMap xmap,
                    const __grid_constant__ CUtensorMap xmap_tail,
                    const __grid_constant__ CUtensorMap xmap_half, const ScanParams p) {
  extern __shared__ uint8_t smem_raw[];
  const Smem sm = carve(smem_raw, p);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    // with pairs, the first CTA's full barriers take one arrival from each
    // CTA's producer and its acc_empty barriers one from each of the eight
    // epilogue warps (the second CTA's barriers of those kinds go unused)
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&sm.full[s], kPair ? 2 : 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], kPair ? 8 : 4);
    }
    mbar_init(sm.drain, 1);
    mbar_init(sm.epi_bar, 4);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&qmap);
    tma_prefetch_map(&xmap);
    tma_prefetch_map(&xmap_tail);
    if constexpr (kPair) tma_prefetch_map(&xmap_half);
  }
  if (warp == 1) {
    if constexpr (kPair) {
      tmem_alloc_pair(sm.tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(sm.tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  // the peer's barriers are initialised before any remote arrival
  if constexpr (kPair) cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *sm.tmem_slot;
  // Launched as a programmatic dependent: the set-up above overlaps the tail
  // of the kernel before (the query conversion).  Every role but the
  // producer waits for its results here (the producer waits itself, after
  // requesting its first dataset slabs); the merge kernel after this one
  // may be scheduled early.
  if (warp != 0) asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    if (lane == 0) producer<kPair>(&qmap, &xmap, &xmap_tail, &xmap_half, p, sm);
  } else if (warp == 1) {
    if (lane == 0 && (!kPair || cluster_ctarank() == 0)) mma_issuer<kPair>(p, sm, tmem_base);
  } else {
    epilogue<kMetric, kReg, kC, kPair>(p, sm, tmem_base, warp, lane);
  }

  tc_fence_before();
  __syncthreads();
  // neither CTA of a pair leaves while the other may still signal its
  // barriers or the MMAs may still read its shared memory
  if constexpr (kPair) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (kPair) tmem_dealloc_pair(tmem_base, kTmemCols);
    else tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Self-test of the bounded wait: thread 0 waits for phase 0 of a barrier
// that nothing arrives on; the wait must give up after limit_ns and record
// kErrTimeoutFull.  No memory access depends on the barrier.
__global__ void bounded_wait_selftest_kernel(int* err, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, err, kErrTimeoutFull, limit_ns);
}

// Per-query starting threshold from the pilot pass.  Each of the S units
// left its 32 group minima sorted, every value the distance of a distinct
// row.  With j = ceil(k / S) and r = ceil(k / j), tau = the r-th smallest of
// the units' j-th values: r units each hold j values <= tau, so at least k
// distinct rows lie at distance <= tau, and the k-th smallest distance of
// the whole shard is <= tau.  Filtering with d <= tau (thr = the float
// above tau) therefore keeps every row of the result.  When j > 32 or tau is
// not finite the threshold is +inf (no filter).  One block per query.
__global__ void __launch_bounds__(256)
    pilot_threshold_kernel(const float* __restrict__ pilot, int splits, int k,
                           float* __restrict__ thr) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t q = blockIdx.x;
  const float kInf = __int_as_float(0x7f800000);
  const int j = (k + splits - 1) / splits;
  if (j > 32) {
    if (threadIdx.x == 0) thr[q] = kInf;
    return;
  }
  const int r = (k + j - 1) / j;  // <= splits
  extern __shared__ float sv[];   // [splits]
  for (int s = threadIdx.x; s < splits; s += blockDim.x) {
    const float v = pilot[(q * splits + s) * 32 + (j - 1)];  // j <= 32
    sv[s] = v == v ? v : kInf;  // NaN counts as +inf
  }
  __syncthreads();
  // rank counting, ties broken by unit: exactly one unit has rank r - 1
  for (int s = threadIdx.x; s < splits; s += blockDim.x) {
    const float v = sv[s];
    int rank = 0;
    for (int t = 0; t < splits; ++t) {
      const float w = sv[t];
      rank += (w < v || (w == v && t < s)) ? 1 : 0;
    }
    if (rank == r - 1) thr[q] = v < kInf ? next_up(v) : kInf;
  }
}

}  // namespace

cudaError_t launch_pilot_threshold(const float* pilot, int splits, int k, int64_t n_queries,
                                   float* thr, cudaStream_t stream) {
  if (n_queries <= 0) return cudaSuccess;
  if (splits <= 0 || splits > 12288 || n_queries > 0x7fffffff) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(n_queries));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = static_cast<size_t>(splits) * 4;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, pilot_threshold_kernel, pilot, splits, k, thr);
}

cudaError_t launch_bounded_wait_selftest(int* err, uint64_t limit_ns, cudaStream_t stream) {
  bounded_wait_selftest_kernel<<<1, 32, 0, stream>>>(err, limit_ns);
  return cudaGetLastError();
}

int plan_search(int64_t n_rows, int64_t dim, int64_t n_queries, int64_t k, int num_sms,
                Plan* out) {
  if (n_rows <= 0 || dim <= 0 || n_queries <= 0 || k <= 0 || !out) return 1;
  if (k > kMaxK) return 6;
  if (num_sms <= 0) num_sms = 148;
  (void)dim;
  // shared memory per query row: its top-k (full 8-byte keys, or compact
  // 6-byte entries for k > kRegK) and its survivor buffer
  const int64_t heap_full = (k + kRowBuf) * 8;
  const int64_t heap_compact = k * 6 + kRowBuf * 8;
  const int64_t budget = kSmemLimit - kSmemReserve;
  const int64_t row_tiles = (n_rows + kTileRows - 1) / kTileRows;
  *out = Plan{};
  out->row_tiles = row_tiles;
  // Splits of the rows for query_tiles tiles over `slots` concurrent units:
  // the count minimising waves x (tiles per unit + 1), a unit's narrower
  // last tile counted by its width, with the partial lists capped at 1 GiB.
  auto pick_splits = [&](int64_t query_tiles, int64_t n_gran, int64_t gran, int64_t slots) {
    if (query_tiles == 1) return n_gran < slots ? n_gran : slots;
    const int64_t max_s = n_gran < 4 * slots ? n_gran : 4 * slots;
    int64_t best_s = 1;
    double best = -1.0;
    for (int64_t s = 1; s <= max_s; ++s) {
      if (n_queries * s * k * 8 > (int64_t(1) << 30) && s > 1) break;
      const int64_t units = query_tiles * s;
      const int64_t waves = (units + slots - 1) / slots;
      const double per_unit = static_cast<double>((n_gran + s - 1) / s) * gran / kTileRows;
      const double cost = static_cast<double>(waves) * (per_unit + 1.0);
      if (best < 0 || cost < best) {
        best = cost;
        best_s = s;
      }
    }
    return best_s;
  };
  // compact heaps need units of at most kCompactMaxRows rows
  auto compact_fits = [&](int64_t n_gran, int64_t gran, int64_t splits) {
    return k > kRegK && (n_gran + splits - 1) / splits * gran <= kCompactMaxRows;
  };
  // CTA pairs (M = 256 over two SMs, each loading half of every dataset
  // tile into stages of 32 KiB instead of 48) for more than one 128-query
  // tile when either
  //   * the heaps are so large (k >= 62) that one CTA would keep fewer than
  //     3 pipeline stages, or
  //   * pairs pad the queries by at most 5% more rows than single CTAs do
  //     (256-query units against 128).
  // Same-box A/B on one B200, byte-identical results: Q = 10,000, K = 100
  // over 1.25M rows 32.2 -> 28.7 ms; K = 10: Q = 2000 over 200k rows 763 ->
  // 724 us, Q = 10,000 over 1.25M rows 25.7 -> 24.7 ms, Q = 129 over 1M rows
  // 565 -> 481 us; but Q = 300 (512 padded rows against 384) 768 -> 922 us.
  const int64_t single_rows = (n_queries + kQueryRows - 1) / kQueryRows * kQueryRows;
  const int64_t pair_rows = (n_queries + 2 * kQueryRows - 1) / (2 * kQueryRows) * 2 * kQueryRows;
  const bool pair_pays = 20 * pair_rows <= 21 * single_rows;
  const int64_t pair_stages = (budget - kQueryRows * heap_full) / stage_bytes(1);
  const int64_t single_stages = (budget - kQueryRows * heap_full) / kStageBytes;
  if (n_queries > kQueryRows && (single_stages < 3 || pair_pays) && pair_stages >= 2 &&
      num_sms >= 2) {
    const int64_t gran = 2 * kGranRows;
    const int64_t n_gran = (n_rows + gran - 1) / gran;
    const int64_t query_tiles = (n_queries + 2 * kQueryRows - 1) / (2 * kQueryRows);
    const int64_t pairs = num_sms / 2;
    const int64_t splits = pick_splits(query_tiles, n_gran, gran, pairs);
    const int64_t units = query_tiles * splits;
    if (units > INT32_MAX || n_gran * gran > INT32_MAX + int64_t(kTileRows)) return 6;
    // compact heaps where they buy a stage (K = 100: 3 -> 4 stages)
    const int64_t compact_stages = (budget - kQueryRows * heap_compact) / stage_bytes(1);
    const bool compact = compact_stages > pair_stages && compact_fits(n_gran, gran, splits);
    int64_t stages = compact ? compact_stages : pair_stages;
    if (stages > kMaxStages) stages = kMaxStages;
    out->query_block = kQueryRows;
    out->query_tiles = query_tiles;
    out->splits = splits;
    out->units = units;
    out->grid = 2 * (units < pairs ? units : pairs);
    out->stages = stages;
    out->smem_bytes = kSmemReserve + stages * stage_bytes(1) +
                      kQueryRows * (compact ? heap_compact : heap_full);
    out->partial_bytes = n_queries * splits * k * 8;
    out->pair = 1;
    out->heap_rows = kQueryRows;
    out->compact = compact ? 1 : 0;
    out->gran_rows = gran;
    out->unit_queries = 2 * kQueryRows;
    return 0;
  }
  // Single CTAs: the query block (rows per unit) and the stage count follow
  // from the per-query footprint; compact heaps are used where they give
  // more stages (or a larger query block with as many) and every unit fits
  // them.
  struct Single {
    int64_t qb, rows, stages, query_tiles, splits;
  };
  auto single = [&](int64_t per_query, Single* o) {
    int64_t qb_cap = (budget - 2 * kStageBytes) / per_query;
    qb_cap = (qb_cap / 32) * 32;
    if (qb_cap > kQueryRows) qb_cap = kQueryRows;
    if (qb_cap < 32) return false;
    int64_t qb = ((n_queries + 31) / 32) * 32;
    if (qb > qb_cap) qb = qb_cap;
    // a single query tile needs heaps only for the rows the batch has
    const int64_t rows = n_queries <= qb ? (n_queries + 7) / 8 * 8 : qb;
    int64_t stages = (budget - rows * per_query) / kStageBytes;
    if (stages > kMaxStages) stages = kMaxStages;
    if (stages < 2) return false;
    o->qb = qb;
    o->rows = rows;
    o->stages = stages;
    o->query_tiles = (n_queries + qb - 1) / qb;
    o->splits = pick_splits(o->query_tiles, (n_rows + kGranRows - 1) / kGranRows, kGranRows,
                            num_sms);
    return true;
  };
  const int64_t n_gran = (n_rows + kGranRows - 1) / kGranRows;
  Single full{}, cmp{};
  const bool full_ok = single(heap_full, &full);
  const bool cmp_ok = k > kRegK && single(heap_compact, &cmp) &&
                      compact_fits(n_gran, kGranRows, cmp.splits) &&
                      (!full_ok || cmp.stages > full.stages ||
                       (cmp.qb > full.qb && cmp.stages >= full.stages));
  if (!full_ok && !cmp_ok) return 6;
  const Single& c = cmp_ok ? cmp : full;
  const int64_t units = c.query_tiles * c.splits;
  if (units > INT32_MAX || n_gran * kGranRows > INT32_MAX + int64_t(kTileRows)) return 6;
  out->query_block = c.qb;
  out->query_tiles = c.query_tiles;
  out->splits = c.splits;
  out->units = units;
  out->grid = units < num_sms ? units : num_sms;
  out->stages = c.stages;
  out->smem_bytes =
      kSmemReserve + c.stages * kStageBytes + c.rows * (cmp_ok ? heap_compact : heap_full);
  out->heap_rows = c.rows;
  // 32-query blocks with shared-memory heaps spread their queries over the
  // 4 epilogue warps (spread_query_row)
  out->spread = (c.qb == kGranRows && k > kRegK) ? 1 : 0;
  out->partial_bytes = n_queries * c.splits * k * 8;
  out->pair = 0;
  out->compact = cmp_ok ? 1 : 0;
  out->gran_rows = kGranRows;
  out->unit_queries = c.qb;
  return 0;
}

cudaError_t launch_scan(const CUtensorMap& qmap, const CUtensorMap& xmap,
                        const CUtensorMap& xmap_tail, const CUtensorMap& xmap_half,
                        const ScanParams& p, const Plan& plan, cudaStream_t stream,
                        bool overlap) {
  // the opt-in shared-memory limit is a per-device function attribute
  static std::atomic<bool> configured[64] = {};  // set once; idempotent
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (p.metric != KNN_METRIC_L2_EXPANDED && p.metric != KNN_METRIC_INNER_PRODUCT)
    return cudaErrorInvalidValue;
  const bool ip = p.metric == KNN_METRIC_INNER_PRODUCT;
  // [metric][pair][top-k kind: full-key heap, registers, compact heap]
#define KNN_SCAN_FNS(M, P)                                                       \
  reinterpret_cast<const void*>(knn_scan_kernel<M, false, false, P>),           \
      reinterpret_cast<const void*>(knn_scan_kernel<M, true, false, P>),        \
      reinterpret_cast<const void*>(knn_scan_kernel<M, false, true, P>)
  static const void* const fns[12] = {
      KNN_SCAN_FNS(KNN_METRIC_L2_EXPANDED, false), KNN_SCAN_FNS(KNN_METRIC_L2_EXPANDED, true),
      KNN_SCAN_FNS(KNN_METRIC_INNER_PRODUCT, false), KNN_SCAN_FNS(KNN_METRIC_INNER_PRODUCT, true)};
#undef KNN_SCAN_FNS
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    for (const void* fn : fns) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kSmemLimit));
      if (e != cudaSuccess) return e;
    }
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  // compact heaps: rebased row offsets fit 16 bits in every unit
  const bool compact_ok =
      p.k > kRegK && (p.n_gran + p.splits - 1) / p.splits * p.gran_rows <= kCompactMaxRows;
  if (p.n_gran != (p.n_rows + p.gran_rows - 1) / p.gran_rows || p.splits < 1 ||
      p.splits > p.n_gran || (p.pair != 0) != (plan.pair != 0) ||
      (p.compact != 0) != (plan.compact != 0) || (p.compact && !compact_ok) ||
      p.heap_rows != plan.heap_rows || p.heap_rows <= 0 || p.heap_rows > p.query_block ||
      p.heap_rows % 8 != 0 || p.spread != plan.spread ||
      (p.spread && (p.pair || p.query_block != kGranRows || p.k <= kRegK ||
                    p.q_rows < static_cast<int64_t>(p.query_tiles) * kQueryRows)) ||
      (p.pair && (plan.grid % 2 != 0 || p.gran_rows != 2 * kGranRows ||
                  p.unit_queries != 2 * kQueryRows || p.query_block != kQueryRows)))
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(plan.grid));
  cfg.blockDim = dim3(kScanThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(plan.smem_bytes);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = overlap ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = p.pair ? 2 : 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.pair ? 2 : 1;
  // small k: the register top-k (the pilot pass only runs for k > kRegK)
  const bool reg = p.k <= kRegK && !p.pilot;
  const void* fn = fns[(ip ? 6 : 0) + (p.pair ? 3 : 0) + (reg ? 1 : (p.compact ? 2 : 0))];
  void* args[] = {const_cast<CUtensorMap*>(&qmap), const_cast<CUtensorMap*>(&xmap),
                  const_cast<CUtensorMap*>(&xmap_tail), const_cast<CUtensorMap*>(&xmap_half),
                  const_cast<ScanParams*>(&p)};
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace knn
