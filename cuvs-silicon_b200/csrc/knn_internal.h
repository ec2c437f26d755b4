// knn_internal.h -- declarations shared by the engine's translation units.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "cuvs_b200.h"

namespace knn {

// Scan-kernel geometry (fixed for sm_100a).
constexpr int kTileRows = 256;    // dataset rows per full tile = UMMA N
constexpr int kGranRows = 32;     // work units split the rows in granules of this many
constexpr int kTailBox = 32;      // TMA box rows for a unit's last (narrower) tile
constexpr int kQueryRows = 128;   // query rows per tile  = UMMA M
constexpr int kKChunk = 64;       // fp16 per 128-byte swizzled row segment
constexpr int kStageA = kQueryRows * kKChunk * 2;  // 16 KiB query slab
constexpr int kStageB = kTileRows * kKChunk * 2;   // 32 KiB dataset slab
constexpr int kStageBytes = kStageA + kStageB;     // 48 KiB per stage
constexpr int kAccCols = 256;     // TMEM columns per accumulator
constexpr int kTmemCols = 512;    // double-buffered accumulators
constexpr int kScanThreads = 192; // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kMaxStages = 8;
constexpr int kSmemLimit = 232448;        // sm_100 opt-in dynamic smem per CTA
constexpr int kSmemReserve = 1024 + 4096 + 512;  // alignment slack + norm staging + barriers
constexpr int kMaxK = 256;
constexpr int kRowBuf = 16;       // buffered survivors per query row
constexpr int64_t kCompactMaxRows = 65535;  // rows of a unit with compact heaps
constexpr uint32_t kNoIndex = 0xFFFFFFFFu;

// Device-side error codes (written to a kernel's error word; 0 = ok).
constexpr int kErrTimeoutFull = 1;      // MMA waiting for a TMA stage
constexpr int kErrTimeoutEmpty = 2;     // producer waiting for a free stage
constexpr int kErrTimeoutAccFull = 3;   // epilogue waiting for an accumulator
constexpr int kErrTimeoutAccEmpty = 4;  // MMA waiting for the epilogue
constexpr int kErrTimeoutDrain = 5;     // unwinding waits
constexpr int kErrBounds = 6;           // debug build: a bounds check tripped
constexpr int kErrTimeoutEpilogue = 8;  // an epilogue warp waiting for the others

struct ScanParams {
  const float* row_norms;    // [n_rows]
  const float* query_norms;  // [n_queries]
  float* part_d;             // [n_queries][splits][k]
  uint32_t* part_i;          // [n_queries][splits][k]
  int* err;                  // device error word (0 = ok)
  int64_t n_rows;
  int64_t n_queries;
  int64_t n_gran;  // ceil(n_rows / kGranRows)
  int64_t q_rows;  // rows of the fp16 query buffer (padded_query_rows)
  int64_t ld;      // leading dimension of the fp16 rows and queries (halves)
  // CTA pairs (pair = 1): clusters of two CTAs share each dataset tile
  // (cta_group::2 MMAs, M = 256); a unit then covers 256 query rows, 128
  // per CTA.  Work units split the rows in granules of gran_rows.
  int32_t pair;
  // Compact heaps (compact = 1, k > 16 only): a heap entry is the distance's
  // order image (32 bits) and the row's offset from the unit's first row
  // (16 bits), 6 bytes instead of 8; needs units of at most kCompactMaxRows
  // rows.
  int32_t compact;
  int32_t gran_rows;     // kGranRows, or 2 * kGranRows with pairs
  int32_t unit_queries;  // query rows of a unit: query_block, or 256 with pairs
  int32_t k;
  int32_t query_block;  // query rows owned per work unit (multiple of 32, <= 128)
  // rows of the shared-memory top-k heaps and survivor buffers (<=
  // query_block): with a single query tile, only the rows the batch has
  // (rounded up to 8), which can leave room for another pipeline stage
  int32_t heap_rows;
  // spread = 1: 32-query blocks in the spread layout (spread_query_row):
  // block m's slab starts at query row 128 * m and query j of the block is
  // TMEM lane 32 * (j % 4) + j / 4
  int32_t spread;
  int32_t query_tiles;
  int32_t splits;
  int32_t units;
  int32_t k_chunks;  // ceil(ld / 64)
  int32_t stages;
  int32_t dataset_evict_first;
  int32_t metric;  // KNN_METRIC_L2_EXPANDED or KNN_METRIC_INNER_PRODUCT
  // Pilot pass (pilot = 1): each unit scans only its first tile and writes
  // its 32 sorted group minima per query to pilot_out[q][splits][32].
  int32_t pilot;
  float* pilot_out;
  // Main pass: per-query starting threshold (nullptr: none).
  const float* thr_init;
  // Per-query bound shared by all CTAs (nullptr: none), as order-preserving
  // bits of a distance B such that some unit holds k rows at d <= B;
  // 0xFFFFFFFF = none yet.  Reset by the query conversion of each search.
  uint32_t* bound;
};

// k above which a search runs the pilot pass first (see knn_scan.cu).
constexpr int kPilotMinK = 17;

// Per-query starting thresholds from a pilot pass's group minima
// (pilot_threshold_kernel in knn_scan.cu); thr: [n_queries].
cudaError_t launch_pilot_threshold(const float* pilot, int splits, int k, int64_t n_queries,
                                   float* thr, cudaStream_t stream);

struct Plan {
  int64_t query_block, query_tiles, row_tiles, splits, units, grid, stages;
  int64_t smem_bytes, partial_bytes;
  int64_t pair = 0, gran_rows = kGranRows, unit_queries = 0;
  int64_t compact = 0;
  int64_t heap_rows = 0;
  int64_t spread = 0;
};

// Returns 0 and fills `out`, or a KNN_E* status (KNN_EUNSUPPORTED when k is
// too large for the shared-memory budget).
int plan_search(int64_t n_rows, int64_t dim, int64_t n_queries, int64_t k, int num_sms,
                Plan* out);

// Launchers (return the CUDA error of the launch).
// `overlap` launches the kernel as a programmatic dependent of the one
// before it (its set-up overlaps that kernel's tail); off when the caller
// brackets kernels with timing events.  xmap: the dataset rows with
// kTileRows-row boxes; xmap_tail: the same rows with kTailBox-row boxes (a
// unit's last tile is loaded as several of these); xmap_half: the same rows
// with kTileRows / 2-row boxes (each CTA's half of a full tile with CTA
// pairs).
cudaError_t launch_scan(const CUtensorMap& qmap, const CUtensorMap& xmap,
                        const CUtensorMap& xmap_tail, const CUtensorMap& xmap_half,
                        const ScanParams& p, const Plan& plan, cudaStream_t stream,
                        bool overlap = true);

// fp32/fp16 rows -> fp16 rows with leading dimension ld (zero padded) plus
// fp32 norms of the rounded rows.  in_is_half selects the input type.
// Output rows [rows, rows_out) are written as zeros (no norm).  fill
// (optional): fill_n words set to 0xFFFFFFFF (the scan's shared per-query
// bounds, reset by the query conversion of every search).  epoch (optional):
// a device word incremented once (the exchange epoch of the search that this
// conversion opens).
cudaError_t launch_convert_rows(const void* in, bool in_is_half, int64_t rows,
                                int64_t rows_out, int64_t dim, __half* out, int64_t ld,
                                float* norms, cudaStream_t stream, uint32_t* fill = nullptr,
                                int64_t fill_n = 0, uint32_t* epoch = nullptr,
                                bool spread = false);

// Spread query blocks (ScanParams::spread): query j of a 32-query block
// sits in row 32 * (j % 4) + j / 4 of the block's 128-row slab, so each of
// the 4 TMEM lane quadrants (one epilogue warp each) holds up to 8 of them.
// launch_convert_rows(..., spread = true) writes that layout (the slab of
// block m starts at row 128 * m; rows holding no query are zeros).
inline int64_t spread_query_row(int64_t q) {
  return q / 32 * kQueryRows + 32 * (q % 4) + (q % 32) / 4;
}

// Rows of the fp16 query buffer a search needs: every 128-row query slab
// the scan kernel loads lies inside it, so no TMA box leaves the buffer.
inline int64_t padded_query_rows(const Plan& plan) {
  if (plan.pair) return plan.query_tiles * 2 * kQueryRows;
  if (plan.spread) return plan.query_tiles * kQueryRows;
  return (plan.query_tiles - 1) * plan.query_block + kQueryRows;
}

// Launches the bounded-wait self-test kernel (see knn_scan.cu).
cudaError_t launch_bounded_wait_selftest(int* err, uint64_t limit_ns, cudaStream_t stream);

// Peer exchange of per-rank top-k lists over NVLink (replaces the NCCL
// all-gather for searches that fit).  Every rank owns one exchange buffer
// of 16-byte entries [2 parities][n_ranks][cap_qk]: entry (p, r, q*k + e)
// holds element e of rank r's list for query q as two 8-byte words, (epoch
// << 32 | distance bits) and (epoch << 32 | row index).  An 8-byte store is
// seen whole or not at all, so a reader that finds the search's epoch in
// both words has the entry: no fence and no separate flag are needed.
// `base[r]` is rank r's buffer as this GPU addresses it (its own allocation
// or a CUDA IPC mapping).  Searches alternate parities, so a rank can write
// search e + 1 while a slower peer still reads search e.
//
// The epoch lives in device memory (`epoch`), not in the kernel arguments:
// the query conversion that opens every search adds one to it (after waiting
// for the previous search's kernels), and both exchange kernels read it only
// after their own griddepcontrol.wait, by which time that conversion has
// completed.  A search's kernels therefore carry no per-search argument and
// can be captured once in a CUDA graph and replayed.
constexpr int kMaxRanks = 8;
struct Exchange {
  float* base[kMaxRanks];
  int64_t cap_qk;
  int n_ranks;
  int rank;
  int mode;               // 0 none; 1 exchange (push, receive every rank's list, merge)
  const uint32_t* epoch;  // device word: the current search's epoch (>= 1)
  uint64_t wait_ns;       // how long to wait for a peer's list
  int* err;               // device error word (wait timeouts, debug bounds checks)
  float* dec_d;           // received lists, decoded: [q][n_ranks][k]
  uint32_t* dec_i;
  int64_t in_len;         // entries of the merge's in_d / in_i (debug bounds checks)
};
constexpr int kErrTimeoutPeer = 7;  // a peer's list never arrived
constexpr uint64_t kPeerWaitDefaultNs = 1000000000ull;  // 1 s

inline int64_t exchange_words(int n_ranks, int64_t cap_qk) {
  return static_cast<int64_t>(n_ranks) * cap_qk * 8;  // 2 parities x 16 bytes, in 4-byte words
}

// Merges n_lists sorted top-k lists per query into the final top-k.
// List l of query q starts at in_{d,i}[q * stride_query + l * stride_list].
// Valid indices get index_offset added.  out_i is uint32 (no-neighbour =
// UINT32_MAX) or int64 (no-neighbour = -1) per out_i64.
// `ex` (optional, mode 1) selects the peer exchange: the block of query q
// merges this rank's lists, writes the result into every rank's exchange
// buffer, then receives every rank's list for q from this rank's buffer
// (bounded wait), decodes them to ex->dec_d/dec_i and merges those into
// out_d/out_i.  `negate_out` writes -d to out_d (the inner-product metric
// orders by -q.x internally and reports q.x; padding becomes -inf); lists
// written to an exchange buffer are never negated.
// err, in_len (optional): the device error word and the number of entries
// of in_d / in_i, for the debug build's bounds checks (with an exchange,
// ex->err and ex->in_len are used instead).
cudaError_t launch_merge(const float* in_d, const uint32_t* in_i, int64_t stride_list,
                         int64_t stride_query, int n_lists, int k, int64_t n_queries,
                         int64_t index_offset, float* out_d, void* out_i, bool out_i64,
                         cudaStream_t stream, bool overlap = true,
                         const Exchange* ex = nullptr, bool negate_out = false,
                         int* err = nullptr, int64_t in_len = 0);

// Exact fp32 re-ranking (knn_rerank.cu).  cand_{d,i}: per query the scan's
// top kc (kc >= k, kc <= kMaxK) sorted candidates, local row indices,
// scan distances in the internal order (minus the score for the inner
// product).  rows: the fp32 rows (n x dim, dense).  Writes the k best by
// exact fp32 distance to out_{d,i} (index_offset added; negate_out as in
// launch_merge) and adds 1 to *uncertified for every query whose result is
// not proven to be the exact fp32 top-k.  max_norm2: device scalar, the
// largest fp32 norm |x16|^2 of the fp16 rows.
cudaError_t launch_rerank(const float* queries, const float* rows, int64_t dim,
                          const float* cand_d, const uint32_t* cand_i, int kc, int k,
                          int64_t n_queries, int metric, const float* max_norm2,
                          int64_t index_offset, float* out_d, void* out_i, bool out_i64,
                          bool negate_out, int* uncertified, cudaStream_t stream);

// The certificate's bound of |scan distance - fp32 distance| (knn_rerank.cu)
// for a row that could beat a re-ranked distance r; qn = |q|, xn >= |x|.
double rerank_bound(int metric, double r, double qn, double xn, int64_t dim);

// out = the largest of norms[0..n) (norms >= 0).
cudaError_t launch_max_norm(const float* norms, int64_t n, float* out, cudaStream_t stream);

// Candidates the fp16 scan keeps per query for a re-ranked top-k: twice k,
// at least 32 (the scan seeds its threshold for up to 32), at most kMaxK.
inline int rerank_candidates(int64_t k) {
  int64_t kc = 2 * k < 32 ? 32 : 2 * k;
  return static_cast<int>(kc > kMaxK ? kMaxK : kc);
}

}  // namespace knn
