/*
 * cuvs_b200.h -- C ABI of the B200 exact brute-force k-NN engine.
 *
 * This is the drop-in boundary for the reference's exact L2 search path
 * (ysys143/cuvs-silicon): everything the reference's C++ layer asks of its
 * device runtime for that path is one of the functions below.  Plain C
 * types only: pointers, sizes and int status codes.  Pointers may be host
 * or device memory; the engine classifies them and stages host buffers.
 *
 * Reference interfaces replaced (file:line in the reference repository):
 *   knn_index_create / knn_index_destroy
 *       cuvs_silicon::MetalContext::instance() / is_available()
 *       (include/cuvs_silicon/metal_context.hpp:15-19,
 *        src/metal_context.mm:59-101)
 *   knn_index_build
 *       the lazy dataset cache of search_brute_force: fp16 copy of the
 *       dataset and fp32 row norms keyed on (ptr, N, D)
 *       (src/metal_context.mm:22-55,155-175), moved to build time, plus the
 *       validation of cuvs::neighbors::cagra::build (src/cagra.cpp:26-32)
 *   knn_index_search
 *       MetalContext::search_brute_force (metal_context.hpp:36-41,
 *       src/metal_context.mm:139-255), reached from cagra::search
 *       (src/cagra.cpp:197-202) and, on hosts without a GPU, its CPU exact
 *       path (src/cagra.cpp:211-252) whose output contract it keeps:
 *       squared L2, ascending (distance, index), k > n padded with
 *       UINT32_MAX / +inf
 *   knn_dispatch_count / knn_reset_dispatch_count
 *       cuvs::neighbors::cagra::metal_dispatch_count /
 *       reset_metal_dispatch_count (include/cuvs/neighbors/cagra.hpp:119-122,
 *       src/cagra.cpp:258-266,369-371)
 *
 * Functions with no counterpart in the reference (it runs on one device and
 * has no configuration surface) say so in their comment.
 *
 * Status codes: every function returning int returns KNN_OK (0) or one of
 * the KNN_E* codes; knn_last_error() then describes the failure (thread
 * local).  The C++ layer maps KNN_EINVAL to std::invalid_argument and the
 * rest to std::runtime_error, as the reference throws
 * (src/cagra.cpp:26-32,100-111; src/metal_context.mm:146-147,245-246).
 */
#ifndef CUVS_B200_H_
#define CUVS_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KNN_OK 0
#define KNN_EINVAL 1       /* invalid argument (reference: invalid_argument) */
#define KNN_ECUDA 2        /* CUDA runtime/driver error or no usable GPU */
#define KNN_ENCCL 3        /* NCCL error */
#define KNN_ETIMEOUT 4     /* a bounded device wait expired */
#define KNN_ENOMEM 5       /* device or host allocation failed */
#define KNN_EUNSUPPORTED 6 /* valid request outside the engine's limits */

#define KNN_DTYPE_F32 0
#define KNN_DTYPE_F16 1

/* Metrics.  L2Expanded: squared L2 distances, ascending.  InnerProduct
 * (declared by the reference at include/cuvs/distance/distance.hpp:5-8 and
 * rejected by its cagra::build, src/cagra.cpp:26-28): the inner products
 * q.x, descending, ties by ascending index, padding -inf. */
#define KNN_METRIC_L2_EXPANDED 0 /* cuvs::distance::DistanceType::L2Expanded */
#define KNN_METRIC_INNER_PRODUCT 1 /* cuvs::distance::DistanceType::InnerProduct */

/* Largest k one search accepts (per-CTA top-k state must fit in shared
 * memory next to a two-stage pipeline and a survivor buffer).  The reference's Metal kernel caps k
 * at 16 (shaders/cagra_kernels.metal:538); its CPU path has no cap. */
#define KNN_MAX_K 256

/* UINT32_MAX marks "no neighbour" (src/cagra.cpp:248-249). */
#define KNN_NO_INDEX 0xFFFFFFFFu

typedef struct knn_index knn_index;

/* Search-plan description (host-side planner; no counterpart in the
 * reference, exposed for tests and tooling). */
typedef struct knn_plan {
  int64_t query_block;   /* queries per CTA work unit (multiple of 32) */
  int64_t query_tiles;   /* ceil(n_queries / unit_queries) */
  int64_t row_tiles;     /* ceil(n_rows / 256) */
  int64_t splits;        /* row-range splits per query tile */
  int64_t units;         /* query_tiles * splits */
  int64_t grid;          /* persistent CTAs launched */
  int64_t stages;        /* shared-memory pipeline stages */
  int64_t smem_bytes;    /* dynamic shared memory per CTA */
  int64_t partial_bytes; /* scratch for per-unit top-k lists */
  int64_t pair;          /* 1: pairs of CTAs share each dataset tile (cta_group::2) */
  int64_t unit_queries;  /* queries per work unit (query_block, or 256 with pairs) */
  int64_t compact_heap;  /* 1: k > 16 top-k heaps of 6-byte entries (units of <= 65535 rows) */
} knn_plan;

/* Human-readable text for the calling thread's last failure. */
const char* knn_last_error(void);
/* Static name of a status code. */
const char* knn_status_string(int status);

/* Creates an empty index bound to CUDA device `device`.  Replaces the
 * reference's MetalContext singleton (metal_context.hpp:15-19); one index
 * per dataset instead of one process-wide cache keyed on a raw pointer. */
int knn_index_create(int device, knn_index** out);
int knn_index_destroy(knn_index* index);

/* Orders the index's work on a caller-owned cudaStream_t (NULL restores the
 * index's own stream).  No counterpart: the reference blocks on every
 * command buffer (src/metal_context.mm:222-225,242-243). */
int knn_index_set_stream(knn_index* index, void* cuda_stream);

/* Loads `rows` (n_rows x dim, row-major, fp32 or fp16, host or device) into
 * device HBM as fp16 rows (round-to-nearest-even) and fills the fp32 row
 * norms ||x16||^2.  Replaces the first-search cache fill of
 * search_brute_force (src/metal_context.mm:155-175) and the checks of
 * cagra::build (src/cagra.cpp:26-32): only L2 (and inner product) metrics,
 * non-null non-empty data.  n_rows must be below 2^32 - 1 (neighbour indices
 * are uint32, cagra.hpp:54-55). */
int knn_index_build(knn_index* index, const void* rows, int dtype,
                    int64_t n_rows, int64_t dim, int metric);

/* Same as knn_index_build for one row shard of a larger dataset: rows
 * [row_offset, row_offset + n_rows) of a total_rows-row dataset.  Neighbour
 * indices reported by searches are global (row_offset added).  No
 * counterpart: the reference runs on one device. */
int knn_index_build_shard(knn_index* index, const void* rows, int dtype,
                          int64_t n_rows, int64_t dim, int metric,
                          int64_t row_offset, int64_t total_rows);

/* Dataset file formats for knn_index_build_file. */
#define KNN_FILE_FVECS 0   /* per row: int32 dim, dim float32 (src/sift_loader.cpp:21-64) */
#define KNN_FILE_BIN_F32 1 /* int32 rows, int32 cols, rows x cols float32
                              (tests/test_cohere_wiki_validation.cpp:40-52) */

/* Builds the index from a dataset file without holding it in host memory:
 * the file is read in 64 MiB chunks into two pinned buffers, and each chunk
 * is copied to the device and converted while the next one is read.  With
 * n_ranks > 1 only this rank's row shard (knn_shard_range) is read and the
 * index reports global row indices (as knn_index_build_shard).  Every fvecs
 * record must have the width of the first; the file must end at a record
 * boundary.  Replaces the reference's load-then-build sequence
 * (load_fvecs / load_bin followed by cagra::build, which copies the whole
 * fp32 dataset into the index). */
int knn_index_build_file(knn_index* index, const char* path, int format, int metric,
                         int n_ranks, int rank);

int64_t knn_index_rows(const knn_index* index);
int64_t knn_index_dim(const knn_index* index);
/* The CUDA device the index lives on (-1 for a null index). */
int knn_index_device(const knn_index* index);

/* The index's device cache, the state the reference's MetalContext keeps for
 * a dataset (src/metal_context.mm:38-54,155-175: the fp16 copy of the rows
 * and the fp32 d_norms), owned here by the index: the fp16 rows (n_rows rows
 * of `ld` halves each, the first dim of them the values, the rest zero) and
 * the fp32 squared norms of those fp16 rows (n_rows floats).  Device
 * pointers, valid until the index is rebuilt or destroyed; read only. */
int knn_index_device_rows(knn_index* index, const void** rows_f16, int64_t* ld);
int knn_index_device_norms(knn_index* index, const float** norms);

/* Builds the index (or one row shard, as knn_index_build_shard) from rows
 * already in the engine's storage format: fp16 rows (host or device,
 * n_rows x dim, dense) and the fp32 norms a previous build computed for
 * them (knn_index_device_norms), as cuvs::neighbors::brute_force::serialize
 * stores them with its fp16 payload.  Nothing is converted or recomputed:
 * the norms must belong to these rows.  No counterpart in the reference
 * (its cache is rebuilt from fp32 rows on every first search). */
int knn_index_build_prepared(knn_index* index, const void* rows_f16, const float* norms,
                             int64_t n_rows, int64_t dim, int metric, int64_t row_offset,
                             int64_t total_rows);

/* Copies the index's stored rows (n_rows x dim, row-major, the fp16 values
 * the engine searches) into `out`: dtype KNN_DTYPE_F16 to host or device
 * memory, KNN_DTYPE_F32 (exact widening) to host memory.  Used to save an
 * index in the reference's container (src/cagra.cpp:305-328 writes the
 * dataset as fp32). */
int knn_index_copy_rows(knn_index* index, void* out, int dtype);

/* Exact k-NN of n_queries fp32 queries (host or device, row-major, index
 * dim columns), 1 <= k <= KNN_MAX_K.  Writes neighbours (uint32) and
 * distances (fp32), each n_queries x k: squared L2 distances ascending by
 * (distance, index), or for KNN_METRIC_INNER_PRODUCT the inner products
 * descending (ties by ascending index); slots beyond the number of rows
 * hold KNN_NO_INDEX / +inf (-inf for the inner product).  Blocks until the
 * results are in place, like the reference (src/metal_context.mm:222-252).
 * k == 0 or n_queries == 0 is a no-op.  Page-locked host buffers are read
 * and written in place; pageable ones are staged through device memory.
 * A search repeating the buffers and shape of an earlier one replays a CUDA
 * graph (knn_index_set_graphs).  When a communicator is attached
 * (knn_index_attach_comm) every rank must call this with the same queries
 * and k; each rank receives the merged global result.
 * Replaces MetalContext::search_brute_force (src/metal_context.mm:139-255). */
int knn_index_search(knn_index* index, const float* queries, int64_t n_queries,
                     int64_t k, uint32_t* neighbors, float* distances);

/* As knn_index_search with int64 neighbours (cuVS brute_force convention);
 * "no neighbour" is written as -1.  No counterpart in the reference. */
int knn_index_search_i64(knn_index* index, const float* queries,
                         int64_t n_queries, int64_t k, int64_t* neighbors,
                         float* distances);

/* Size of the device scratch array used by knn_index_search_noalloc. */
#define KNN_NOALLOC_SCRATCH_BYTES (16 * 1024 * 1024)

/* knn_index_search without allocating: same arguments, same results, same
 * blocking behaviour.  No counterpart in the reference.  It is for callers
 * that cannot call cudaMalloc while they search: a serving process whose
 * device memory is owned by another allocator or budget, or code that must
 * not risk the device-wide synchronisation that cudaMalloc/cudaFree may
 * cause.  Its per-search scratch is one static device array of
 * KNN_NOALLOC_SCRATCH_BYTES (16 MiB) that every GPU loading the library
 * holds until exit.  A search whose scratch (fp16 queries, norms, per-split
 * top-k lists, staging of host buffers) exceeds it fails with
 * KNN_EUNSUPPORTED; the headline search (100 queries, k = 10, dim 1024)
 * needs about 2 MiB.  The first call on a device looks up the array's
 * device address, so make it before any stream capture.  Calls share the
 * array: concurrent calls on one device are serialised by the library; other
 * work that overlaps them on the GPU and touches the array would race.
 * The index must be built, and no communicator may be attached.  Unlike
 * knn_index_search it runs neither the pilot pass (k >= 17) nor the
 * per-query bound the scan's CTAs share, whose scratch it does not carve:
 * results are the same, but searches with k >= 17 run the slower unseeded
 * scan (k = 256 at 1M x 1024 took 2.5-3.4x as long before the engine had
 * these two steps).  The array's device address is
 * cached per device for the life of the process; a device reset
 * (cudaDeviceReset), which also invalidates every index on that device, is
 * not supported. */
int knn_index_search_noalloc(knn_index* index, const float* queries,
                             int64_t n_queries, int64_t k, uint32_t* neighbors,
                             float* distances);

/* Stream-ordered search: all four pointers must be device memory; returns
 * after enqueueing on the index's stream without synchronising.  Errors
 * raised by the kernels themselves (bounded-wait timeouts) are reported by
 * the next knn_index_sync.  No counterpart in the reference. */
int knn_index_search_async(knn_index* index, const float* queries,
                           int64_t n_queries, int64_t k, uint32_t* neighbors,
                           float* distances);
/* Waits for the index's stream and reports device-side errors. */
int knn_index_sync(knn_index* index);

/* Stream-ordered search of one row shard whose result is merged later with
 * other shards' (knn_merge_lists): as knn_index_search_async (device
 * buffers, global row indices), but distances stay in the order the merge
 * works in: squared L2 ascending, or for the inner product -q.x ascending
 * (so that ties still go to the smaller index).  The index must not have a
 * communicator attached.  No counterpart in the reference. */
int knn_index_search_lists(knn_index* index, const float* queries, int64_t n_queries,
                           int64_t k, uint32_t* list_neighbors, float* list_distances);

/* Merges n_lists per-shard results of knn_index_search_lists into the
 * final top-k on device `device`, stream-ordered on `cuda_stream` (NULL:
 * the legacy default stream).  lists_*: [n_lists][n_queries][k] in device
 * memory of `device` (copy other devices' lists there first); outputs, in
 * device memory of `device`, as knn_index_search (inner product: q.x
 * descending), with int64 neighbours (-1 = none) when neighbors_i64 != 0.
 * No counterpart in the reference, which searches on one device. */
int knn_merge_lists(int device, void* cuda_stream, const float* lists_distances,
                    const uint32_t* lists_neighbors, int n_lists, int64_t n_queries, int64_t k,
                    int metric, void* neighbors, int neighbors_i64, float* distances);

/* Exact fp32 re-ranking (no counterpart in the reference's Metal path; it
 * makes searches return what the reference's portable exact search,
 * src/cagra.cpp:211-252, returns for the same fp32 rows).
 *
 * enabled != 0 before knn_index_build keeps the fp32 rows on the device
 * (n_rows x dim x 4 bytes next to the fp16 copy; fp32 input only).  Each
 * search then keeps max(32, 2k) (at most KNN_MAX_K) fp16-scan candidates
 * per query, recomputes their distances from the fp32 rows with the
 * reference's arithmetic (sequential fp32 sum of (q[d] - x[d])^2, no fused
 * multiply-add; inner product: sequential fp32 sum of q[d] * x[d]) and
 * returns the k best by (distance, index).  Reported distances are
 * bit-identical to the reference's.  A query is CERTIFIED when a rounding
 * bound proves that no row outside its candidates can enter its top-k
 * (then its result is exactly the reference's).  A blocking search on one
 * device repeats itself once with KNN_MAX_K candidates when some query is
 * not certified.  Returns KNN_EINVAL (and keeps re-ranking enabled for the
 * next build) when the index already holds rows built without their fp32
 * copy.  enabled = 0 frees the fp32 rows. */
int knn_index_set_rerank(knn_index* index, int enabled);

/* For the most recent re-ranked search that completed (a blocking search,
 * or knn_index_sync after knn_index_search_async): the number of queries
 * whose result is not certified, and the number that were not certified
 * with the first candidate count (and so were searched again). */
int knn_index_rerank_stats(knn_index* index, int64_t* uncertified, int64_t* widened);

/* The re-rank certificate's bound on |scan distance - fp32 distance| for a
 * row whose fp32 distance does not exceed r (for the inner product, on the
 * scores), given |q| = query_norm and |x| <= row_norm; the same function
 * the kernel evaluates.  Pure host arithmetic, exposed for tests; -1 on
 * invalid arguments.  No counterpart in the reference. */
double knn_rerank_bound(int metric, double r, double query_norm, double row_norm,
                        int64_t dim);

/* Plans a search without running it (pure host arithmetic).  num_sms <= 0
 * uses 148 (B200).  No counterpart in the reference. */
int knn_plan_search(int64_t n_rows, int64_t dim, int64_t n_queries, int64_t k,
                    int num_sms, knn_plan* out);

/* Contiguous row shard [begin, end) of rank `rank` among n_ranks:
 * begin = rank * ceil(n_rows / n_ranks), clipped to n_rows.  Pure host
 * arithmetic.  No counterpart in the reference. */
int knn_shard_range(int64_t n_rows, int n_ranks, int rank, int64_t* begin,
                    int64_t* end);

/* Multi-GPU, one process per GPU.  knn_comm_unique_id fills 128 bytes on one
 * rank; the caller broadcasts them; every rank then calls
 * knn_index_attach_comm with the same bytes.  Searches on an index with a
 * communicator all-gather the per-rank top-k lists over NCCL and merge them
 * on the device.  No counterpart in the reference (single device). */
int knn_comm_unique_id(void* out_128_bytes);
int knn_index_attach_comm(knn_index* index, const void* unique_id_128_bytes,
                          int n_ranks, int rank);

/* CUDA graphs (on by default): a search is captured once into a CUDA graph
 * (query conversion, scan, merges and, with a communicator, the peer
 * exchange) and replayed when later searches repeat the same buffers, sizes
 * and stream.  Rebuilding the index, changing its stream, communicator,
 * peer-exchange setting or peer timeout, or growing its scratch memory
 * discards the graphs.  Searches that exchange their lists through NCCL
 * (see knn_index_set_peer_exchange) are always launched directly.  No
 * counterpart in the reference. */
int knn_index_set_graphs(knn_index* index, int enabled);

/* Peer exchange (on by default when every rank could map every other
 * rank's exchange buffer at knn_index_attach_comm): the per-rank top-k
 * lists of a search travel as direct NVLink stores into every rank's
 * buffer, every entry tagged with the search's epoch, and each rank's final
 * merge waits for its peers' entries for at most the peer timeout (below),
 * counted from the moment this rank's own lists are complete.  Searches
 * with more than 65,536 query x k entries, and indexes with the exchange
 * off, use the NCCL all-gather.  Every rank must make the same choice.  No
 * counterpart in the reference. */
int knn_index_set_peer_exchange(knn_index* index, int enabled);

/* Bound of the peer-exchange wait, in microseconds (1 ms .. 600 s; default
 * 1 s).  Every rank must issue each search within this bound of the others
 * (the slowest rank's lists must arrive before the fastest rank's wait
 * runs out): host-side skew between ranks (Python, first-call set-up, a
 * rank that computes something else first) counts against it.  When the
 * bound expires the search returns KNN_ETIMEOUT and the communicator must
 * be attached again.  No counterpart in the reference. */
int knn_index_set_peer_timeout(knn_index* index, int64_t microseconds);

/* Kernel timing: when enabled, the engine records CUDA events around its
 * fused scan kernel and its merge kernels on the stream they are launched on
 * and accumulates their durations.  No counterpart in the reference. */
int knn_index_set_profiling(knn_index* index, int enabled);
int knn_index_kernel_stats(knn_index* index, double* scan_ms, double* merge_ms,
                           int64_t* scan_launches, int64_t* kernel_launches);
int knn_index_reset_kernel_stats(knn_index* index);

/* Failure-detection self-test: launches one kernel whose thread waits on a
 * shared-memory barrier that nothing arrives on, with the engine's bounded
 * wait limited to limit_us microseconds (1..2,000,000).  Returns
 * KNN_ETIMEOUT when the wait gave up and reported it, as designed; the
 * device stays usable.  No counterpart in the reference. */
int knn_selftest_bounded_wait(int device, int64_t limit_us);

/* Number of engine kernels launched since the last reset (all indices).
 * Replaces cagra::metal_dispatch_count (cagra.hpp:119-122). */
uint64_t knn_dispatch_count(void);
void knn_reset_dispatch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* CUVS_B200_H_ */
