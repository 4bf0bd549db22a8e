/*
 * circuit-b200 C ABI: exact top-k inner-product search over a .circuit index on
 * one B200 (sm_100a) per process.
 *
 * Every entry point takes plain pointers and sizes; no torch or C++ types cross
 * this boundary.  The first four functions and the two structs keep the exact
 * names, argument meaning, layout and error behaviour of the reference's native
 * library, so existing callers (e.g. circuit_bench) relink unchanged:
 *
 *   reference native/include/circuit/circuit.h:8-46  (declarations)
 *   reference native/src/api.cpp:7-51                (NULL / -1 conventions)
 *
 * Differences a caller can observe (all deliberate):
 *   - k is not clamped to 32; any 1 <= k <= CIRCUIT_MAX_K works (reference
 *     clamps at gpu_index.cpp:243, :334).  When k exceeds the number of rows
 *     N, every row is returned first (in score order) and the remaining
 *     k - N slots hold score -INFINITY and id -1, so the output buffers are
 *     always fully written (the reference's Python path instead shortens the
 *     result to N, circuit_rag/search.py:51; the Python package here does the
 *     same).  This holds for every single-query, batched and no-alloc call.
 *   - pruning is on: the hierarchical path seeds an on-device threshold and
 *     prunes with rigorously inflated bounds; the reference native path runs
 *     with threshold -1e9 (gpu_index.cpp:279) and never prunes.  Results are
 *     identical to brute force in both.
 *   - circuit_trace_t.vectors_scored counts the rows of the children that
 *     survive the seed threshold's bounds (reference always reports N,
 *     gpu_index.cpp:326); circuit_trace_ex_t.rows_streamed counts the rows the
 *     scan actually read.
 *   - errors return a negative CIRCUIT_ERR_* code (reference returns 0 even
 *     when CUDA calls fail); circuit_last_error() describes the last one.
 *
 * Threading: one in-flight search per index handle (the handle owns one
 * device workspace for single queries and one for batches, each used by one
 * call at a time), as in the reference.  Use one handle per thread/stream.
 */
#ifndef CIRCUIT_H
#define CIRCUIT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CIRCUIT_ABI_VERSION 2
#define CIRCUIT_MAX_K 256
#define CIRCUIT_MAX_RANK 64
#define CIRCUIT_MAX_DIM 2048

/* error codes (0 = success) */
#define CIRCUIT_OK 0
#define CIRCUIT_ERR_NULL (-1)        /* null index handle (reference api.cpp:28-29, :41-42) */
#define CIRCUIT_ERR_ARG (-2)         /* bad argument: k, pointer, size, alignment */
#define CIRCUIT_ERR_CUDA (-3)        /* a CUDA runtime call failed */
#define CIRCUIT_ERR_TIMEOUT (-4)     /* a bounded device-side wait gave up */
#define CIRCUIT_ERR_IO (-5)          /* file open / read / mmap failed */
#define CIRCUIT_ERR_FORMAT (-6)      /* malformed .circuit file or index arrays */
#define CIRCUIT_ERR_UNSUPPORTED (-7) /* dim / rank / k outside the supported range */

typedef struct circuit_index_opaque* circuit_index_t;

/* reference circuit.h:10-14 (declared there, unused there and here) */
typedef struct {
  int top_k;
  float threshold;
  int use_cuda_graph;
} circuit_search_config_t;

/* reference circuit.h:16-19 */
typedef struct {
  float latency_us;
  int vectors_scored;
} circuit_trace_t;

/* Extended per-search statistics (no reference counterpart). */
typedef struct {
  float latency_us;            /* host wall time of the call (0 for async calls) */
  int32_t path;                /* 0 = flat scan, 1 = hierarchical */
  int64_t vectors_scored;      /* rows of the children whose bound is not below the seed threshold:
                                  what a scan of the survivors alone reads (flat path: N) */
  int64_t vectors_total;       /* N */
  int32_t surviving_roots;     /* roots not pruned (seed root included) */
  int32_t surviving_children;  /* non-empty children scanned */
  int32_t total_children;      /* num_total_children */
  int32_t best_root;           /* the seed root */
  float seed_threshold;        /* k-th best score among the sampled rows of the seed root (-inf if none) */
  int32_t device_error;        /* device error bits of the last search (0 = none) */
  int32_t seed_sample_rows;    /* rows of the seed root scored beforehand for the threshold (not in
                                  vectors_scored; scanned again when their children survive);
                                  ABI version 2 */
  int32_t rows_streamed;       /* leaf rows the main scan read.  The hierarchical scan runs beside the
                                  bounds kernel and streams every child whose bound is not known yet,
                                  then skips the children whose bound is below the running threshold
                                  (which rises above the seed's): more rows than vectors_scored on
                                  small corpora, which stream whole before the bounds are ready, and
                                  at most as many once the bounds lead the scan.  ABI version 2 */
} circuit_trace_ex_t;

/* ------------------------------------------------------------------ reference ABI */

/* Load a .circuit file onto device `device_id`.  NULL on failure.
 * reference: circuit.h:22, api.cpp:7-19, gpu_index.cpp:50-141 */
circuit_index_t circuit_load_index(const char* filepath, int device_id);

/* Host query [dim] -> host out_scores[k] (descending), out_ids[k] (original ids).
 * Blocking.  From the second call with the same k (and path) the search replays a
 * CUDA graph: the kernels read the query from, and write the results into, the
 * handle's mapped pinned staging block (no copy-engine operation), and the call
 * returns as soon as the final kernel has written them -- it polls a completion
 * word in that block for up to 200 us, then waits on the stream -- so it needs no
 * spin scheduling flag for low latency.
 * reference: circuit.h:25-32, gpu_index.cpp:242-330 */
int circuit_search(circuit_index_t index, const float* query, int k, float* out_scores, int* out_ids,
                   circuit_trace_t* trace);

/* Device query -> device outputs.  Blocking: returns once the results are in the
 * caller's buffers (the first calls synchronise the handle's stream; graph replays
 * watch the completion word as above, so the kernel may still be retiring, and later
 * work on the handle is ordered after it).
 * Graph replay as above when the query is 16-byte aligned, the outputs 4-byte
 * aligned and all three are device (or managed) memory of the index's device:
 * the kernels then read the query from, and write scores / ids to, the caller's
 * buffers directly.  Other pointers take copies, which report bad ones as errors.
 * reference: circuit.h:36-43, gpu_index.cpp:333-386 */
int circuit_search_device(circuit_index_t index, const float* dev_query, int k, float* dev_out_scores,
                          int* dev_out_ids, circuit_trace_t* trace);

/* Free device memory, the mapping and the handle.  reference: circuit.h:46, api.cpp:47-51 */
void circuit_destroy_index(circuit_index_t index);

/* ------------------------------------------------------------------ extensions */

/* Description of the last error on this thread ("" if none). */
const char* circuit_last_error(void);
int circuit_abi_version(void);
/* Diagnostic: runs, on `device_id`, one kernel whose mbarrier wait is never
 * satisfied, through the same bounded wait every search kernel uses (2 s of
 * %globaltimer).  The wait gives up, the kernel records its error bit and
 * returns; *out_error_bits receives the bits (1 = a "full" wait timed out).
 * Blocking; the context stays usable.  No reference counterpart. */
int circuit_selftest_wait_timeout(int device_id, int* out_error_bits);
/* Diagnostic for the batched path's error reporting: runs the same
 * never-satisfied bounded wait (2 s) with the handle's batch workspace as its
 * error target, exactly as a k_batch_scan wait that gave up would leave it.
 * Afterwards circuit_batch_overflow returns CIRCUIT_ERR_TIMEOUT; the next
 * batched search clears the bits and runs normally.  Blocking.  No reference
 * counterpart. */
int circuit_selftest_batch_wait_timeout(circuit_index_t index, int* out_error_bits);

/* Wrap index arrays that already live on `device_id` (borrowed: the caller keeps
 * them alive and unmodified until circuit_destroy_index).  Shapes as in the
 * .circuit format: root_centers [R,D], root_radii [R], bases [R,D,rank],
 * child_intervals_l/u [C,rank], child_radii [C], child_parent_ids [C],
 * leaf_offsets [C], leaf_sizes [C], leaf_vectors [N,D], original_ids [N].
 * The small int arrays are read back once to build the per-root child lists.
 * Backs the Python CircuitIndex (reference circuit_rag/hierarchy/build.py:7-49). */
circuit_index_t circuit_index_from_device(int device_id, int dim, int rank, int num_roots, int num_total_children,
                                          int64_t n, const float* root_centers, const float* root_radii,
                                          const float* bases, const float* child_intervals_l,
                                          const float* child_intervals_u, const float* child_radii,
                                          const int* child_parent_ids, const int* leaf_offsets,
                                          const int* leaf_sizes, const float* leaf_vectors,
                                          const int* original_ids);

/* info[0..7] = dim, rank, num_roots, num_total_children, N, device, scan CTAs, max k */
int circuit_index_info(circuit_index_t index, int64_t* info);

/* Asynchronous single-query search on `stream` (a cudaStream_t; NULL = the
 * legacy default stream, as in the CUDA runtime).  Routes to the flat scan when N < min_hierarchy_n
 * (reference circuit_rag/search.py:55-57), else the hierarchical pipeline.
 * dev_out_rows (optional, int64 [k]) receives leaf-row positions.
 * ev_scan_begin / ev_scan_end (optional cudaEvent_t) are recorded on `stream`
 * around the dominant leaf-scan kernel.  No host synchronisation. */
int circuit_search_async(circuit_index_t index, const float* dev_query, int k, int64_t min_hierarchy_n,
                         float* dev_out_scores, int* dev_out_ids, int64_t* dev_out_rows, void* stream,
                         void* ev_scan_begin, void* ev_scan_end);

/* Statistics of the last search on this handle (synchronises the stream it ran on). */
int circuit_last_trace(circuit_index_t index, circuit_trace_ex_t* out);

/* Non-blocking trace capture: enqueue on `stream` a copy of the last search's
 * CIRCUIT_TRACE_SNAPSHOT_BYTES of device statistics into `dst` (device memory
 * or pinned host memory).  Once those bytes are on the host,
 * circuit_trace_decode turns them into a circuit_trace_ex_t (path: 0 flat,
 * 1 hierarchical).
 * Lets a caller keep per-query traces without a host sync per query. */
#define CIRCUIT_TRACE_SNAPSHOT_BYTES 96
int circuit_trace_snapshot_async(circuit_index_t index, void* dst, void* stream);
int circuit_trace_decode(circuit_index_t index, const void* snapshot, int path, circuit_trace_ex_t* out);

/* The hierarchical search in two phases, for a corpus sharded over several
 * GPUs (no reference counterpart).  circuit_search_seed_async resets the
 * handle's search state, scans the roots, scores an evenly spaced sample of
 * the best root's rows (max(4k, 128) of them, at most 1,024) and writes this
 * shard's seed threshold (k-th best sampled score, -inf if fewer than k rows
 * were sampled) to dev_threshold_out[0] (float, device).
 * The caller may replace it by the maximum over all shards (e.g. an NCCL
 * all-reduce MAX): each shard's value is the k-th best of k real rows, so the
 * maximum never exceeds the global k-th best score.  circuit_search_finish_async
 * then prunes with max(own seed, dev_threshold_in[0]) (dev_threshold_in may be
 * NULL) and writes this shard's top-k (empty slots -inf / -1 when fewer than k
 * rows reach the threshold).  Both run on `stream`, in this order, with the
 * same query and k and no other search on the handle in between. */
int circuit_search_seed_async(circuit_index_t index, const float* dev_query, int k, float* dev_threshold_out,
                              void* stream);
int circuit_search_finish_async(circuit_index_t index, const float* dev_query, int k, const float* dev_threshold_in,
                                float* dev_out_scores, int* dev_out_ids, int64_t* dev_out_rows, void* stream,
                                void* ev_scan_begin, void* ev_scan_end);

/* Batched exact top-k on the tensor cores (no reference counterpart: the
 * reference searches one query at a time).  dev_queries [num_queries, dim]
 * (device, 16-byte aligned) -> dev_out_scores / dev_out_ids [num_queries, k]
 * (original ids, scores descending).  One tf32 tcgen05 pass over all leaf rows
 * selects candidates within a rigorous error band of each query's running
 * k-th best; the candidates are rescored exactly in fp32, so results equal
 * the single-query search's.  Limits: dim <= 2048 with dim % 4 == 0,
 * 1 <= k <= 256 (CIRCUIT_ERR_UNSUPPORTED otherwise).
 * A query with more candidate rows inside the band than the batch's pool
 * holds (16,384 per query for a 4,096-query batch, up to 65,536 for smaller
 * batches; e.g. tens of thousands of near-identical rows) gets id -2 in its
 * first slot;
 * circuit_batch_overflow counts them and circuit_search_batch answers them
 * with the single-query search.
 * Asynchronous on `stream`; the first call per handle allocates its batch
 * workspace and synchronises once.  ev_scan_begin / ev_scan_end (cudaEvent_t,
 * optional) are recorded around the tensor-core scan kernel. */
int circuit_search_batch_async(circuit_index_t index, const float* dev_queries, int num_queries, int k,
                               float* dev_out_scores, int* dev_out_ids, void* stream, void* ev_scan_begin,
                               void* ev_scan_end);
/* Queries of the last batch whose candidate list overflowed (synchronises its
 * stream).  Returns CIRCUIT_ERR_TIMEOUT (with *out_count still written) when a
 * bounded device-side wait of that batch gave up, i.e. its results are
 * incomplete; every batch starts with the error bits cleared.  The blocking
 * calls below return the same code for such a batch. */
int circuit_batch_overflow(circuit_index_t index, int* out_count);
/* Blocking host-buffer variant of circuit_search_batch_async (host_scores / host_ids [num_queries, k]). */
int circuit_search_batch(circuit_index_t index, const float* host_queries, int num_queries, int k, float* host_scores,
                         int* host_ids);
/* Blocking device-buffer variant (runs on and synchronises the handle's own
 * stream, so the caller makes sure the queries are ready, e.g. by synchronising
 * the stream that wrote them): like circuit_search_batch_async, and rows whose
 * candidate list overflowed are answered in place by the single-query search,
 * so no id -2 remains. */
int circuit_search_batch_device(circuit_index_t index, const float* dev_queries, int num_queries, int k,
                                float* dev_out_scores, int* dev_out_ids);

/* Exact top-k of corpus[n, dim] . query that allocates no device memory (no
 * counterpart in the reference).  For callers that cannot call cudaMalloc: an
 * engine plugin whose host framework owns all device memory, a serving loop
 * that must not touch the allocator after start-up.  The caller passes the
 * device corpus (row-major float32, 16-byte aligned, dim % 4 == 0), the query
 * and the outputs (scores[k] descending, ids[k] = row numbers); the scan's
 * scratch is a fixed 256 KiB array inside the library's device image, held by
 * every GPU that loads the library until the process exits.  Limits: k <= 128,
 * n < 2^31, dim <= 2048 (larger values return CIRCUIT_ERR_ARG /
 * CIRCUIT_ERR_UNSUPPORTED with a message).  The first call on a device looks up
 * that array's device address with the device current; make that first call
 * before any stream capture.  All calls share the array: calls that overlap on
 * the GPU race and must be serialised by the caller.  Asynchronous on `stream`
 * (NULL = legacy default stream). */
int circuit_flat_search_noalloc(const float* dev_corpus, int64_t n, int dim, const float* dev_query, int k,
                                float* dev_out_scores, int* dev_out_ids, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CIRCUIT_H */
