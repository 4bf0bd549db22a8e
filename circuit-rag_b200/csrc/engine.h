// Internal (non-ABI) declarations shared by the kernels (.cu) and the host
// library (index.cpp / ops).  Nothing here crosses the C ABI: include/circuit.h
// is the only public header.
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>

namespace cb {

// Dynamic shared-memory opt-in of one kernel, raised on demand.  The attribute
// set by cudaFuncSetAttribute belongs to the current device's context, so the
// size already configured is remembered per device: a process that searches on
// several GPUs configures each one before its first launch there.  Thread-safe
// (the slow path takes a mutex; the size recorded for a device only grows).
class SmemOptIn {
 public:
  static constexpr int kMaxDevices = 64;
  cudaError_t ensure(const void* func, int bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices)
      return cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (set_[dev].load(std::memory_order_acquire) >= bytes) return cudaSuccess;
    std::lock_guard<std::mutex> lock(mu_);
    if (set_[dev].load(std::memory_order_relaxed) >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    // all of the unified L1 as shared memory: kernels of one search alternate on
    // the SMs, and a different split would have to be set up between them
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e == cudaSuccess) set_[dev].store(bytes, std::memory_order_release);
    return e;
  }

 private:
  std::mutex mu_;
  std::atomic<int> set_[kMaxDevices] = {};
};

constexpr int KMAX = 256;          // largest k a search accepts
// Seed sample of a root: blocks of up to SEED_BLOCK consecutive rows starting at
// evenly spaced positions among the root's rows (the first SEED_SAMPLE_MAX
// children in leaf order), `want` rows in all: min(rows, max(4k, 128), 1024).
// For k <= 32 (want = min(rows, 128)) the blocks are precomputed per root at
// set-up: entry 0 = {blocks, rows sampled, 0, 0}, entries 1.. = {leaf row,
// length, position in the sample, 0}.
constexpr int SEED_SAMPLE_MAX = 1024;
constexpr int SEED_BLOCK = 16;
constexpr int SEED_TAB_W = 1 + 128 / SEED_BLOCK;
constexpr int MAX_RANK = 64;       // largest rank r of a parent basis
constexpr int MAX_DIM = 2048;      // largest vector dimension D (D % 4 == 0)
constexpr int SCAN_CONSUMER_WARPS = 8;
constexpr int SCAN_THREADS = (SCAN_CONSUMER_WARPS + 1) * 32;  // + one TMA producer warp
constexpr int BOUNDS_WARPS = 4;
constexpr int ROOT_SCAN_WARPS = 8;

// Per-query control block, zeroed at the start of every search (by the search
// prologue kernel, or by the caller of launch_flat_scan).
struct SearchCtrl {
  unsigned long long best_packed;  // argmax root: prio<<62 | key<<30 | (2^30-1-root)
  unsigned long long seed_packed;  // rows scored by the seed sample
  unsigned long long main_packed;  // children kept by the seed threshold << 32 | their rows (atomicAdd)
  uint32_t k1_done;                // last-CTA tickets (root scan, main scan)
  uint32_t pad0;
  uint32_t main_done;
  uint32_t theta_key;              // running global threshold key (atomicMax)
  uint32_t seed_T_key;             // k-th best key of the seed rows (0 = none)
  uint32_t n_surv_roots;           // roots whose bound survived (seed root included)
  uint32_t n_surv_children;        // non-empty children kept by the seed threshold
  float qn2;                       // fl(sum q_i^2)
  int best_root;
  int error;                       // cb::ERR_* bits
  uint32_t call_seq;               // blocking calls: the call's sequence number (see HostIO)
  uint32_t chunk_next;             // a long flat scan's next chunk to claim
  uint32_t epoch;                  // this search's number (tags the bounds it computes; never 0)
  uint32_t rows_streamed;          // leaf rows the main scan read (atomicAdd per CTA)
  uint32_t pad[4];
};
constexpr int CTRL_SEQ_WORD = 8;   // 64-bit word of the header: call_seq (low half), chunk_next (high, zero)
constexpr int CTRL_EPOCH_WORD = 9; // epoch (low half), rows_streamed (high, zero)
constexpr size_t CTRL_RESET_BYTES = 96;
static_assert(sizeof(SearchCtrl) == CTRL_RESET_BYTES, "ctrl layout");

// Per-search words of the hierarchical main scan and the bounds kernel that
// take many atomics while both run, each group on its own 128-byte line, away
// from the control header (whose running threshold every consumer warp
// raises); cleared by the search prologue.
struct alignas(128) ScanSync {
  // chunks claimed in order (low half); the bounds kernel adds 1 to the high
  // half once its live-chunk list is complete
  unsigned long long chunk_claims;
  uint32_t list_next;              // the next live-list entry to claim
  uint32_t pad_a[29];
  uint32_t n_live;                 // chunks in the live list
  uint32_t bounds_done;            // the bounds kernel's last-CTA ticket
  uint32_t pad_b[30];
};
static_assert(sizeof(ScanSync) == 256, "sync layout");

// Read-only device view of one index (all pointers are device pointers).
struct IndexView {
  const float* root_centers;    // [R, D]
  const float* root_radii;      // [R]
  const float* bases;           // [R, D, r]  (r innermost)
  const float* child_l;         // [C, r]
  const float* child_u;         // [C, r]
  const float* child_radii;     // [C]
  const int* child_parent;      // [C]
  const int* leaf_offsets;      // [C]
  const int* leaf_sizes;        // [C]
  const float* leaf;            // [N, D]
  const int* original_ids;      // [N]
  // derived once per index by prepare()
  const int* root_child_ptr;    // [R+1]  CSR over non-empty children, grouped by parent
  const int* root_child_list;   // [nnz children]
  const int2* root_child_span;  // [nnz] per CSR entry: {leaf offset, first row within its root's rows}
  const int4* seed_tab;         // [R * SEED_TAB_W] the seed sample of each root for k <= 32 (see below)
  const int4* all_ranges;       // [nnz] every CSR entry in order: {first virtual row, leaf row begin, end, child}
  const unsigned long long* all_packed;  // [1] nnz << 32 | N
  int all_nnz;                  // entries of all_ranges
  const int* root_rows;         // [R]  leaf rows under each root
  const double* root_cn;        // [R]  upper bound of ||c_r||
  const double* root_defect;    // [R]  upper bound of ||V_r^T V_r - I||_2
  int D, D4, rank, R, C, N;
};

// Device workspace owned by one index handle (one in-flight search at a time).
struct Workspace {
  SearchCtrl* ctrl;
  ScanSync* sync;
  uint32_t* epoch_counter;           // [1] the last search's epoch (not cleared between searches)
  int4* flat_range;                  // [1] = {0, 0, N, -1}
  unsigned long long* flat_packed;   // [1] = 1<<32 | N
  float* ub_root;                    // [R] rigorous root bounds (rounded up to float)
  float* ub_child;                   // [C] rigorous child bounds
  // [nnz] per CSR entry: epoch << 32 | key of min(root bound, child bound);
  // an entry whose epoch is not the running search's is not known yet
  unsigned long long* ub_tagged;
  const int* chunk_first_range;      // [n_chunks] the all_ranges entry holding each chunk's first row
  int chunk_rows;                    // rows per chunk of the hierarchical main scan
  int n_chunks;
  uint32_t* chunk_mark;              // [n_chunks] epoch of the last search that listed the chunk as live
  int* live_list;                    // [n_chunks] the live chunks of this search (ctrl->n_live of them)
  uint32_t* chunk_taken;             // [n_chunks] epoch of the last search that streamed the chunk
  unsigned long long* cta_lists;     // [scan_grid * KMAX]
  int scan_grid;
};

// Endpoints of a blocking search replayed from a CUDA graph.  All four point
// into mapped pinned host memory except out_indirect (device memory).  The
// start of the search copies the query from q_host (host-buffer calls) or from
// the device pointer slots[0] (device-buffer calls) and clears the control
// header in one kernel; the final merge writes scores / ids to the launch's
// out_scores / out_ids, or, with slots, to the device pointers slots[1] /
// slots[2] (staged in out_indirect by the start kernel), and a copy of the
// control header to ctrl_out.  No copy-engine operation remains in the graph.
//
// Completion: the host writes the call's sequence number to seq_in before the
// launch; the start kernel copies it into the control header, and the final
// merge, after its results and the header copy, writes it to done_out (mapped
// host memory, system-scope fence first).  The blocking call returns once it
// sees its number there, without waiting for the stream's completion report.
struct HostIO {
  const float* q_host;               // [D] or null
  void* const* slots;                // {query, scores, ids} device pointers, or null
  void** out_indirect;               // [2]
  SearchCtrl* ctrl_out;              // receives the first CTRL_RESET_BYTES
  const uint32_t* seq_in;            // mapped host word: this call's sequence number
  uint32_t* done_out;                // mapped host word: set to it when the results are out
};

// ---- launchers (search_kernels.cu); all asynchronous on `stream` ----
cudaError_t launch_prepare_roots(const IndexView& ix, double* root_cn, double* root_defect, cudaStream_t stream);

// One single-query search.  hierarchical != 0 runs prologue -> root scan (with
// the seed sample) -> bounds -> main scan, the main scan streaming beside the
// bounds kernel and skipping each child once its bound is known and below the
// running threshold; otherwise prologue -> one flat scan over all rows.
// Outputs k results sorted by (score desc, row asc).  ev_scan0/1 (may be null)
// are recorded around the main (dominant) scan kernel.
cudaError_t launch_search(const IndexView& ix, const Workspace& ws, const float* q, int k, int hierarchical,
                          float* out_scores, int* out_ids, long long* out_rows, cudaStream_t stream,
                          cudaEvent_t ev_scan0, cudaEvent_t ev_scan1, const HostIO* io = nullptr);
// The hierarchical search in two phases, so that shards can exchange their seed
// thresholds in between: seed = reset + root scan with the seed sample (writes
// the k-th best sampled score to T_export, -inf if fewer than k rows were
// sampled); finish = bounds + main scan with threshold max(own seed, *T_ext).
cudaError_t launch_search_seed(const IndexView& ix, const Workspace& ws, const float* q, int k, float* T_export,
                               cudaStream_t stream, const HostIO* io = nullptr);
// A running threshold shared by the shards searching one query: this shard's
// 64-bit word and a device array of the peers' words (in their GPUs' memory),
// each holding tag << 32 | threshold key; the main scan raises them all and
// prunes with the largest key carrying this query's tag.
struct SharedThreshold {
  unsigned long long* local;
  unsigned long long* const* peers;
  int n_peers;
  uint32_t tag;
};
cudaError_t launch_search_finish(const IndexView& ix, const Workspace& ws, const float* q, int k, const float* T_ext,
                                 float* out_scores, int* out_ids, long long* out_rows, cudaStream_t stream,
                                 cudaEvent_t ev_scan0, cudaEvent_t ev_scan1, const HostIO* io = nullptr,
                                 const SharedThreshold* shared = nullptr);

// Flat exact top-k of leaf[0..N) . q with caller-provided scratch: ctrl (its
// first CTRL_RESET_BYTES zeroed by the caller), range = {0, 0, N, -1},
// packed = 1 << 32 | N, cta_lists >= (grid + 1) * k entries.  Output ids are
// row numbers.
cudaError_t launch_flat_scan(const float* leaf, int D, int N, const float* q, int k, int grid, SearchCtrl* ctrl,
                             const int4* range, const unsigned long long* packed, unsigned long long* cta_lists,
                             float* out_scores, int* out_ids, cudaStream_t stream);

// ---- batched search (batch_kernels.cu) ----
constexpr int BATCH_MAX_DIM = 2048;  // the rescoring keeps the query in registers (16 float4 per lane)
constexpr int BATCH_MAX_K = KMAX;  // any k of the single-query search
constexpr int BATCH_CAND_CAP = 16384;  // candidate entries per query of a full-capacity batch
constexpr int BATCH_CAND_MAX = 65536;  // per query when the batch is smaller than the workspace
// threshold slots per query: 4k for k > 32 (rows r -> slot r mod 4k, threshold
// = k-th largest slot), rounded up to whole warps of 32; k for k <= 32
constexpr int batch_slot_count(int k) { return k > 32 ? ((4 * k + 31) / 32) * 32 : k; }
constexpr int BATCH_MAX_SLOTS = batch_slot_count(BATCH_MAX_K);

struct BatchWorkspace {
  uint32_t* theta = nullptr;      // [capacity] running k-th best keys
  uint32_t* slots = nullptr;      // [capacity * BATCH_MAX_SLOTS] per-query threshold slots
  int* unit_counter = nullptr;    // [2] work-unit counters (main pass, threshold pass)
  int* cand_count = nullptr;      // [capacity]
  unsigned long long* cand = nullptr;  // [cand_entries] tf32 key << 32 | row
  int64_t cand_entries = 0;
  int* overflow = nullptr;        // queries whose candidate list overflowed
  int* err = nullptr;
  float* queries = nullptr;       // [capacity * D] staging for host queries
  float* qband = nullptr;         // [capacity] per-query error band (2 eps, padded)
  float* out_scores = nullptr;    // [capacity * KMAX] host-call staging
  int* out_ids = nullptr;
  int cap = BATCH_CAND_CAP;
  int capacity = 0;
  float xmax = 0.f;               // upper bound of max ||x|| over the leaf rows
  int sms = 0;
  alignas(64) unsigned char tmap[128];  // CUtensorMap of leaf_vectors, boxes of 128 rows x 32 columns
  alignas(64) unsigned char smap[128];  // the same over evenly spaced rows (threshold pass)
  int sample_rows = 0;                  // rows of smap (0: no threshold pass)
};

bool make_leaf_tensor_map(const float* leaf, int N, int D, void* out_map);
int sample_rows_for(int N);
bool make_sample_tensor_map(const float* leaf, int N, int D, void* out_map);
cudaError_t launch_max_row_norm(const float* leaf, int N, int D, unsigned int* out_key, int sms, cudaStream_t st);
// queries [B, D] (device) -> out_scores / out_ids [B, k], original ids, (score desc, row asc).
cudaError_t launch_batch_search(const IndexView& ix, const BatchWorkspace& bw, const float* Q, int B, int k,
                                float* out_scores, int* out_ids, cudaStream_t st, cudaEvent_t ev_scan_begin,
                                cudaEvent_t ev_scan_end);

int scan_smem_bytes(int D);
// Rows per chunk of the hierarchical main scan over N rows of dimension D on
// `grid` CTAs: a multiple of the rows of one ring stage (at least 4 stages),
// about 48 chunks per CTA.
int overlap_chunk_rows(int N, int D, int grid);
// One kernel whose mbarrier wait nothing satisfies, run through the bounded
// wait every search kernel uses: after the limit it or-s ERR_TIMEOUT_FULL into
// *err and returns (merge_kernels.cu).
cudaError_t launch_selftest_wait(int* err, cudaStream_t stream);
int sm_count(int device);

}  // namespace cb
