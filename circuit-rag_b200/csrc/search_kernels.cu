// Single-query exact top-k search kernels for B200 (sm_100a).
//
// Pipeline for one query (all on one stream, no host synchronisation):
//   k_search_prologue  clears the control header and numbers the search (its
//                 epoch); in graph-replayed blocking calls it also stages the
//                 query
//   k_root_scan   warp per root: q.c_r for every root, ||q||^2, argmax root
//                 (the seed root); its last CTA scores an evenly spaced
//                 sample of the seed root's rows (bulk copies into shared
//                 memory, the leaf scan's exact arithmetic) and publishes
//                 T = k-th best sampled score on the device.
//                                               (reference: search.py:26-41,
//                                                 root_bounds.cu:31-54)
//   k_bounds      warp per root: rigorous root bound, rank-r projection of q
//                 (basis staged in shared memory by TMA), rigorous child box
//                 bounds, published per child tagged with the search's epoch;
//                 then (after the seed) the survivor counts of the trace.
//                                               (reference: parent_projection.cu:125-178,
//                                                 child_bounds.cu:11-83)
//   k_scan<final> streams the leaves child by child (TMA bulk copies into a
//                 3..8-stage shared-memory ring, one producer warp, eight
//                 consumer warps), fused top-k; its last CTA merges all lists
//                 and writes scores / original ids.  It runs BESIDE the bounds
//                 kernel: a child whose bound is already published and below
//                 the running threshold is skipped, any other child is
//                 streamed, so the scan never waits for the bounds (the
//                 reference scores only the survivors, after host syncs).
//                                               (reference: dense_score.cu:116-164,
//                                                 topk.cu:56-170, search.py:63-84)
// The flat path (small corpora) is the final scan over one range [0, N).
#include <cmath>
#include <cstdio>
#include <type_traits>
#include <utility>

#include "common.cuh"
#include "engine.h"
#include "topk.cuh"

namespace cb {

// ============================================================ rounding model
// u = 2^-24 (fp32 unit roundoff); gamma_n = n u / (1 - n u) bounds the error of
// any fp32 dot product of length n, in any summation order, with or without FMA
// (Higham, Accuracy and Stability of Numerical Algorithms, 2nd ed., sec. 3.1).
__device__ __forceinline__ double gamma_n(int n) {
  const double u = 5.9604644775390625e-08;
  return n * u / (1.0 - n * u);
}

// ============================================================ leaf scan kernel
struct ScanParams {
  const float* leaf;                          // [N, D]
  const float* q;                             // [D]
  const int4* ranges;                         // {vbegin, row_begin, row_end, child}
  const unsigned long long* packed_counts;    // n_ranges << 32 | n_rows (read when packed_value is 0)
  unsigned long long packed_value;            // the same, when the host knows it
  uint32_t* theta_key;                        // running global threshold (atomicMax)
  unsigned long long* cta_lists;              // [(gridDim.x + 1) * k]
  uint32_t* done;                             // last-CTA ticket
  int* err;
  int D4;
  int row_bytes;
  int k;
  int stages;
  int min_rows;                               // rows per CTA below which fewer CTAs take part
  uint32_t* chunk_counter;                    // long streams: chunks claimed so far (zeroed per search)
  float* out_scores;
  int* out_ids;
  long long* out_rows;
  const int* original_ids;
  void* const* out_indirect;                  // final: {scores, ids} device pointers replacing out_scores / out_ids
  const unsigned long long* ctrl_hdr;         // final: control header, copied to ctrl_out after the merge
  unsigned long long* ctrl_out;               // (mapped host memory; null = no copy)
  const uint32_t* call_seq;                   // blocking calls: the call's number in the control header
  uint32_t* done_out;                         // mapped host word that receives it when the results are out
  // hierarchical scans (all null / 0 for a flat scan)
  const unsigned long long* ub_tagged;        // per range: epoch << 32 | bound key (see Workspace)
  const uint32_t* epoch;                      // this search's epoch (control header)
  const int* chunk_first_range;               // per chunk: the range holding its first row
  uint32_t chunk_rows;                        // rows per chunk, with chunk_first_range
  unsigned long long* chunk_claims;           // in-order claims; high half set once the live list is complete
  const int* live_list;                       // chunks listed by the bounds kernel
  const uint32_t* n_live;
  uint32_t* list_next;
  uint32_t* chunk_taken;                      // per chunk: epoch of the search that streams it
  // sharded search: a running threshold shared by the shards searching the same
  // query, as words tag << 32 | key (key of a k-th best score of k real rows of
  // some shard); this shard reads xth_local and raises it and every peer's word
  unsigned long long* xth_local;              // (null: not shared)
  unsigned long long* const* xth_peers;       // device array of n_peers pointers (peer GPUs' memory)
  int n_peers;
  uint32_t xth_tag;                           // the query's number, the same on every shard
  const float* T_ext;                         // a threshold from outside the index (or null)
  uint32_t* rows_streamed;                    // rows read, summed over CTAs (or null)
  int overlapped;                             // launched beside the bounds kernel (no wait before streaming)
};

template <int VPL> struct ScanShape {
  static constexpr int RPW = VPL <= 4 ? 4 : (VPL <= 8 ? 2 : 1);       // rows per consumer warp per stage
  static constexpr int ROWS = SCAN_CONSUMER_WARPS * RPW;               // rows per stage
};
template <int KCAP> struct TopkShape {
  static constexpr int BUF = 64;
  static constexpr int SORTN = (KCAP + BUF <= 128) ? 128 : ((KCAP + BUF <= 256) ? 256 : 512);
};
constexpr int MAX_STAGES = 8;

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct ScanLayout {
  size_t stage_bytes, stages_off, bars_off, rows_off, n_off, side_off, topk_off, sel_off, scratch_off, total;
};
__host__ __device__ inline ScanLayout scan_layout(int rows_per_stage, int row_bytes, int stages, int sortn,
                                                  int kcap) {
  ScanLayout L;
  L.stage_bytes = align_up((size_t)rows_per_stage * row_bytes, 128);
  L.stages_off = 0;
  L.bars_off = align_up(L.stages_off + stages * L.stage_bytes, 128);
  L.rows_off = L.bars_off + 2 * MAX_STAGES * sizeof(uint64_t);           // runs: [stage][32] int2
  L.n_off = L.rows_off + (size_t)MAX_STAGES * 32 * sizeof(int2);          // rows, runs per stage
  L.side_off = align_up(L.n_off + 2 * MAX_STAGES * sizeof(int), 16);   // [stage] 16 B: threshold snapshot
  L.topk_off = align_up(L.side_off + (size_t)MAX_STAGES * 16, 128);
  L.sel_off = L.topk_off + (size_t)SCAN_CONSUMER_WARPS * sortn * 8;
  L.scratch_off = align_up(L.sel_off + (size_t)kcap * 8, 128);
  L.total = align_up(L.scratch_off + sizeof(SelectScratch) + 16, 128);
  return L;
}

// Merges whose survivors number at most this many rank them directly.
constexpr int RANK_CAP = 256;
// The final merge ranks up to this many candidates directly.
constexpr int FINAL_RANK_CAP = 512;
// Streams of at least SCAN_DYN_CHUNKS chunks of SCAN_DYN_MIN_STAGES stages per
// CTA are taken in claimed chunks (about SCAN_DYN_CHUNKS per CTA) instead of
// equal slices.
constexpr int SCAN_DYN_CHUNKS = 48;
constexpr int SCAN_DYN_MIN_STAGES = 8;

// A new running threshold key of this shard, for the other shards searching the
// same query (fire-and-forget atomics, over NVLink for a peer's word).
__device__ __forceinline__ void share_threshold(const ScanParams& P, uint32_t key) {
  if (!P.xth_local) return;
  const unsigned long long w = ((unsigned long long)P.xth_tag << 32) | key;
  atomicMax(P.xth_local, w);
  for (int i = 0; i < P.n_peers; ++i) atomicMax(P.xth_peers[i], w);
}

template <int VPL, int KCAP>
__global__ void __launch_bounds__(SCAN_THREADS, 1) k_scan(ScanParams P) {
  using SS = ScanShape<VPL>;
  using TS = TopkShape<KCAP>;
  constexpr int RPW = SS::RPW, ROWS = SS::ROWS, SORTN = TS::SORTN, BUF = TS::BUF;
  extern __shared__ __align__(128) unsigned char smem[];
  const ScanLayout L = scan_layout(ROWS, P.row_bytes, P.stages, SORTN, KCAP);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars_off);
  uint64_t* empty = full + MAX_STAGES;
  // A stage holds up to ROWS rows made of runs of consecutive leaf rows:
  // stage_runs[stage][i] = {first slot, first row}, stage_n[stage] = rows
  // (-1 = end of stream), stage_nr[stage] = runs.
  int2* stage_runs = reinterpret_cast<int2*>(smem + L.rows_off);
  int* stage_n = reinterpret_cast<int*>(smem + L.n_off);
  int* stage_nr = stage_n + MAX_STAGES;
  unsigned long long* topk_all = reinterpret_cast<unsigned long long*>(smem + L.topk_off);
  unsigned long long* sel = reinterpret_cast<unsigned long long*>(smem + L.sel_off);
  SelectScratch* scratch = reinterpret_cast<SelectScratch*>(smem + L.scratch_off);
  // Each stage's bulk copies also bring the 16-byte line holding theta_key, on
  // the same barrier: consumers refresh the shared threshold from shared memory
  // instead of waiting on an L2 round trip per stage.
  const uint32_t* side = reinterpret_cast<const uint32_t*>(smem + L.side_off);
  const int theta_word = (int)(((uintptr_t)P.theta_key & 15u) >> 2);
  __shared__ int s_is_last, s_err;
  __shared__ unsigned long long s_pc;
  __shared__ uint32_t s_theta, s_rank_count, s_fin_count, s_text, s_epoch, s_theta0;
  __shared__ uint32_t s_warp_theta[SCAN_CONSUMER_WARPS];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int STAGES = P.stages;
  const int k = P.k;

  for (int i = tid; i < SCAN_CONSUMER_WARPS * SORTN; i += blockDim.x) topk_all[i] = 0ull;
  // A flat scan is a programmatic dependent of the search prologue, which
  // clears its control words: it waits here.  A hierarchical scan is one of the
  // bounds kernel, and everything it reads before its last CTA (the static
  // range list, the query, the control words) was written by kernels that had
  // completed before the bounds kernel was launched (the root scan waits for
  // the prologue before it lets the bounds kernel start); the bounds it reads
  // while they are being written carry the epoch, so it does not wait.
  if (!P.overlapped) griddep_wait();
  // the producer's first chunk is chunk blockIdx.x (see below): its table entry
  // and its range windows are requested before the shared-memory set-up (the
  // windows' bounds are decoded once the epoch is known)
  int first_range = -1;
  int4 fw0 = make_int4(0, 0, 0, 0), fw1 = fw0;
  unsigned long long ft0 = 0ull, ft1 = 0ull;
  if (warp == SCAN_CONSUMER_WARPS && P.chunk_first_range && P.packed_value &&
      blockIdx.x < ((uint32_t)P.packed_value + P.chunk_rows - 1) / P.chunk_rows) {
    first_range = __ldcg(P.chunk_first_range + blockIdx.x);
    const int nr = (int)(P.packed_value >> 32), b0 = (first_range & ~31) + lane, b1 = b0 + 32;
    if (first_range >= 0 && first_range < nr) {
      if (b0 < nr) {
        fw0 = __ldcg(&P.ranges[b0]);
        if (P.ub_tagged) ft0 = __ldcg(&P.ub_tagged[b0]);
      }
      if (b1 < nr) {
        fw1 = __ldcg(&P.ranges[b1]);
        if (P.ub_tagged) ft1 = __ldcg(&P.ub_tagged[b1]);
      }
    }
  }
  if (tid == 0) {
    // (independent loads, in flight together)
    const float te = P.T_ext ? __ldcg(P.T_ext) : -INFINITY;
    const uint32_t ep = P.epoch ? __ldcg(P.epoch) : 0u;
    const uint32_t th0 = P.ub_tagged ? __ldcg(P.theta_key) : 0u;  // the running threshold so far
    const unsigned long long pc = P.packed_value ? P.packed_value : __ldcg(P.packed_counts);
    s_err = 0;
    s_fin_count = 0;
    const uint32_t tx = te > -INFINITY ? f2key(te) : 0u;
    s_text = tx;
    if (tx && blockIdx.x == 0) atomicMax(P.theta_key, tx);
    s_epoch = ep;
    s_theta0 = max(th0, tx);
    s_pc = pc;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], SCAN_CONSUMER_WARPS);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // Small streams use fewer CTAs (at least min_rows rows each): the per-CTA and
  // grid merges then handle fewer lists, and each warp sees enough rows for its
  // k-th best to raise the shared threshold.  The others leave before any copy.
  const uint32_t n_ranges = (uint32_t)(s_pc >> 32), n_rows = (uint32_t)s_pc;
  const uint32_t G = max(1u, min((uint32_t)gridDim.x, (n_rows + (uint32_t)P.min_rows - 1) / (uint32_t)P.min_rows));
  if (blockIdx.x >= G) return;

  if (warp == SCAN_CONSUMER_WARPS) {
    // ------------------------------------------------------------ producer
    // Work distribution.  A short flat stream is split into G equal slices.  A
    // long one, and every hierarchical one, is cut into chunks of chunk_rows
    // virtual rows that the CTAs claim from a counter in the control block:
    // SMs do not stream at the same rate (measured at 100M rows, equal slices
    // finished up to 17 % apart), and a hierarchical scan's CTAs start at
    // different times (an SM running a root-scan or bounds CTA takes its scan
    // CTA later), so the CTAs that stream more take more chunks and all finish
    // within about a chunk of each other.
    // CTA b starts with chunk b; claim c stands for chunk G + c.
    // Hierarchical scans claim chunks in order while the bounds are being
    // computed.  The bounds kernel marks the chunks that hold a child whose
    // bound is not below the seed threshold, lists the marked chunks not taken
    // yet and then adds 1 to the high half of the claim word: a CTA whose claim
    // returns a non-zero high half takes its chunks from the list from then on,
    // so dead chunks cost nothing.  A chunk
    // can reach one CTA in order and another from the list: whoever swaps this
    // search's epoch into its taken word first streams it, so each chunk is
    // streamed once, and every listed chunk is streamed.
    const bool table = P.chunk_first_range != nullptr;
    const bool dyn = table || (P.chunk_counter != nullptr &&
                               n_rows >= G * (uint32_t)(SCAN_DYN_CHUNKS * SCAN_DYN_MIN_STAGES * ROWS));
    uint32_t chunk_rows = 0, n_chunks = 0;
    uint32_t vb = 0, ve = 0;  // the piece of the stream being streamed
    if (dyn) {
      if (table) {
        chunk_rows = P.chunk_rows;
      } else {
        const uint32_t per = n_rows / (G * (uint32_t)SCAN_DYN_CHUNKS);
        chunk_rows = max((uint32_t)(SCAN_DYN_MIN_STAGES * ROWS), (per + ROWS - 1) / ROWS * ROWS);
      }
      n_chunks = (n_rows + chunk_rows - 1) / chunk_rows;
    } else {
      vb = (uint32_t)(((unsigned long long)blockIdx.x * n_rows) / G);
      ve = (uint32_t)(((unsigned long long)(blockIdx.x + 1) * n_rows) / G);
    }
    // the range holding virtual row vv, searched from range `lo` (which starts
    // at or before vv): a 32-way search by the whole warp (ranges sorted by
    // .x), 3 L2 round trips for 4,096 ranges
    const auto locate = [&](uint32_t vv, int lo) {
      int hi = (int)n_ranges - 1;
      while (hi > lo) {
        const int step = (hi - lo + 32) >> 5;
        const int pos = lo + lane * step;
        const int4 e = pos <= hi ? __ldcg(&P.ranges[pos]) : make_int4(0x7fffffff, 0, 0, 0);
        const int j = 31 - __clz(__ballot_sync(FULL_MASK, (uint32_t)e.x <= vv));
        lo += j * step;
        hi = min(hi, lo + step - 1);
      }
      return lo;
    };
    // The whole warp walks the ranges: lane j holds entry base + j of the
    // current 32-entry window and of the next one (loaded a window ahead), so
    // moving from one child's rows to the next is a register shuffle; an L2
    // round trip happens once per 32 ranges and overlaps the stages in flight.
    // Short children (a few rows each) do not stall the stream.  Lane j
    // records and issues the stage's run j, so up to 32 bulk copies per stage
    // go out in parallel.
    // Pruning (hierarchical): each window lane also holds its range's bound key
    // when the bounds kernel has published it for this search (the epoch in the
    // same 64-bit word says so), else 0xffffffff.  A range is skipped when that
    // key is below pkey = max(external threshold, the running threshold read
    // before the piece): every row of the child then scores below a value that
    // never exceeds the final k-th best.
    const bool prune = P.ub_tagged != nullptr;
    const uint32_t epoch = s_epoch;
    const uint64_t policy = policy_evict_first();
    const void* theta_line = reinterpret_cast<const void*>((uintptr_t)P.theta_key & ~(uintptr_t)15);
    const char* leaf_bytes = reinterpret_cast<const char*>(P.leaf);
    // a window: lane j's range entry and its raw tagged bound (decoded only
    // when the window becomes current, so that loading it never stalls)
    const auto load_window = [&](int b, unsigned long long& tag) {
      const int idx = b + lane;
      const bool in = idx < (int)n_ranges;
      tag = (prune && in) ? __ldcg(&P.ub_tagged[idx]) : 0ull;
      return in ? __ldcg(&P.ranges[idx]) : make_int4(0, 0, 0, 0);
    };
    const auto decode = [&](unsigned long long t) {
      return (prune && (uint32_t)(t >> 32) == epoch) ? (uint32_t)t : 0xffffffffu;
    };
    int s = 0, base = 0;
    int4 win = make_int4(0, 0, 0, 0), win_next = win, rg = win;
    unsigned long long tag_cur = 0ull, tag_next = 0ull;
    uint32_t ubk = 0xffffffffu, rkey = 0xffffffffu, pkey = 0u;
    bool bad_range = false;
    const auto fail_range = [&]() {
      if (lane == 0) atomicOr(P.err, ERR_BAD_RANGE);
      bad_range = true;
    };
    const auto set_range = [&]() {  // rg / rkey from the windows
      rg.x = __shfl_sync(FULL_MASK, win.x, s - base);
      rg.y = __shfl_sync(FULL_MASK, win.y, s - base);
      rg.z = __shfl_sync(FULL_MASK, win.z, s - base);
      rg.w = __shfl_sync(FULL_MASK, win.w, s - base);
      rkey = __shfl_sync(FULL_MASK, ubk, s - base);
    };

    // ---- chunk claims: one claim in flight (lane 0), resolved a chunk ahead
    unsigned long long pend = 0ull;
    bool list_mode = false;
    uint32_t n_live = 0;
    const auto claim = [&]() {
      if (lane == 0) {
        if (!table) pend = atomicAdd(P.chunk_counter, 1u);
        else if (!list_mode) pend = atomicAdd(P.chunk_claims, 1ull);
        else pend = atomicAdd(P.list_next, 1u);
      }
    };
    // the chunk that the claim in flight gives (claiming again where it gives
    // none), with the following claim issued: >= 0 = that chunk (it still has to
    // be won through its taken word), -1 = none left, -2 = a live-list entry
    // requested (list_entry, read a step later)
    uint32_t list_entry = 0u;
    const auto resolve = [&]() -> int {
      for (uint32_t guard = 0; guard <= 2 * n_chunks + 2; ++guard) {
        const unsigned long long r = __shfl_sync(FULL_MASK, pend, 0);
        if (!list_mode) {
          if ((r >> 32) == 0ull) {
            const uint32_t lo = (uint32_t)r + G;
            if (lo >= n_chunks) return -1;
            claim();
            return (int)lo;
          }
          // the list is complete (the bounds kernel fenced it before the add)
          __threadfence();
          n_live = ld_volatile_u32(P.n_live);
          list_mode = true;
          claim();
          continue;
        }
        const uint32_t i = (uint32_t)r;
        if (i >= n_live || i >= n_chunks) return -1;
        list_entry = (uint32_t)__ldcg(P.live_list + i);
        claim();
        return -2;
      }
      return -1;
    };
    // the next chunk, prepared one step per issued stage: 0 = nothing yet,
    // 1 = a live-list entry requested, 2 = chunk known, its taken word swapped
    // and its first range requested, 3 = its windows and the threshold
    // requested, 4 = no chunk left; the swap is checked when the chunk is taken
    // (a lost chunk is dropped then)
    int pf = 0, nj = -1, ns = -1, pbase = 0;
    uint32_t taken_old = 0u;
    int4 pw = make_int4(0, 0, 0, 0), pw2 = pw;
    unsigned long long pt = 0ull, pt2 = 0ull;
    uint32_t pth = 0u;               // (the running threshold as read for the next chunk)
    unsigned long long pxw = 0ull;   // (the shared word as read for the next chunk)
    const auto start_chunk = [&]() {
      if (table) {
        if (lane == 0) taken_old = atomicExch(P.chunk_taken + nj, epoch);
        ns = __ldcg(P.chunk_first_range + nj);
      } else {
        ns = locate((uint32_t)nj * chunk_rows, s);
      }
      pf = 2;
    };
    const auto prefetch = [&]() {
      if (pf == 0) {
        nj = resolve();
        if (nj == -1) pf = 4;
        else if (nj == -2) pf = 1;
        else start_chunk();
      } else if (pf == 1) {
        if (list_entry < n_chunks) {
          nj = (int)list_entry;
          start_chunk();
        } else {
          pf = 0;
        }
      } else if (pf == 2) {
        pbase = ns & ~31;
        if (ns >= 0 && ns < (int)n_ranges) {
          pw = load_window(pbase, pt);
          pw2 = load_window(pbase + 32, pt2);
        }
        // raw reads, combined when the chunk is taken (no stall here)
        if (prune) {
          pth = ld_volatile_u32(P.theta_key);
          if (P.xth_local) pxw = ld_volatile_u64(P.xth_local);
        }
        pf = 3;
      }
    };
    if (dyn) {
      claim();
      if (blockIdx.x < n_chunks) {  // the first chunk needs no claim
        nj = (int)blockIdx.x;
        if (table) {
          if (lane == 0) taken_old = atomicExch(P.chunk_taken + nj, epoch);
          ns = first_range >= 0 ? first_range : __ldcg(P.chunk_first_range + nj);
        } else {
          ns = locate((uint32_t)nj * chunk_rows, 0);
        }
        pf = 2;
        if (first_range >= 0) {  // its windows are in flight already
          pbase = first_range & ~31;
          pw = fw0;
          pw2 = fw1;
          pt = ft0;
          pt2 = ft1;
          pth = s_theta0;
          pf = 3;
        }
      }
    } else if (vb < ve && n_ranges > 0) {
      s = locate(vb, 0);
      base = s & ~31;
      win = load_window(base, tag_cur);
      win_next = load_window(base + 32, tag_next);
      ubk = decode(tag_cur);
      set_range();
      if ((uint32_t)rg.x > vb) {
        fail_range();
        ve = vb;
      }
    }
    uint32_t v = vb, streamed = 0;
    int it = 0;
    bool ok = true;
    for (;;) {
      if (v >= ve) {
        if (!dyn || bad_range) break;
        for (;;) {
          while (pf < 3) prefetch();  // what the stages of the last chunk did not prepare
          if (pf == 4 || !table || __shfl_sync(FULL_MASK, taken_old, 0) != epoch) break;
          pf = 0;  // another CTA streams it
        }
        if (pf == 4) break;
        vb = (uint32_t)nj * chunk_rows;  // < n_rows
        ve = min(n_rows, vb + chunk_rows);
        v = vb;
        s = ns;
        pf = 0;
        if (s < 0 || s >= (int)n_ranges) {
          fail_range();
          break;
        }
        base = pbase;
        win = pw;
        win_next = pw2;
        ubk = decode(pt);
        tag_next = pt2;
        pkey = max(s_text, pth);
        if (P.xth_local && (uint32_t)(pxw >> 32) == P.xth_tag && (uint32_t)pxw > pkey) {
          // another shard's k-th best is higher: it becomes this shard's running
          // threshold too (the consumers read it from the threshold line)
          pkey = (uint32_t)pxw;
          if (lane == 0) atomicMax(P.theta_key, pkey);
        }
        set_range();
        if ((uint32_t)rg.x > vb) {  // the range must start at or before the chunk
          fail_range();
          break;
        }
      }
      const int stage = it % STAGES, f = it / STAGES;
      bool free_stage = true;
      if (lane == 0 && f > 0) free_stage = mbar_wait(&empty[stage], (f - 1) & 1, P.err, ERR_TIMEOUT_EMPTY);
      if (!__shfl_sync(FULL_MASK, free_stage, 0)) {
        ok = false;
        if (lane == 0) s_err = 1;
        break;
      }
      int n = 0, nr = 0;
      uint32_t run_end = 0xffffffffu;  // leaf row just past the open run
      int my_slot = 0, my_row = 0;     // this lane's run (lane < nr)
      while (n < ROWS && v < ve) {
        const uint32_t rlen = (uint32_t)(rg.z - rg.y);
        if (v >= (uint32_t)rg.x + rlen) {
          ++s;
          if (s >= (int)n_ranges) {
            fail_range();
            v = ve;
            break;
          }
          if (s - base == 32) {
            base += 32;
            win = win_next;
            ubk = decode(tag_next);
            win_next = load_window(base + 32, tag_next);
          }
          set_range();
          continue;
        }
        if (rkey < pkey) {  // the rest of this child is below the threshold
          v = min(ve, (uint32_t)rg.x + rlen);
          continue;
        }
        const uint32_t row = (uint32_t)rg.y + (v - (uint32_t)rg.x);
        const uint32_t take = min(min((uint32_t)(ROWS - n), ve - v), (uint32_t)rg.z - row);
        if (row != run_end) {  // adjacent children extend the open run
          if (lane == nr) {
            my_slot = n;
            my_row = (int)row;
          }
          ++nr;
        }
        run_end = row + take;
        n += (int)take;
        v += take;
      }
      if (n == 0) continue;  // every child left in the piece was skipped: no stage
      streamed += (uint32_t)n;
      // run j covers slots [start_j, start_{j+1}) (the last one up to n)
      const int next_slot = __shfl_down_sync(FULL_MASK, my_slot, 1);
      const int slot_end = (lane + 1 < nr) ? next_slot : n;
      if (lane < nr) stage_runs[stage * 32 + lane] = make_int2(my_slot, my_row);
      if (lane == 0) {
        stage_n[stage] = n;
        stage_nr[stage] = nr;
      }
      __syncwarp();  // the stage's run table is written before lane 0's arrive releases it
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[stage], (uint32_t)n * (uint32_t)P.row_bytes + 16u);
        tma_load_1d(smem + L.side_off + (size_t)stage * 16, theta_line, 16u, &full[stage]);
      }
      __syncwarp();
      if (lane < nr) {
        unsigned char* dst = smem + L.stages_off + (size_t)stage * L.stage_bytes;
        tma_load_1d_stream(dst + (size_t)my_slot * P.row_bytes, leaf_bytes + (size_t)my_row * P.row_bytes,
                           (uint32_t)(slot_end - my_slot) * (uint32_t)P.row_bytes, &full[stage], policy);
      }
      ++it;
      if (dyn && pf < 3) prefetch();  // with the stage's copies out
    }
    if (lane == 0) {
      if (P.rows_streamed && streamed) atomicAdd(P.rows_streamed, streamed);
      const int stage = it % STAGES, f = it / STAGES;
      if (ok && f > 0 && !mbar_wait(&empty[stage], (f - 1) & 1, P.err, ERR_TIMEOUT_EMPTY)) s_err = 1;
      stage_n[stage] = -1;
      mbar_arrive(&full[stage]);
    }
  } else {
    // ------------------------------------------------------------ consumers
    float4 qv[VPL];
    const float4* q4 = reinterpret_cast<const float4*>(P.q);
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int c = lane + 32 * v;
      qv[v] = (c < P.D4) ? __ldg(q4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    unsigned long long* tk = topk_all + warp * SORTN;
    uint32_t theta_w = 0;                                 // this warp's k-th best key
    uint32_t theta = max(ld_volatile_u32(P.theta_key), s_text);  // filter key (max of both)
    int cnt = 0;                                          // buffered candidates
    uint32_t published = 0;

    // tk[0..k) holds the warp's k best (sorted), tk[k..k+cnt) the buffered
    // candidates, everything above is zero; a merge sorts only the live prefix
    // (rounded up to a power of two) and clears what falls below the k-th
    // up to 128 live values are sorted in registers (R per lane), more in shared memory
    auto sort_regs = [&](auto r_tag) {
      constexpr int R = decltype(r_tag)::value;
      unsigned long long v[R];
#pragma unroll
      for (int r = 0; r < R; ++r) v[r] = tk[lane * R + r];
      warp_sort_regs_desc<R>(v, lane);
#pragma unroll
      for (int r = 0; r < R; ++r) tk[lane * R + r] = (lane * R + r < k) ? v[r] : 0ull;
    };
    auto merge = [&]() {
      __syncwarp();
      const int live = k + cnt;  // <= k + BUF <= SORTN
      if (live <= 32) {
        sort_regs(std::integral_constant<int, 1>{});
      } else if (live <= 64) {
        sort_regs(std::integral_constant<int, 2>{});
      } else if (live <= 128) {
        sort_regs(std::integral_constant<int, 4>{});
      } else {
        int n2 = 256;
        while (n2 < live) n2 <<= 1;
        warp_bitonic_desc(tk, n2, lane);
        for (int i = k + lane; i < n2; i += 32) tk[i] = 0ull;
      }
      __syncwarp();
      cnt = 0;
      const uint32_t kth = cand_key(tk[k - 1]);
      if (kth > theta_w) {
        theta_w = kth;
        if (kth > published) {
          if (lane == 0) {
            atomicMax(P.theta_key, kth);
            share_threshold(P, kth);
          }
          published = kth;
        }
      }
      theta = max(theta, theta_w);
      __syncwarp();
    };

    for (int it = 0;; ++it) {
      const int stage = it % STAGES, f = it / STAGES;
      if (!mbar_wait(&full[stage], f & 1, P.err, ERR_TIMEOUT_FULL)) {
        s_err = 1;
        break;
      }
      const int n = stage_n[stage];
      if (n < 0) break;
      theta = max(theta, side[stage * 4 + theta_word]);
      const float4* stage_f4 =
          reinterpret_cast<const float4*>(smem + L.stages_off + (size_t)stage * L.stage_bytes);
      float acc[RPW];
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        acc[r] = 0.f;
        const int slot = warp * RPW + r;
        if (slot < n) {
          const float4* row = stage_f4 + (size_t)slot * P.D4;
#pragma unroll
          for (int v = 0; v < VPL; ++v) {
            const int c = lane + 32 * v;
            if (c < P.D4) {
              const float4 x = row[c];
              acc[r] = fmaf(x.x, qv[v].x, acc[r]);
              acc[r] = fmaf(x.y, qv[v].y, acc[r]);
              acc[r] = fmaf(x.z, qv[v].z, acc[r]);
              acc[r] = fmaf(x.w, qv[v].w, acc[r]);
            }
          }
        }
      }
      // multi-row butterfly: every row is reduced with the same xor tree
      // (16, 8, 4, 2, 1), so a row's score does not depend on its slot.
      float score;
      int rloc;
      if constexpr (RPW == 4) {
        const bool h16 = lane & 16, h8 = lane & 8;
        const float t0 = __shfl_xor_sync(FULL_MASK, h16 ? acc[0] : acc[2], 16);
        const float t1 = __shfl_xor_sync(FULL_MASK, h16 ? acc[1] : acc[3], 16);
        const float b0 = (h16 ? acc[2] : acc[0]) + t0;
        const float b1 = (h16 ? acc[3] : acc[1]) + t1;
        const float t = __shfl_xor_sync(FULL_MASK, h8 ? b0 : b1, 8);
        score = (h8 ? b1 : b0) + t;
        score += __shfl_xor_sync(FULL_MASK, score, 4);
        score += __shfl_xor_sync(FULL_MASK, score, 2);
        score += __shfl_xor_sync(FULL_MASK, score, 1);
        rloc = (h16 ? 2 : 0) + (h8 ? 1 : 0);
      } else if constexpr (RPW == 2) {
        const bool h16 = lane & 16;
        const float t = __shfl_xor_sync(FULL_MASK, h16 ? acc[0] : acc[1], 16);
        score = (h16 ? acc[1] : acc[0]) + t;
        score += __shfl_xor_sync(FULL_MASK, score, 8);
        score += __shfl_xor_sync(FULL_MASK, score, 4);
        score += __shfl_xor_sync(FULL_MASK, score, 2);
        score += __shfl_xor_sync(FULL_MASK, score, 1);
        rloc = h16 ? 1 : 0;
      } else {
        score = acc[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) score += __shfl_xor_sync(FULL_MASK, score, o);
        rloc = 0;
      }
      const bool owner = (lane & (32 / RPW - 1)) == 0;
      const int slot = warp * RPW + rloc;
      const uint32_t key = f2key(score);
      const bool cand = owner && slot < n && key >= theta;
      int row = 0;
      if (cand) {  // rare: map the slot back to its leaf row through the stage's runs
        const int2* runs = stage_runs + stage * 32;
        int i = stage_nr[stage] - 1;
        while (i > 0 && runs[i].x > slot) --i;
        row = runs[i].y + (slot - runs[i].x);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      const uint32_t bal = __ballot_sync(FULL_MASK, cand);
      if (bal) {
        const int nn = __popc(bal);
        if (cnt + nn > BUF) merge();
        if (cand) tk[k + cnt + __popc(bal & lanemask_lt())] = pack_cand(key, (uint32_t)row);
        cnt += nn;
      }
    }
    if (cnt > 0) merge();
    if (lane == 0) s_warp_theta[warp] = theta;
  }
  __syncthreads();
  // the merges' threshold: the best any warp of this CTA saw (no L2 read)
  if (tid == 0) {
    uint32_t t = 0;
    for (int w = 0; w < SCAN_CONSUMER_WARPS; ++w) t = max(t, s_warp_theta[w]);
    s_theta = t;
  }
  __syncthreads();
  // error path: one of this CTA's waits gave up, so its own bulk copies may still
  // land in the stage ring, which the merges below reuse
  if (s_err) {
    if (tid == 0) grace_period();
    __syncthreads();
  }

  // ---------------------------------------------------------- CTA merge
  // theta_key is the k-th best of k distinct scanned rows (or an external
  // bound), so no candidate below it can reach the final list: both merges
  // skip those, and usually little more than k candidates remain grid-wide.
  // The CTA's k-th best is published as a threshold too (k distinct rows).
  const int selN = KCAP;  // KCAP is a power of two >= k
  unsigned long long* ring = reinterpret_cast<unsigned long long*>(smem + L.stages_off);  // idle now
  if constexpr (KCAP == 32) {
    // k <= 32: warp 0 merges the eight sorted warp lists in registers (lane j
    // holds the j-th value) as a tree of independent pairwise merges; left
    // operands come out descending and right ones ascending, so no list is
    // reversed between levels.  Warp 0 then takes the CTA's ticket itself.
    static_assert(SCAN_CONSUMER_WARPS == 8, "three merge levels");
    if (warp == 0) {
      unsigned long long r[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        r[i] = warp_merge_top32(topk_all[(2 * i) * SORTN + lane], topk_all[(2 * i + 1) * SORTN + (31 - lane)],
                                (i & 1) == 0, lane);
      const unsigned long long s0 = warp_merge_top32(r[0], r[1], true, lane);
      const unsigned long long s1 = warp_merge_top32(r[2], r[3], false, lane);
      const unsigned long long m = warp_merge_top32(s0, s1, true, lane);
      const unsigned long long kth = __shfl_sync(FULL_MASK, m, k - 1);
      if (lane < k) {
        P.cta_lists[(size_t)blockIdx.x * k + lane] = m;
        if (lane == 0 && kth != 0ull && cand_key(kth) > s_theta) {
          atomicMax(P.theta_key, cand_key(kth));
          share_threshold(P, cand_key(kth));
        }
        __threadfence();
      }
      __syncwarp();
      if (lane == 0) s_is_last = (atomicAdd(P.done, 1u) == G - 1);
    }
  } else {
    if (block_rank_topk<RANK_CAP>(topk_all, SCAN_CONSUMER_WARPS * SORTN, k, sel, selN, ring, &s_rank_count,
                                  s_theta) < 0)
      block_select_topk<false>(topk_all, SCAN_CONSUMER_WARPS * SORTN, k, sel, selN, scratch, s_theta);
    static_assert(KMAX <= SCAN_THREADS, "one thread per list entry");
    if (tid < k) {
      const unsigned long long c = sel[tid];
      P.cta_lists[(size_t)blockIdx.x * k + tid] = c;
      if (tid == k - 1 && c != 0ull && cand_key(c) > s_theta) {
        atomicMax(P.theta_key, cand_key(c));
        share_threshold(P, cand_key(c));
      }
      __threadfence();
    }
  }
  __syncthreads();
  if constexpr (KCAP != 32) {
    if (tid == 0) {
      __threadfence();
      s_is_last = (atomicAdd(P.done, 1u) == G - 1);
    }
    __syncthreads();
  }
  if (!s_is_last) return;
  // an overlapped scan does not finish before the bounds kernel (nor, through
  // it, the root scan): later work on the stream and the control-header copy
  // below see both complete
  if (P.overlapped) griddep_wait();
  __threadfence();

  // ---------------------------------------------------------- grid merge (last CTA)
  // Every CTA published its k-th best before its ticket, so the global
  // threshold is final here; the last CTA's threads load the G lists (eight
  // entries in flight per thread), keep what is not below it -- usually little
  // more than k entries -- rank those directly and write each result to its
  // slot: one block barrier between the loads and the outputs.
  // The control header is final too (every CTA updated it before its ticket).
  if (P.ctrl_out)
    for (int i = tid; i < (int)(CTRL_RESET_BYTES / 8); i += blockDim.x) P.ctrl_out[i] = __ldcg(P.ctrl_hdr + i);
  float* out_scores = P.out_scores;
  int* out_ids = P.out_ids;
  if (P.out_indirect) {
    const unsigned long long* ptrs = reinterpret_cast<const unsigned long long*>(P.out_indirect);
    out_scores = reinterpret_cast<float*>(__ldcg(ptrs));
    out_ids = reinterpret_cast<int*>(__ldcg(ptrs + 1));
  }
  const auto emit = [&](int r, unsigned long long c) {
    if (c != 0ull) {
      const uint32_t row = cand_row(c);
      out_scores[r] = key2f(cand_key(c));
      if (out_ids) out_ids[r] = P.original_ids ? P.original_ids[row] : (int)row;
      if (P.out_rows) P.out_rows[r] = (long long)row;
    } else {
      out_scores[r] = -INFINITY;
      if (out_ids) out_ids[r] = -1;
      if (P.out_rows) P.out_rows[r] = -1;
    }
  };
  const int M = (int)G * k;  // gathered lists
  uint32_t th = 0u;
  if (lane == 0) th = ld_volatile_u32(P.theta_key);
  th = max(__shfl_sync(FULL_MASK, th, 0), s_theta);  // per warp; any of these bounds is valid
  unsigned long long* tmp = ring;                       // idle now; holds FINAL_RANK_CAP entries
  for (int b0 = 0; b0 < M; b0 += 8 * SCAN_THREADS) {
    unsigned long long v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = b0 + u * SCAN_THREADS + warp * 32 + lane;
      v[u] = i < M ? __ldcg(P.cta_lists + i) : 0ull;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const bool pass = v[u] != 0ull && cand_key(v[u]) >= th;
      const uint32_t bal = __ballot_sync(FULL_MASK, pass);
      uint32_t pos = 0;
      if (lane == 0 && bal) pos = atomicAdd(&s_fin_count, (uint32_t)__popc(bal));
      pos = __shfl_sync(FULL_MASK, pos, 0) + __popc(bal & lanemask_lt());
      if (pass && pos < (uint32_t)FINAL_RANK_CAP) tmp[pos] = v[u];
    }
  }
  __syncthreads();
  const int n = (int)s_fin_count;
  if (n <= FINAL_RANK_CAP) {
    // rank = number of larger kept entries (entries are unique); for every
    // entry of the true top-k all larger entries were kept, whatever bound
    // each warp used, so these ranks are the global ranks
    for (int t = tid; t < n; t += blockDim.x) {
      const unsigned long long c = tmp[t];
      int r = 0, j = 0;
      for (; j + 8 <= n; j += 8) {
#pragma unroll
        for (int u = 0; u < 8; ++u) r += tmp[j + u] > c;
      }
      for (; j < n; ++j) r += tmp[j] > c;
      if (r < k) emit(r, c);
    }
    for (int r = n + tid; r < k; r += blockDim.x) emit(r, 0ull);
  } else {
    block_select_topk<true>(P.cta_lists, M, k, sel, selN, scratch, s_theta);
    for (int i = tid; i < k; i += blockDim.x) emit(i, sel[i]);
  }
  if (P.done_out) {
    // every thread's results (and the header copy) reach the system before the
    // completion word that the blocking caller spins on
    __threadfence_system();
    __syncthreads();
    if (tid == 0) *reinterpret_cast<volatile uint32_t*>(P.done_out) = ld_volatile_u32(P.call_seq);
  }
}

// ============================================================ search prologue
// First kernel of every search: clears the control header and, in a
// graph-replayed blocking search, stages the query (replacing a host-to-device
// copy and a memset, two copy-engine operations of a few microseconds each at
// this size).  The query comes from mapped pinned memory (q_host) or from the
// device pointer slots[0]; slots[1..2] (the caller's device outputs) are staged
// for the final merge; with neither, only the header is cleared.  The kernels
// after it are its programmatic dependents.
__global__ void __launch_bounds__(128) k_search_prologue(const float4* q_host, void* const* slots, float4* dq, int D4,
                                                         unsigned long long* ctrl_hdr, void** out_indirect,
                                                         const uint32_t* seq_in, uint32_t* epoch_counter,
                                                         unsigned long long* sync_words) {
  const int tid = threadIdx.x;
  const float4* src = q_host;
  if (slots) {
    src = static_cast<const float4*>(slots[0]);
    if (tid < 2) out_indirect[tid] = slots[tid + 1];
  }
  if (src)
    for (int i = tid; i < D4; i += blockDim.x) dq[i] = src[i];
  if (tid < (int)(CTRL_RESET_BYTES / 8)) {
    unsigned long long w = 0ull;
    if (tid == CTRL_SEQ_WORD && seq_in) w = *seq_in;
    if (tid == CTRL_EPOCH_WORD && epoch_counter) {
      // searches on one workspace run one after another: a plain increment;
      // 0 is skipped, so a never-written bound entry (epoch 0) is never current
      uint32_t e = *epoch_counter + 1u;
      if (e == 0u) e = 1u;
      *epoch_counter = e;
      w = e;
    }
    ctrl_hdr[tid] = w;
  }
  if (sync_words && tid < (int)(sizeof(ScanSync) / 8)) sync_words[tid] = 0ull;
}

// ============================================================ root scan (K1)
// Seed threshold (reference search.py:26-41 takes the k-th best score of every
// row of the best root, after four host syncs): the last CTA of the root scan
// scores a sample of up to min(rows of the seed root, max(4k, 128), 1024) of
// its rows -- blocks of up to 16 consecutive rows (one bulk copy each) starting
// at evenly spaced positions -- and keeps T = the k-th best sampled score.
// Any k distinct rows give a valid threshold (T never exceeds the global k-th
// best), and the sampled scores use the leaf scan's exact arithmetic (per lane
// FMAs over float4 columns lane, lane + 32, ...; then one xor butterfly), so T
// equals the main scan's own score of a real row.  The seed root's rows are
// scanned by the main scan like any surviving root's.
constexpr int SEED_RING_BYTES = 192 * 1024;

struct RootScanLayout {
  int ring_rows;
  size_t keys_off, rows_off, sel_off, scratch_off, q_off, bar_off, total;
};
__host__ __device__ inline RootScanLayout root_scan_layout(int row_bytes) {
  RootScanLayout L;
  L.ring_rows = SEED_RING_BYTES / row_bytes < 128 ? SEED_RING_BYTES / row_bytes : 128;
  L.keys_off = align_up((size_t)L.ring_rows * row_bytes, 128);
  L.rows_off = L.keys_off + (size_t)SEED_SAMPLE_MAX * 8;
  L.sel_off = align_up(L.rows_off + (size_t)(SEED_SAMPLE_MAX / SEED_BLOCK) * 3 * 4, 16);
  L.scratch_off = L.sel_off + (size_t)KMAX * 8;
  L.q_off = align_up(L.scratch_off + sizeof(SelectScratch), 16);
  L.bar_off = L.q_off + (size_t)MAX_DIM * 4;
  L.total = L.bar_off + 16;
  return L;
}

__global__ void __launch_bounds__(ROOT_SCAN_WARPS * 32) k_root_scan(IndexView ix, const float* __restrict__ q,
                                                                     SearchCtrl* ctrl, int k,
                                                                     float* __restrict__ T_export) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ unsigned long long s_best[ROOT_SCAN_WARPS];
  __shared__ int s_last, s_nsample, s_ok, s_nblk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  griddep_wait();    // the control header is cleared (and the query staged) by the kernel before
  griddep_launch();  // the bounds kernel's threshold-free phase runs beside this one
  const float4* q4 = reinterpret_cast<const float4*>(q);
  unsigned long long packed = 0ull;
  for (int p = blockIdx.x * ROOT_SCAN_WARPS + warp; p < ix.R; p += gridDim.x * ROOT_SCAN_WARPS) {
    const float4* c4 = reinterpret_cast<const float4*>(ix.root_centers + (size_t)p * ix.D);
    float acc = 0.f;
    for (int c = lane; c < ix.D4; c += 32) {
      const float4 a = __ldg(q4 + c), b = __ldg(c4 + c);
      acc = fmaf(a.x, b.x, acc);
      acc = fmaf(a.y, b.y, acc);
      acc = fmaf(a.z, b.z, acc);
      acc = fmaf(a.w, b.w, acc);
    }
    const float dot = warp_sum(acc);
    const int rows = ix.root_rows[p];
    const unsigned long long prio = rows >= k ? 2ull : (rows > 0 ? 1ull : 0ull);
    const unsigned long long pk =
        (prio << 62) | ((unsigned long long)f2key(dot) << 30) | (unsigned long long)(0x3fffffff - p);
    packed = pk > packed ? pk : packed;
  }
  if (blockIdx.x == 0 && warp == 0) {
    float acc = 0.f;
    for (int c = lane; c < ix.D4; c += 32) {
      const float4 a = __ldg(q4 + c);
      acc = fmaf(a.x, a.x, acc);
      acc = fmaf(a.y, a.y, acc);
      acc = fmaf(a.z, a.z, acc);
      acc = fmaf(a.w, a.w, acc);
    }
    const float qn2 = warp_sum(acc);
    if (lane == 0) ctrl->qn2 = qn2;
  }
  if (lane == 0) s_best[warp] = packed;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < ROOT_SCAN_WARPS; ++w) b = max(b, s_best[w]);
    if (b) atomicMax(&ctrl->best_packed, b);
    __threadfence();
    const uint32_t t = atomicAdd(&ctrl->k1_done, 1u);
    s_last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // ---- last CTA: the seed sample
  const RootScanLayout L = root_scan_layout(ix.D * 4);
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem + L.keys_off);
  int* blk = reinterpret_cast<int*>(smem + L.rows_off);  // [SEED_BLOCKS] leaf row, length, sample position
  unsigned long long* sel = reinterpret_cast<unsigned long long*>(smem + L.sel_off);
  SelectScratch* scratch = reinterpret_cast<SelectScratch*>(smem + L.scratch_off);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  // the children of the seed root (the first SEED_SAMPLE_MAX of them in CSR
  // order) as row intervals within the root: ch_v[c] = first row, ch_off[c] =
  // its leaf row (precomputed per CSR entry); the key area is free until the
  // sample is scored
  int* ch_v = reinterpret_cast<int*>(keys);
  int* ch_off = ch_v + SEED_SAMPLE_MAX;
  float4* sq4 = reinterpret_cast<float4*>(smem + L.q_off);
  if (warp == 0) {
    const unsigned long long best = ld_volatile_u64(&ctrl->best_packed);
    int pb = 0x3fffffff - (int)(best & 0x3fffffffull);
    if (pb < 0 || pb >= ix.R) pb = 0;  // only reachable with NaN scores; keeps the table reads in bounds
    if (k <= 32 && ix.seed_tab) {
      // precomputed blocks of this root: one read per lane
      const int4 e = lane < SEED_TAB_W ? __ldg(ix.seed_tab + (size_t)pb * SEED_TAB_W + lane) : make_int4(0, 0, 0, 0);
      const int nb = __shfl_sync(FULL_MASK, e.x, 0), S = __shfl_sync(FULL_MASK, e.y, 0);
      if (lane >= 1 && lane <= nb) {
        blk[3 * (lane - 1)] = e.x;
        blk[3 * (lane - 1) + 1] = e.y;
        blk[3 * (lane - 1) + 2] = e.z;
      }
      if (lane == 0) {
        s_nblk = nb;
        s_nsample = S;
      }
    } else {
      const int cb = ix.root_child_ptr[pb];
      const int nall = ix.root_child_ptr[pb + 1] - cb;
      const int nch = min(nall, SEED_SAMPLE_MAX);
      for (int ci = lane; ci < nch; ci += 32) {
        const int2 sp = __ldg(ix.root_child_span + cb + ci);
        ch_off[ci] = sp.x;
        ch_v[ci] = sp.y;
      }
      // rows of those children: the whole root, or up to the first child left out
      const int vrows = nall > nch ? __ldg(ix.root_child_span + cb + nch).y : ix.root_rows[pb];
      __syncwarp();
      // blocks of up to SEED_BLOCK consecutive rows starting at evenly spaced
      // virtual rows, each inside one child (one bulk copy per block); block b
      // ends before block b + 1 starts, so no row is sampled twice
      const int want = min(min(vrows, max(4 * k, 128)), SEED_SAMPLE_MAX);
      const int nb = (want + SEED_BLOCK - 1) / SEED_BLOCK;
      int pos_base = 0;
      for (int b0 = 0; b0 < nb; b0 += 32) {
        const int b = b0 + lane;
        int row = 0, len = 0;
        if (b < nb) {
          // exact in double: vrows < 2^31, nb <= 64
          const int v = (int)floor((double)b * (double)vrows / (double)nb);
          const int v_next = (b + 1 < nb) ? (int)floor((double)(b + 1) * (double)vrows / (double)nb) : vrows;
          int lo = 0, hi = nch - 1;
          while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (ch_v[mid] <= v) lo = mid; else hi = mid - 1;
          }
          const int child_end = (lo + 1 < nch) ? ch_v[lo + 1] : vrows;
          len = min(min(SEED_BLOCK, v_next - v), child_end - v);
          row = ch_off[lo] + (v - ch_v[lo]);
        }
        const int incl = warp_incl_scan(len, lane);
        if (b < nb) {
          blk[3 * b] = row;
          blk[3 * b + 1] = len;
          blk[3 * b + 2] = pos_base + incl - len;
        }
        pos_base += __shfl_sync(FULL_MASK, incl, 31);
      }
      if (lane == 0) {
        s_nblk = nb;
        s_nsample = pos_base;
      }
    }
    if (lane == 0) {
      s_ok = 1;
      ctrl->best_root = pb;
      mbar_init(bar, 1);
      fence_mbar_init();
    }
  } else {
    // the other warps stage the query meanwhile
    for (int c = threadIdx.x - 32; c < ix.D4; c += blockDim.x - 32) sq4[c] = __ldg(q4 + c);
  }
  __syncthreads();
  const int S = s_nsample, nb = s_nblk;
  const int rb = ix.D * 4;
  // (the query is in shared memory: this code runs once per search on a cold
  // instruction cache, so the scoring loop below is kept compact)
  uint32_t phase = 0;
  for (int r0 = 0; r0 < S; r0 += L.ring_rows) {
    const int nr = min(L.ring_rows, S - r0);
    if (warp == 0) {
      if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(nr * rb));
      __syncwarp();
      // the part of each block that falls into this round's sample positions
      for (int b = lane; b < nb; b += 32) {
        const int p0 = blk[3 * b + 2], p1 = p0 + blk[3 * b + 1];
        const int a = max(p0, r0), e = min(p1, r0 + nr);
        if (a < e)
          tma_load_1d(smem + (size_t)(a - r0) * rb, ix.leaf + (size_t)(blk[3 * b] + (a - p0)) * ix.D,
                      (uint32_t)((e - a) * rb), bar);
      }
    }
    if (threadIdx.x == 0 && !mbar_wait(bar, phase, &ctrl->error, ERR_TIMEOUT_FULL)) s_ok = 0;
    __syncthreads();
    if (!s_ok) break;
    phase ^= 1u;
    // four rows per warp at a time (independent FMA chains); each row's score
    // is computed exactly as the leaf scan computes it
    for (int i0 = warp * 4; i0 < nr; i0 += ROOT_SCAN_WARPS * 4) {
      const float4* r0p = reinterpret_cast<const float4*>(smem + (size_t)i0 * rb);
      const int rstride = rb / 16, live = min(4, nr - i0);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
      for (int c = lane; c < ix.D4; c += 32) {
        const float4 a = sq4[c];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float4 x = t < live ? r0p[t * rstride + c] : make_float4(0.f, 0.f, 0.f, 0.f);
          acc[t] = fmaf(x.x, a.x, acc[t]);
          acc[t] = fmaf(x.y, a.y, acc[t]);
          acc[t] = fmaf(x.z, a.z, acc[t]);
          acc[t] = fmaf(x.w, a.w, acc[t]);
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) acc[t] = warp_sum(acc[t]);
      if (lane < live) {
        const float dot = lane == 0 ? acc[0] : (lane == 1 ? acc[1] : (lane == 2 ? acc[2] : acc[3]));
        keys[r0 + i0 + lane] = pack_cand(f2key(dot), (uint32_t)(r0 + i0 + lane));
      }
    }
    __syncthreads();  // the ring is refilled by the next round
  }
  if (!s_ok) {
    if (threadIdx.x == 0) grace_period();  // copies of the round that gave up may still land
    __syncthreads();
  }
  // T = k-th best sampled key (0 = no threshold: fewer than k rows sampled)
  uint32_t T = 0u;
  if (s_ok && S >= k) {
    if (S <= 128) {
      // warp 0, four keys per lane
      if (warp == 0) {
        uint32_t kv[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) kv[r] = (lane * 4 + r < S) ? cand_key(keys[lane * 4 + r]) : 0u;
        if (k <= 32) {
          // k rounds: the largest key left, one copy of it removed
          for (int i = 0; i < k; ++i) {
            const uint32_t m = max(max(kv[0], kv[1]), max(kv[2], kv[3]));
            const uint32_t wm = __reduce_max_sync(FULL_MASK, m);
            T = wm;
            const int lead = __ffs(__ballot_sync(FULL_MASK, m == wm)) - 1;
            if (lane == lead) {
              if (kv[0] == wm) kv[0] = 0u;
              else if (kv[1] == wm) kv[1] = 0u;
              else if (kv[2] == wm) kv[2] = 0u;
              else kv[3] = 0u;
            }
          }
        } else {
          // the largest t with at least k keys >= t, decided bit by bit (that t
          // is the k-th largest key)
          uint32_t t = 0u;
          for (int bit = 31; bit >= 0; --bit) {
            const uint32_t tr = t | (1u << bit);
            int cnt = 0;
#pragma unroll
            for (int r = 0; r < 4; ++r) cnt += __popc(__ballot_sync(FULL_MASK, kv[r] >= tr));
            if (cnt >= k) t = tr;
          }
          T = t;
        }
      }
    } else {
      int selN = 1;
      while (selN < k) selN <<= 1;
      if (block_select_topk<false>(keys, S, k, sel, selN, scratch) == k) T = cand_key(sel[k - 1]);
    }
  }
  if (threadIdx.x == 0) {
    ctrl->seed_T_key = T;
    ctrl->seed_packed = (unsigned long long)(uint32_t)S;  // rows scored by the sample
    if (T) atomicMax(&ctrl->theta_key, T);  // the main scan may be raising it already
    if (T_export) *T_export = T ? key2f(T) : -INFINITY;
  }
}

// ============================================================ bounds (K3)
struct BoundsLayout {
  size_t q_off, warp_off, chunk_bytes, warp_bytes, total;
};
__host__ __device__ inline BoundsLayout bounds_layout(int D, int rank, int chunk_rows) {
  BoundsLayout L;
  L.q_off = 0;
  L.chunk_bytes = align_up((size_t)chunk_rows * rank * 4, 128);
  L.warp_off = align_up((size_t)D * 4, 128);
  // 2 chunk buffers + 64 red(a) + 64 red(s)... + a[64] + s[64] + 2 mbarriers
  L.warp_bytes = align_up(2 * L.chunk_bytes + (64 + 64 + 64 + 64) * 4 + 2 * 8, 128);
  L.total = L.warp_off + BOUNDS_WARPS * L.warp_bytes;
  return L;
}

// Two phases, so that the bound arithmetic overlaps the root scan (the kernel
// is launched as a programmatic dependent of it):
//  1. before griddep_wait(): per root (warp per root), fl(q.c) and ||q||^2
//     recomputed here (any fp32 order is covered by the error terms), the
//     rigorous root bound, the projection a = V^T q with the basis staged by
//     TMA, and every child's rigorous bound; all rounded up to float and kept
//     in ub_root[R] / ub_child[C].  None of this depends on the threshold.
//     Each child's min(root bound, child bound) is also published for the main
//     scan, which runs beside this kernel: ub_tagged[CSR entry] = epoch << 32 |
//     key, one 64-bit store, so the scan sees either this search's bound or a
//     stale epoch (and then streams the child).
//  2. after griddep_wait(): T = max(seed threshold, T_ext) is known; the roots,
//     children and rows whose bound is not below T are counted for the trace
//     (what a scan of the survivors alone would read), and every main-scan
//     chunk that holds such a child and that no scan CTA holds yet is listed
//     once (an epoch swap per chunk).  The last CTA then adds 1 to the high half
//     of the main scan's claim word: the scan's CTAs take the listed chunks from
//     then on.
// T_ext (optional): a threshold from outside this index (the max of all shards'
// seed thresholds); the main scan prunes with it too.
__global__ void __launch_bounds__(BOUNDS_WARPS * 32) k_bounds(IndexView ix, const float* __restrict__ q,
                                                               SearchCtrl* ctrl, float* __restrict__ ub_root,
                                                               float* __restrict__ ub_child,
                                                               unsigned long long* __restrict__ ub_tagged,
                                                               int chunk_rows, const float* __restrict__ T_ext,
                                                               uint32_t scan_chunk_rows, uint32_t n_scan_chunks,
                                                               uint32_t* __restrict__ chunk_mark,
                                                               int* __restrict__ live_list, uint32_t scan_ctas,
                                                               ScanSync* __restrict__ sync) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_abort;
  griddep_launch();  // the main scan may start as soon as every CTA of this kernel runs
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int D = ix.D, r = ix.rank;
  const BoundsLayout L = bounds_layout(D, r, chunk_rows);
  float* sq = reinterpret_cast<float*>(smem + L.q_off);
  unsigned char* wb = smem + L.warp_off + (size_t)warp * L.warp_bytes;
  float* buf0 = reinterpret_cast<float*>(wb);
  float* buf1 = reinterpret_cast<float*>(wb + L.chunk_bytes);
  float* red = reinterpret_cast<float*>(wb + 2 * L.chunk_bytes);  // [64] a partials, [64] s partials
  float* sa = red + 128;                                           // [64]
  float* ss = sa + 64;                                             // [64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(ss + 64);

  // the query was complete before the kernel this one depends on was launched
  // (an earlier kernel of the search, or the caller's own work): read through L2
  for (int i = threadIdx.x; i < D; i += blockDim.x) sq[i] = __ldcg(q + i);
  const uint32_t epoch = ld_volatile_u32(&ctrl->epoch);
  const unsigned long long tag = (unsigned long long)epoch << 32;
  if (threadIdx.x == 0) s_abort = 0;
  if (lane == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();

  const double gD = gamma_n(D);
  // QN >= ||q||: fl(sum q_i^2) errs by at most gamma_D sum q_i^2 in any order
  float qacc = 0.f;
  for (int d = lane; d < D; d += 32) qacc = fmaf(sq[d], sq[d], qacc);
  const double QN = sqrt((double)warp_sum(qacc) / (1.0 - gD)) * (1.0 + 1e-15);
  const int n_chunks = (D + chunk_rows - 1) / chunk_rows;
  uint32_t ph0 = 0, ph1 = 0;
  bool abort_all = false;

  // ---- phase 1: bounds (independent of the threshold)
  for (int p = blockIdx.x * BOUNDS_WARPS + warp; p < ix.R && !abort_all; p += gridDim.x * BOUNDS_WARPS) {
    if (ix.root_rows[p] == 0) continue;
    // the basis copies go out first; q.c_r is computed while they are in flight
    const char* Vp = reinterpret_cast<const char*>(ix.bases + (size_t)p * D * r);
    if (lane == 0) {
      const int nr0 = min(chunk_rows, D);
      mbar_arrive_expect_tx(&bars[0], (uint32_t)(nr0 * r * 4));
      tma_load_1d(buf0, Vp, (uint32_t)(nr0 * r * 4), &bars[0]);
      if (n_chunks > 1) {
        const int nr1 = min(chunk_rows, D - chunk_rows);
        mbar_arrive_expect_tx(&bars[1], (uint32_t)(nr1 * r * 4));
        tma_load_1d(buf1, Vp + (size_t)chunk_rows * r * 4, (uint32_t)(nr1 * r * 4), &bars[1]);
      }
    }
    const float* cp = ix.root_centers + (size_t)p * D;
    float dacc = 0.f;
    for (int d = lane; d < D; d += 32) dacc = fmaf(sq[d], __ldg(cp + d), dacc);
    const double dot = (double)warp_sum(dacc);
    const double cn = ix.root_cn[p];
    const double rad = (double)ix.root_radii[p];
    const double e_dot = gD * QN * cn;            // |fl(q.c) - q.c|
    const double e_leaf = gD * QN * (cn + rad);   // |fl(q.x) - q.x| for ||x|| <= ||c|| + rad
    double ub_r = dot + e_dot + QN * rad + e_leaf;
    ub_r += 1e-12 * (fabs(dot) + QN * rad + e_dot + e_leaf);
    const float ub_rf = __double2float_ru(ub_r);  // the same in every lane (butterfly sums)
    if (lane == 0) ub_root[p] = ub_rf;
    // the children's boxes and radii are read after the projection: start
    // bringing them into L2 while the basis copies are in flight
    const int cb = ix.root_child_ptr[p], ce = ix.root_child_ptr[p + 1];
    for (int ci = cb + lane; ci < ce; ci += 32) {
      const int c = ix.root_child_list[ci];
      prefetch_l2(ix.child_l + (size_t)c * r);
      prefetch_l2(ix.child_u + (size_t)c * r);
      prefetch_l2(ix.child_radii + c);
      prefetch_l2(ix.leaf_sizes + c);  // read by phase 2, while the main scan may be saturating HBM
      prefetch_l2(ix.all_ranges + ci);
    }

    // ---- projection a = V^T q (and s = |V|^T |q|)
    float a0 = 0.f, a1 = 0.f, s0 = 0.f, s1 = 0.f;
    for (int ch = 0; ch < n_chunks; ++ch) {
      const int b = ch & 1;
      const bool ok = b ? mbar_wait(&bars[1], ph1, &ctrl->error, ERR_TIMEOUT_BASIS)
                        : mbar_wait(&bars[0], ph0, &ctrl->error, ERR_TIMEOUT_BASIS);
      if (!ok) { abort_all = true; break; }
      if (b) ph1 ^= 1u; else ph0 ^= 1u;
      const float* Vc = b ? buf1 : buf0;
      const int d0 = ch * chunk_rows;
      const int nr = min(chunk_rows, D - d0);
      if (r <= 32) {
        const int G = 32 / r, g = lane / r, j = lane - g * r;
        if (g < G) {
          for (int dl = g; dl < nr; dl += G) {
            const float v = Vc[dl * r + j], qq = sq[d0 + dl];
            a0 = fmaf(v, qq, a0);
            s0 = fmaf(fabsf(v), fabsf(qq), s0);
          }
        }
      } else {
        const bool two = lane + 32 < r;
        for (int dl = 0; dl < nr; ++dl) {
          const float qq = sq[d0 + dl];
          const float v0 = Vc[dl * r + lane];
          a0 = fmaf(v0, qq, a0);
          s0 = fmaf(fabsf(v0), fabsf(qq), s0);
          if (two) {
            const float v1 = Vc[dl * r + lane + 32];
            a1 = fmaf(v1, qq, a1);
            s1 = fmaf(fabsf(v1), fabsf(qq), s1);
          }
        }
      }
      __syncwarp();
      if (lane == 0 && ch + 2 < n_chunks) {
        const int d2 = (ch + 2) * chunk_rows;
        const int nr2 = min(chunk_rows, D - d2);
        uint64_t* bar = b ? &bars[1] : &bars[0];
        mbar_arrive_expect_tx(bar, (uint32_t)(nr2 * r * 4));
        tma_load_1d(b ? buf1 : buf0, Vp + (size_t)d2 * r * 4, (uint32_t)(nr2 * r * 4), bar);
      }
    }
    if (abort_all) break;
    if (r <= 32) {
      red[lane] = a0;
      red[64 + lane] = s0;
      __syncwarp();
      if (lane < r) {
        const int G = 32 / r;
        float A = 0.f, S = 0.f;
        for (int g = 0; g < G; ++g) { A += red[g * r + lane]; S += red[64 + g * r + lane]; }
        sa[lane] = A;
        ss[lane] = S;
      }
    } else {
      sa[lane] = a0;
      ss[lane] = s0;
      if (lane + 32 < r) { sa[lane + 32] = a1; ss[lane + 32] = s1; }
    }
    __syncwarp();

    // ---- rigorous residual norm ||q - V a|| (upper bound)
    double an2 = 0.0, sad = 0.0;
    for (int j = 0; j < r; ++j) {
      const double aj = sa[j];
      an2 += aj * aj;
      sad += fabs(aj) * gD * (double)ss[j] * (1.0 + 2.0 * gD);
    }
    an2 *= (1.0 + 1e-15);
    const double E = ix.root_defect[p];
    const double perp_sq = QN * QN - an2 + 2.0 * sad + E * an2;
    const double perp = sqrt(fmax(perp_sq, 0.0)) * (1.0 + 1e-15);
    const double an = sqrt(an2) * (1.0 + 1e-15);

    // ---- children: lane per child
    for (int c0 = cb; c0 < ce; c0 += 32) {
      const int ci = c0 + lane;
      if (ci >= ce) continue;
      const int c = ix.root_child_list[ci];
      const float* lp = ix.child_l + (size_t)c * r;
      const float* up = ix.child_u + (size_t)c * r;
      double box = 0.0, ebox = 0.0, wn2 = 0.0;
      if ((r & 3) == 0) {
        for (int j = 0; j < r; j += 4) {
          const float4 l4 = __ldg(reinterpret_cast<const float4*>(lp + j));
          const float4 u4 = __ldg(reinterpret_cast<const float4*>(up + j));
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, uv[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const double aj = sa[j + t];
            box += fmax(aj * lv[t], aj * uv[t]);
            const double w = fmax(fabs((double)lv[t]), fabs((double)uv[t]));
            ebox += (double)ss[j + t] * w;
            wn2 += w * w;
          }
        }
      } else {
        for (int j = 0; j < r; ++j) {
          const double aj = sa[j];
          const double lv = lp[j], uv = up[j];
          box += fmax(aj * lv, aj * uv);
          const double w = fmax(fabs(lv), fabs(uv));
          ebox += (double)ss[j] * w;
          wn2 += w * w;
        }
      }
      ebox *= gD * (1.0 + 2.0 * gD);
      const double rho = (double)ix.child_radii[c];
      double ub = dot + e_dot + box + ebox + an * E * sqrt(wn2) * (1.0 + 1e-15) + perp * rho + e_leaf;
      ub += 1e-12 * (fabs(dot) + fabs(box) + perp * rho + e_dot + e_leaf + ebox);
      const float ub_cf = __double2float_ru(ub);
      ub_child[c] = ub_cf;
      // a NaN bound (NaN query) is never published: the child is streamed
      const float m = fminf(ub_cf, ub_rf);
      if (!isnan(ub_cf) && !isnan(ub_rf)) ub_tagged[ci] = tag | f2key(m);
    }
    __syncwarp();  // sa / ss are rewritten for the next root
  }
  if (abort_all) {
    if (lane == 0) grace_period();  // basis copies may still be in flight into this warp's buffers
    s_abort = 1;                    // this CTA's roots are then all kept (the error bit is set)
  }
  __syncthreads();

  // ---- phase 2: the threshold is known
  griddep_wait();
  uint32_t Tkey = ctrl->seed_T_key;
  if (T_ext) {
    const float te = *T_ext;
    if (te > -INFINITY) {
      const uint32_t ek = f2key(te);
      if (ek > Tkey) Tkey = ek;
    }
  }
  const float T = Tkey ? key2f(Tkey) : -INFINITY;
  const bool keep_all = s_abort != 0;
  // chunks [0, frontier) are held by scan CTAs already (each CTA's first chunk
  // and every in-order claim so far)
  const uint32_t frontier = chunk_mark ? (uint32_t)ld_volatile_u64(&sync->chunk_claims) + scan_ctas : 0u;
  // Live-chunk list.  Inside a root, a chunk is listed by the first surviving
  // child that covers it (a max-scan over the warp's lanes, carried across the
  // root's 32-child groups); only a chunk that reaches past the root's rows can
  // also be listed by a neighbouring root, and only for those an epoch swap on
  // its mark keeps it listed once.  Entries gather in shared memory (one list
  // append per CTA); a CTA that lists more than LIST_SMEM appends the rest per
  // warp.
  constexpr uint32_t LIST_SMEM = 1024;
  __shared__ int s_list[LIST_SMEM];
  __shared__ uint32_t s_nlist, s_roots, s_children, s_rows, s_base;
  if (threadIdx.x == 0) s_nlist = s_roots = s_children = s_rows = 0u;
  __syncthreads();
  const uint32_t cr = scan_chunk_rows;
  uint32_t surv_roots = 0, surv_children = 0, surv_rows = 0;
  for (int p = blockIdx.x * BOUNDS_WARPS + warp; p < ix.R; p += gridDim.x * BOUNDS_WARPS) {
    if (ix.root_rows[p] == 0) continue;
    if (!keep_all && __ldcg(ub_root + p) < T) continue;
    ++surv_roots;
    const int cb = ix.root_child_ptr[p], ce = ix.root_child_ptr[p + 1];
    // the root's virtual rows [r_lo, r_hi)
    uint32_t r_lo = 0u, r_hi = 0u;
    if (chunk_mark && ce > cb) {
      const int4 e0 = __ldg(&ix.all_ranges[cb]), e1 = __ldg(&ix.all_ranges[ce - 1]);
      r_lo = (uint32_t)e0.x;
      r_hi = (uint32_t)e1.x + (uint32_t)(e1.z - e1.y);
    }
    int carry = -1;  // the last chunk listed by this root's children so far
    for (int c0 = cb; c0 < ce; c0 += 32) {
      const int ci = c0 + lane;
      bool surv = false;
      int size = 0;
      if (ci < ce) {
        const int c = ix.root_child_list[ci];
        surv = keep_all || !(__ldcg(ub_child + c) < T);
        size = surv ? ix.leaf_sizes[c] : 0;
      }
      if (chunk_mark) {
        int jlo = 0, jhi = -1;
        if (size > 0) {
          const uint32_t x = (uint32_t)__ldg(&ix.all_ranges[ci].x);
          jlo = (int)(x / cr);
          jhi = (int)min((x + (uint32_t)size - 1u) / cr, n_scan_chunks - 1u);
        }
        // the last chunk covered by this root's surviving children before this lane
        int m = jhi;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int t = __shfl_up_sync(FULL_MASK, m, o);
          if (lane >= o) m = max(m, t);
        }
        int before = __shfl_up_sync(FULL_MASK, m, 1);
        before = max(lane == 0 ? -1 : before, carry);
        carry = max(carry, __shfl_sync(FULL_MASK, m, 31));
        if (size > 0) jlo = max(max(jlo, before + 1), (int)frontier);  // chunks below the frontier are held
        const int cnt = jhi >= jlo ? jhi - jlo + 1 : 0;
        const int steps = __reduce_max_sync(FULL_MASK, cnt);
        for (int t0 = 0; t0 < steps; t0 += 8) {
          bool fresh[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint32_t j = (uint32_t)(jlo + t0 + u);
            bool ok = t0 + u < cnt;
            if (ok && (j * cr < r_lo || (j + 1u) * cr > r_hi)) ok = atomicExch(chunk_mark + j, epoch) != epoch;
            fresh[u] = ok;
          }
          uint32_t bal[8], total = 0u;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            bal[u] = __ballot_sync(FULL_MASK, fresh[u]);
            total += (uint32_t)__popc(bal[u]);
          }
          if (total == 0u) continue;
          // the first entries fill the shared staging up to LIST_SMEM, the
          // others go straight to the list (their own reservation): no slot
          // of either is left unused, so the list holds at most n_scan_chunks
          uint32_t at = 0u, gat = 0u;
          if (lane == 0) at = atomicAdd(&s_nlist, total);
          at = __shfl_sync(FULL_MASK, at, 0);
          const uint32_t n_sm = at < LIST_SMEM ? min(total, LIST_SMEM - at) : 0u;
          if (lane == 0 && total > n_sm) gat = atomicAdd(&sync->n_live, total - n_sm);
          gat = __shfl_sync(FULL_MASK, gat, 0);
          uint32_t idx = 0u;  // entries of this batch before the current step
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            if (fresh[u]) {
              const uint32_t e = idx + (uint32_t)__popc(bal[u] & lanemask_lt());
              if (e < n_sm) {
                s_list[at + e] = jlo + t0 + u;
              } else if (gat + (e - n_sm) < n_scan_chunks) {
                live_list[gat + (e - n_sm)] = jlo + t0 + u;
              } else {
                atomicOr(&ctrl->error, ERR_BAD_RANGE);  // (cannot happen: every chunk is listed once)
              }
            }
            idx += (uint32_t)__popc(bal[u]);
          }
        }
      }
      surv_children += (uint32_t)__popc(__ballot_sync(FULL_MASK, surv));
      surv_rows += (uint32_t)__shfl_sync(FULL_MASK, warp_incl_scan(size, lane), 31);
    }
  }
  if (lane == 0) {
    if (surv_roots) atomicAdd(&s_roots, surv_roots);
    if (surv_children) atomicAdd(&s_children, surv_children);
    if (surv_rows) atomicAdd(&s_rows, surv_rows);
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // one update of each trace counter and one list append per CTA
    if (s_roots) atomicAdd(&ctrl->n_surv_roots, s_roots);
    if (s_children) {
      atomicAdd(&ctrl->n_surv_children, s_children);
      atomicAdd(&ctrl->main_packed, ((unsigned long long)s_children << 32) | (unsigned long long)s_rows);
    }
    const uint32_t n = min(s_nlist, LIST_SMEM);
    s_base = (chunk_mark && n) ? atomicAdd(&sync->n_live, n) : 0u;
  }
  if (!chunk_mark) return;
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < min(s_nlist, LIST_SMEM); i += blockDim.x) {
    if (s_base + i < n_scan_chunks) live_list[s_base + i] = s_list[i];
    else atomicOr(&ctrl->error, ERR_BAD_RANGE);  // (cannot happen: every chunk is listed once)
  }
  __threadfence();  // each thread's list entries reach the GPU before the CTA's ticket
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(&sync->bounds_done, 1u) == gridDim.x - 1) {
    __threadfence();  // every CTA's entries (fenced before its ticket) before the signal
    atomicAdd(&sync->chunk_claims, 1ull << 32);
  }
}


// ============================================================ index preparation
// Per root: an upper bound of ||c_r|| and of ||V_r^T V_r - I||_2 (Frobenius norm
// of the Gram defect, accumulated in fp64 with an absolute slack per entry).
__global__ void k_prepare_roots(IndexView ix, double* __restrict__ root_cn, double* __restrict__ root_defect) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int p = blockIdx.x * (blockDim.x >> 5) + warp;
  if (p >= ix.R) return;
  const int D = ix.D, r = ix.rank;
  const float* c = ix.root_centers + (size_t)p * D;
  double acc = 0.0;
  for (int d = lane; d < D; d += 32) acc += (double)c[d] * (double)c[d];
  acc = warp_sum_d(acc);
  const float* V = ix.bases + (size_t)p * D * r;
  double fro = 0.0;
  const int npairs = r * (r + 1) / 2;
  for (int t = lane; t < npairs; t += 32) {
    int j = 0, rem = t;
    while (rem >= r - j) { rem -= r - j; ++j; }
    const int kk = j + rem;
    double g = 0.0, ga = 0.0;
    for (int d = 0; d < D; ++d) {
      const double x = (double)V[(size_t)d * r + j] * (double)V[(size_t)d * r + kk];
      g += x;
      ga += fabs(x);
    }
    const double e = fabs(g - (j == kk ? 1.0 : 0.0)) + 1e-13 * (1.0 + ga);
    fro += (j == kk ? 1.0 : 2.0) * e * e;
  }
  fro = warp_sum_d(fro);
  if (lane == 0) {
    root_cn[p] = sqrt(acc) * (1.0 + 1e-12) + 1e-30;
    root_defect[p] = sqrt(fro) * (1.0 + 1e-12) + 1e-30;
  }
}

// ============================================================ host launchers
int sm_count(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
  return n;
}

static int vpl_bucket(int D4) {
  const int v = (D4 + 31) / 32;
  if (v <= 1) return 1;
  if (v <= 2) return 2;
  if (v <= 3) return 3;
  if (v <= 4) return 4;
  if (v <= 6) return 6;
  if (v <= 8) return 8;
  if (v <= 12) return 12;
  return 16;
}
static int kcap_bucket(int k) { return k <= 32 ? 32 : (k <= 128 ? 128 : 256); }
static int rows_per_stage(int vpl) { return vpl <= 4 ? 32 : (vpl <= 8 ? 16 : 8); }
static int sortn_for(int kcap) { return kcap + 64 <= 128 ? 128 : (kcap + 64 <= 256 ? 256 : 512); }
// Rows per CTA below which a scan uses fewer CTAs: 64 (one to eight stages),
// so that every CTA's k-th best (k <= 32) is a useful threshold.
constexpr int SCAN_MIN_ROWS = 64;
static int stages_for(int vpl, int row_bytes) {
  const size_t sb = align_up((size_t)rows_per_stage(vpl) * row_bytes, 128);
  int s = (int)(147456 / sb);
  return s < 2 ? 2 : (s > MAX_STAGES ? MAX_STAGES : s);
}

int overlap_chunk_rows(int N, int D, int grid) {
  const long long rows = rows_per_stage(vpl_bucket(D / 4));
  const long long parts = (long long)(grid > 0 ? grid : 1) * SCAN_DYN_CHUNKS;
  const long long per = ((long long)N + parts - 1) / parts;
  const long long c = (per + rows - 1) / rows * rows;
  return (int)(c > 4 * rows ? c : 4 * rows);
}

int scan_smem_bytes(int D) {
  const int vpl = vpl_bucket(D / 4);
  const ScanLayout L = scan_layout(rows_per_stage(vpl), D * 4, stages_for(vpl, D * 4), sortn_for(256), 256);
  return (int)L.total;
}

// Launches `kern` as a programmatic dependent of the previous kernel on `stream`
// (it may start while that kernel runs and waits in griddep_wait()).
template <typename... KArgs, typename... Args>
static cudaError_t launch_dependent(void (*kern)(KArgs...), int grid, int block, size_t smem, cudaStream_t stream,
                                    Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <int VPL, int KCAP>
static cudaError_t launch_scan_t(const ScanParams& P0, int grid, cudaStream_t stream) {
  // as many ring stages as the shared-memory budget leaves after the top-k areas
  constexpr size_t SMEM_BUDGET = 225 * 1024;
  ScanParams P = P0;
  const size_t fixed = scan_layout(ScanShape<VPL>::ROWS, P.row_bytes, 0, TopkShape<KCAP>::SORTN, KCAP).total;
  const size_t sb = align_up((size_t)ScanShape<VPL>::ROWS * P.row_bytes, 128);
  int st = (int)((SMEM_BUDGET - fixed) / sb);
  P.stages = st < 2 ? 2 : (st > MAX_STAGES ? MAX_STAGES : st);
  const ScanLayout L = scan_layout(ScanShape<VPL>::ROWS, P.row_bytes, P.stages, TopkShape<KCAP>::SORTN, KCAP);
  static SmemOptIn opt_in;  // per instantiation, per device
  cudaError_t e = opt_in.ensure(reinterpret_cast<const void*>(k_scan<VPL, KCAP>), (int)L.total);
  if (e != cudaSuccess) return e;
  return launch_dependent(k_scan<VPL, KCAP>, grid, SCAN_THREADS, L.total, stream, P);
}

template <int VPL>
static cudaError_t launch_scan_v(const ScanParams& P, int grid, cudaStream_t stream) {
  const int kc = kcap_bucket(P.k);
  if (kc == 32) return launch_scan_t<VPL, 32>(P, grid, stream);
  if (kc == 128) return launch_scan_t<VPL, 128>(P, grid, stream);
  return launch_scan_t<VPL, 256>(P, grid, stream);
}

static cudaError_t launch_scan(const ScanParams& P, int grid, cudaStream_t stream) {
  switch (vpl_bucket(P.D4)) {
    case 1: return launch_scan_v<1>(P, grid, stream);
    case 2: return launch_scan_v<2>(P, grid, stream);
    case 3: return launch_scan_v<3>(P, grid, stream);
    case 4: return launch_scan_v<4>(P, grid, stream);
    case 6: return launch_scan_v<6>(P, grid, stream);
    case 8: return launch_scan_v<8>(P, grid, stream);
    case 12: return launch_scan_v<12>(P, grid, stream);
    default: return launch_scan_v<16>(P, grid, stream);
  }
}

static int bounds_chunk_rows(int D, int rank) {
  int rows = (12288 / (rank * 4)) & ~3;
  if (rows < 4) rows = 4;
  const int Dr = (D + 3) & ~3;
  return rows > Dr ? Dr : rows;
}

cudaError_t launch_prepare_roots(const IndexView& ix, double* root_cn, double* root_defect, cudaStream_t stream) {
  const int warps = 4;
  k_prepare_roots<<<(ix.R + warps - 1) / warps, warps * 32, 0, stream>>>(ix, root_cn, root_defect);
  return cudaGetLastError();
}

// CTAs that take part in a scan of n rows on `grid` CTAs (the kernel's G)
static int scan_ctas(int n, int grid) {
  const int g = (n + SCAN_MIN_ROWS - 1) / SCAN_MIN_ROWS;
  return g < 1 ? 1 : (g < grid ? g : grid);
}

static ScanParams scan_params(const IndexView& ix, const Workspace& ws, const float* q, int k, float* out_scores,
                              int* out_ids, long long* out_rows) {
  ScanParams P{};
  P.leaf = ix.leaf;
  P.q = q;
  P.theta_key = &ws.ctrl->theta_key;
  P.cta_lists = ws.cta_lists;
  P.err = &ws.ctrl->error;
  P.D4 = ix.D4;
  P.row_bytes = ix.D * 4;
  P.k = k;
  P.stages = stages_for(vpl_bucket(ix.D4), P.row_bytes);
  P.min_rows = SCAN_MIN_ROWS;
  P.chunk_counter = &ws.ctrl->chunk_next;
  P.out_scores = out_scores;
  P.out_ids = out_ids;
  P.out_rows = out_rows;
  P.original_ids = ix.original_ids;
  return P;
}

// First kernel of a search (an ordinary launch, so it starts only after the
// previous search on the stream has finished with the workspace): clears the
// control header; with io, also stages the query (see HostIO).
static cudaError_t search_reset(const IndexView& ix, const Workspace& ws, const float* q, cudaStream_t stream,
                                const HostIO* io) {
  k_search_prologue<<<1, 128, 0, stream>>>(io ? reinterpret_cast<const float4*>(io->q_host) : nullptr,
                                           io ? io->slots : nullptr,
                                           reinterpret_cast<float4*>(const_cast<float*>(q)), ix.D4,
                                           reinterpret_cast<unsigned long long*>(ws.ctrl),
                                           io ? io->out_indirect : nullptr, io ? io->seq_in : nullptr,
                                           ws.epoch_counter, reinterpret_cast<unsigned long long*>(ws.sync));
  return cudaGetLastError();
}

static void final_io(ScanParams& M, const Workspace& ws, const HostIO* io) {
  if (!io) return;
  M.out_indirect = io->slots ? io->out_indirect : nullptr;
  M.ctrl_hdr = reinterpret_cast<const unsigned long long*>(ws.ctrl);
  M.ctrl_out = reinterpret_cast<unsigned long long*>(io->ctrl_out);
  M.call_seq = &ws.ctrl->call_seq;
  M.done_out = io->done_out;
}

cudaError_t launch_search_seed(const IndexView& ix, const Workspace& ws, const float* q, int k, float* T_export,
                               cudaStream_t stream, const HostIO* io) {
  cudaError_t e = search_reset(ix, ws, q, stream, io);
  if (e != cudaSuccess) return e;
  const RootScanLayout RL = root_scan_layout(ix.D * 4);
  static SmemOptIn root_opt_in;
  if ((e = root_opt_in.ensure(reinterpret_cast<const void*>(k_root_scan), (int)RL.total)) != cudaSuccess) return e;
  int grid = (ix.R + ROOT_SCAN_WARPS - 1) / ROOT_SCAN_WARPS;
  if (grid > ws.scan_grid) grid = ws.scan_grid;
  return launch_dependent(k_root_scan, grid, ROOT_SCAN_WARPS * 32, RL.total, stream, ix, q, ws.ctrl, k, T_export);
}

cudaError_t launch_search_finish(const IndexView& ix, const Workspace& ws, const float* q, int k, const float* T_ext,
                                 float* out_scores, int* out_ids, long long* out_rows, cudaStream_t stream,
                                 cudaEvent_t ev_scan0, cudaEvent_t ev_scan1, const HostIO* io,
                                 const SharedThreshold* shared) {
  cudaError_t e;
  const int chunk_rows = bounds_chunk_rows(ix.D, ix.rank);
  const BoundsLayout BL = bounds_layout(ix.D, ix.rank, chunk_rows);
  static SmemOptIn bounds_opt_in;
  if ((e = bounds_opt_in.ensure(reinterpret_cast<const void*>(k_bounds), (int)BL.total)) != cudaSuccess) return e;
  int grid_b = (ix.R + BOUNDS_WARPS - 1) / BOUNDS_WARPS;
  if (grid_b > 2 * ws.scan_grid) grid_b = 2 * ws.scan_grid;
  if ((e = launch_dependent(k_bounds, grid_b, BOUNDS_WARPS * 32, BL.total, stream, ix, q, ws.ctrl, ws.ub_root,
                            ws.ub_child, ws.ub_tagged, chunk_rows, T_ext, (uint32_t)ws.chunk_rows,
                            (uint32_t)ws.n_chunks, ws.chunk_mark, ws.live_list,
                            (uint32_t)scan_ctas(ix.N, ws.scan_grid), ws.sync)) != cudaSuccess)
    return e;
  ScanParams M = scan_params(ix, ws, q, k, out_scores, out_ids, out_rows);
  M.ranges = ix.all_ranges;
  M.packed_counts = ix.all_packed;
  M.packed_value = ((unsigned long long)ix.all_nnz << 32) | (unsigned long long)(uint32_t)ix.N;
  M.done = &ws.ctrl->main_done;
  M.ub_tagged = ws.ub_tagged;
  M.epoch = &ws.ctrl->epoch;
  M.chunk_first_range = ws.chunk_first_range;
  M.chunk_rows = (uint32_t)ws.chunk_rows;
  M.chunk_claims = &ws.sync->chunk_claims;
  M.live_list = ws.live_list;
  M.n_live = &ws.sync->n_live;
  M.list_next = &ws.sync->list_next;
  M.chunk_taken = ws.chunk_taken;
  if (shared && shared->local) {
    M.xth_local = shared->local;
    M.xth_peers = shared->peers;
    M.n_peers = shared->peers ? shared->n_peers : 0;
    M.xth_tag = shared->tag;
  }
  M.T_ext = T_ext;
  M.rows_streamed = &ws.ctrl->rows_streamed;
  M.overlapped = 1;
  final_io(M, ws, io);
  if (ev_scan0) cudaEventRecord(ev_scan0, stream);
  e = launch_scan(M, ws.scan_grid, stream);
  if (ev_scan1) cudaEventRecord(ev_scan1, stream);
  return e;
}

cudaError_t launch_search(const IndexView& ix, const Workspace& ws, const float* q, int k, int hierarchical,
                          float* out_scores, int* out_ids, long long* out_rows, cudaStream_t stream,
                          cudaEvent_t ev_scan0, cudaEvent_t ev_scan1, const HostIO* io) {
  if (hierarchical) {
    cudaError_t e = launch_search_seed(ix, ws, q, k, nullptr, stream, io);
    if (e != cudaSuccess) return e;
    return launch_search_finish(ix, ws, q, k, nullptr, out_scores, out_ids, out_rows, stream, ev_scan0, ev_scan1,
                                io);
  }
  cudaError_t e = search_reset(ix, ws, q, stream, io);
  if (e != cudaSuccess) return e;
  ScanParams F = scan_params(ix, ws, q, k, out_scores, out_ids, out_rows);
  F.ranges = ws.flat_range;
  F.packed_counts = ws.flat_packed;
  F.packed_value = (1ull << 32) | (unsigned long long)(uint32_t)ix.N;
  F.done = &ws.ctrl->main_done;
  final_io(F, ws, io);
  if (ev_scan0) cudaEventRecord(ev_scan0, stream);
  e = launch_scan(F, ws.scan_grid, stream);
  if (ev_scan1) cudaEventRecord(ev_scan1, stream);
  return e;
}

cudaError_t launch_flat_scan(const float* leaf, int D, int N, const float* q, int k, int grid, SearchCtrl* ctrl,
                             const int4* range, const unsigned long long* packed, unsigned long long* cta_lists,
                             float* out_scores, int* out_ids, cudaStream_t stream) {
  const int vpl = vpl_bucket(D / 4);
  ScanParams F{};
  F.leaf = leaf;
  F.q = q;
  F.ranges = range;
  F.packed_counts = packed;
  F.theta_key = &ctrl->theta_key;
  F.cta_lists = cta_lists;
  F.done = &ctrl->main_done;
  F.err = &ctrl->error;
  F.D4 = D / 4;
  F.row_bytes = D * 4;
  F.k = k;
  F.stages = stages_for(vpl, F.row_bytes);
  F.min_rows = SCAN_MIN_ROWS;
  F.chunk_counter = &ctrl->chunk_next;
  F.out_scores = out_scores;
  F.out_ids = out_ids;
  F.out_rows = nullptr;
  F.original_ids = nullptr;
  (void)N;
  return launch_scan(F, grid, stream);
}

}  // namespace cb
