// Batched exact top-k search on the B200 tensor cores.
//
// k_query_bands  warp per query: the error band 2 eps (below) of each query.
// k_batch_scan  persistent CTA pairs (clusters of 2, one CTA per SM) computing
//               the score matrix Q X^T tile by tile with 2-SM tcgen05 MMAs
//               (cta_group::2, kind::tf32, M = 256 queries, N = 256 leaf rows,
//               K = 8) and filtering it in the epilogue; no score matrix is
//               ever written.  A work unit is (query tile of 256 queries, slice
//               of 8,192 leaf rows); units are taken in slice-major order from
//               a global counter (dynamic scheduling), so the units in flight
//               share a few consecutive slices and every leaf row comes from
//               HBM about once, then from L2.  Launched twice per batch: a
//               threshold pass over up to 32,768 evenly spaced rows (one unit
//               per query tile, no candidates), then the main pass.
//               - a TMA warp per CTA streams 32-column K-chunks of its 128
//                 queries and of its 128 leaf rows of the tile (fp32, 128-byte
//                 swizzle) through a 6-stage shared-memory ring; completion is
//                 counted on the even CTA's barrier;
//               - the even CTA's MMA warp issues the pair's MMAs (both operands
//                 from shared memory) into one of two 256-column TMEM
//                 accumulators and commits to the barriers of both CTAs, so the
//                 epilogue of tile t overlaps the MMAs of tile t + 1; its issue
//                 loop is kept lean (one MMA instruction takes only ~70 ns);
//               - each epilogue thread owns one query: it reads its 256 scores
//                 with tcgen05.ld, and appends every row whose tf32 score is
//                 within `band` of the query's running threshold to the
//                 query's candidate list, with its tf32 score.  The threshold
//                 is always the tf32 score of the k-th best of k distinct rows:
//                 for k <= 32 a per-thread top-k in registers plus rotated
//                 per-query slots; for larger k, 4k slots keyed by row whose
//                 k-th largest a seventh warp per CTA keeps published (see
//                 threshold_sweeps).
//               Both operands are streamed: with the queries resident in TMEM
//               (384 of 512 columns at D = 384) only N = 64 accumulators fit,
//               4x the MMA instructions per flop of N = 256.
// k_batch_rescore  one CTA per query: threshold = max(final scan threshold, the
//               k-th best tf32 score among its own candidates); drops the
//               candidates below it minus the band, scores the rest exactly in
//               fp32 (the same arithmetic as the single-query scan, so both
//               paths return identical scores), radix select, original ids.
//
// Exactness: with eps >= |tf32 score - fp32 score| for every row (bound:
// (2^-9 + 2^-20 + 2D 2^-23 + gamma_D) ||q|| max||x||, tf32 truncation of both
// operands plus fp32 accumulation), any row in the fp32 top-k has tf32 score
// >= s_k - eps, and any running k-th best tf32 score is <= s_k + eps, so
// band = 2 eps never drops a top-k row.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <string>

#include "common.cuh"
#include "engine.h"
#include "tcgen05.cuh"
#include "topk.cuh"

namespace cb {

constexpr int BQ = 128;                  // queries per CTA (UMMA M = 256 per CTA pair)
constexpr int BN = 256;                  // leaf rows per tile (UMMA N); each CTA loads 128
constexpr int HALF_N = BN / 2;
constexpr int EPI_COLS = 64;             // accumulator columns per epilogue pass
constexpr int BATCH_THREADS = 192;       // warps 0-3 epilogue, 4 TMA, 5 MMA
constexpr int BATCH_THREADS_SLOTS = 224; // k > 32: + warp 6, the threshold warp
constexpr int THRESHOLD_MAX_SWEEPS = 1 << 24;  // bound of the threshold warp's loop
constexpr int BATCH_MAX_STAGES = 8;
constexpr int SLICE_ROWS = 8192;         // rows per work unit of the main pass
constexpr int SEED_ROWS = 32768;         // rows of the threshold pass (one unit per query tile)
constexpr int BATCH_SEED_MIN_N = 65536;  // smaller corpora skip the threshold pass
constexpr int A_BYTES = BQ * 128;        // 128 query rows x 32 floats
constexpr int B_BYTES = HALF_N * 128;    // 128 leaf rows x 32 floats
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;

constexpr int UNIT_RING = 4;             // unit ids published ahead of their consumers

struct BatchScanParams {
  const float* Q;        // [B, D]
  int B, D, N, k;
  int kb;                // K-chunks of 32 columns = ceil(D / 32)
  int stages;            // shared-memory ring depth (<= BATCH_MAX_STAGES)
  int QP, units;         // query pair-tiles (256 queries), work units
  float band_scale;      // band = band_scale * ||q||
  const float* qband;    // [B] band of each query (k_query_bands)
  uint32_t* theta;       // [B] order-preserving keys of the running k-th best
  int* cand_count;       // [B]
  unsigned long long* cand;  // [B * cap]: tf32 score key << 32 | leaf row
  int cap;
  int* err;
  int seed_only;         // threshold pass: raise theta, append no candidates
  uint32_t* slots;       // [B * nslots] per-query threshold slots
  int nslots;            // slots per query (batch_slot_count(k))
  int row_step;          // leaf row = scan row * row_step (threshold pass: sampled rows)
  int* unit_counter;     // next work unit (dynamic scheduling; zeroed before the launch)
  int slice_rows;        // rows per work unit
};

// Top-k variant (k <= 32): one epilogue pass over 64 accumulator columns (leaf
// rows row_base + i) of this thread's query; the thread's k best tf32 scores are
// kept sorted in `top`, so its threshold rises with every insertion.
template <int KB>
__device__ __forceinline__ void epi_pass_topk(const uint32_t (&sc0)[32], const uint32_t (&sc1)[32], int row_base, int nrow,
                                         float band, float& theta, float& theta_local, float (&top)[KB], int q,
                                         float* stash, const BatchScanParams& P) {
  const float lim = theta - band;
  uint64_t mask = 0ull;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    mask |= (uint64_t)(__uint_as_float(sc0[i]) >= lim) << i;
    mask |= (uint64_t)(__uint_as_float(sc1[i]) >= lim) << (32 + i);
  }
  if (nrow < EPI_COLS) mask &= nrow > 0 ? (1ull << nrow) - 1ull : 0ull;
  if (!mask) return;
  // rare: stage the scores ([column][thread], conflict-free), first raise the
  // k best with them, then append the rows still within the band
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    stash[i * BQ + threadIdx.x] = __uint_as_float(sc0[i]);
    stash[(32 + i) * BQ + threadIdx.x] = __uint_as_float(sc1[i]);
  }
  for (uint64_t m = mask; m; m &= m - 1ull) {
    const int i = __ffsll((long long)m) - 1;
    const float sv = stash[i * BQ + threadIdx.x];
    if (sv > theta_local) {
      float x = sv;
#pragma unroll
      for (int j = 0; j < KB; ++j) {
        const float t = top[j];
        const bool gt = x > t;
        top[j] = gt ? x : t;
        x = gt ? t : x;
      }
      float kth = top[0];
#pragma unroll
      for (int j = 0; j < KB; ++j)
        if (j == P.k - 1) kth = top[j];
      theta_local = kth;
    }
  }
  theta = fmaxf(theta, theta_local);
  if (P.seed_only) return;
  // the candidates: one reservation in the query's list for all of them
  const float lim2 = theta - band;
  uint64_t keep = 0ull;
  for (uint64_t m = mask; m; m &= m - 1ull) {
    const int i = __ffsll((long long)m) - 1;
    if (stash[i * BQ + threadIdx.x] >= lim2) keep |= 1ull << i;
  }
  if (!keep) return;
  int slot = atomicAdd(P.cand_count + q, __popcll(keep));
  for (uint64_t m = keep; m; m &= m - 1ull, ++slot) {
    const int i = __ffsll((long long)m) - 1;
    if (slot < P.cap)
      P.cand[(size_t)q * P.cap + slot] =
          ((unsigned long long)f2key(stash[i * BQ + threadIdx.x]) << 32) | (uint32_t)(row_base + i);
  }
}

// Per-query threshold from 4k slots (k > 32).  Leaf row r publishes its tf32
// score key into slot r mod nslots by atomicMax (0 = a slot not yet filled).
// The slots cover disjoint sets of rows, so each holds the score of one real
// row and no row is in two slots: the k-th largest slot is the k-th best of k
// distinct rows, a valid threshold.  A row always maps to the same slot, so
// rows seen twice (the threshold pass samples rows that the main pass scans
// again) cannot count twice.  With nslots = 4k the k-th largest slot sits near
// the 1.15k-th best row seen (k of 4k residue classes are hit among the top
// 4k ln(4/3) rows), where the minimum of k slots (one per residue mod k) sits
// near the k ln k-th.
//
// Warp 6 of every CTA keeps the published thresholds current: it refreshes
// queries blockIdx.x, blockIdx.x + gridDim.x, ... in turn, loading a query's
// slots (PL per lane, coalesced, through L2: other CTAs raise them) while it
// selects the previous query's k-th largest, by bisection on the key bits with
// one warp-wide count per bit.  A query with fewer than k slots above its
// published key is skipped after one count.  The epilogue threads only raise
// slots and read the published key one tile ahead, so no L2 round trip sits on
// their path.  The warp stops when the CTA's epilogue has finished (`done`) or
// after THRESHOLD_MAX_SWEEPS sweeps; a stale threshold only costs candidates.
template <int PL>
__device__ __forceinline__ void load_slots(const uint32_t* sl, int per, int lane, uint32_t (&v)[PL]) {
#pragma unroll
  for (int i = 0; i < PL; ++i) v[i] = i < per ? __ldcg(sl + 32 * i + lane) : 0u;
}

template <int PL>
__device__ void threshold_sweeps(const BatchScanParams& P, const volatile int* done) {
  const int lane = threadIdx.x & 31;
  const int per = P.nslots >> 5;
  const int q0 = (int)blockIdx.x, dq = (int)gridDim.x;
  if (q0 >= P.B) return;
  uint32_t v[PL], nv[PL];
  // the stop decision is made warp-wide: every lane must reach each redux.sync
  for (int sweep = 0; sweep < THRESHOLD_MAX_SWEEPS && !__any_sync(FULL_MASK, *done != 0); ++sweep) {
    load_slots<PL>(P.slots + (size_t)q0 * P.nslots, per, lane, nv);
    for (int q = q0; q < P.B; q += dq) {
#pragma unroll
      for (int i = 0; i < PL; ++i) v[i] = nv[i];
      const uint32_t cur = ld_volatile_u32(P.theta + q);
      if (q + dq < P.B) load_slots<PL>(P.slots + (size_t)(q + dq) * P.nslots, per, lane, nv);
      // empty slots (0) never count: cur >= 0 and every probe below is >= 1
      int c = 0;
#pragma unroll
      for (int i = 0; i < PL; ++i) c += v[i] > cur;
      if (__reduce_add_sync(FULL_MASK, (unsigned)c) < (unsigned)P.k) continue;
      // largest x with #{slots >= x} >= k, i.e. the k-th largest slot (> cur)
      uint32_t x = 0u;
#pragma unroll 1
      for (int bit = 31; bit >= 0; --bit) {
        const uint32_t t = x | (1u << bit);
        int n = 0;
#pragma unroll
        for (int i = 0; i < PL; ++i) n += v[i] >= t;
        if (__reduce_add_sync(FULL_MASK, (unsigned)n) >= (unsigned)P.k) x = t;
      }
      if (lane == 0 && x > cur) atomicMax(P.theta + q, x);
      if (__any_sync(FULL_MASK, *done != 0)) break;
    }
    __nanosleep(500);
  }
}

// One epilogue pass over 64 accumulator columns (rows row_base + i of the scan's
// row space) of this thread's query: rows within `band` of the threshold are
// appended as candidates (main pass), rows above it raise their slot.
__device__ __forceinline__ void epi_pass(const uint32_t (&sc0)[32], const uint32_t (&sc1)[32], int row_base, int nrow,
                                         float band, float theta, int q, float* stash, const BatchScanParams& P) {
  const float lim = theta - band;
  uint64_t mask = 0ull;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    mask |= (uint64_t)(__uint_as_float(sc0[i]) >= lim) << i;
    mask |= (uint64_t)(__uint_as_float(sc1[i]) >= lim) << (32 + i);
  }
  if (nrow < EPI_COLS) mask &= nrow > 0 ? (1ull << nrow) - 1ull : 0ull;
  if (!mask) return;
  // rare: stage the scores ([column][thread], conflict-free) and walk the rows
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    stash[i * BQ + threadIdx.x] = __uint_as_float(sc0[i]);
    stash[(32 + i) * BQ + threadIdx.x] = __uint_as_float(sc1[i]);
  }
  uint32_t* sl = P.slots + (size_t)q * P.nslots;
  // every row of the mask is a candidate: one reservation in the query's list
  int slot = P.seed_only ? 0 : atomicAdd(P.cand_count + q, __popcll(mask));
  for (uint64_t m = mask; m; m &= m - 1ull) {
    const int i = __ffsll((long long)m) - 1;
    const float sv = stash[i * BQ + threadIdx.x];
    const uint32_t key = f2key(sv);
    if (sv > theta) {  // a row below every slot cannot raise one
      const uint32_t leaf_row = (uint32_t)(row_base + i) * (uint32_t)P.row_step;
      atomicMax(sl + leaf_row % (uint32_t)P.nslots, key);
    }
    if (!P.seed_only) {
      if (slot < P.cap) P.cand[(size_t)q * P.cap + slot] = ((unsigned long long)key << 32) | (uint32_t)(row_base + i);
      ++slot;
    }
  }
}

// Launched as clusters of 2 CTAs.  CTA rank r of the pair loads queries
// [256 qp + 128 r, +128) and leaf rows [row0 + 128 r, +128) of every tile; the
// pair's accumulator holds, in CTA r's TMEM lanes, its 128 queries against all
// 256 rows of the tile (columns 0-127: rows loaded by the even CTA, 128-255:
// by the odd CTA).
// Dynamic work units.  The even CTA's producer takes the next unit from a global
// counter and publishes its id into a 4-deep ring in both CTAs' shared memory
// (full barriers, one arrival each); the odd CTA's producer, the MMA warp and
// the 8 epilogue warps take ids in order and release each slot on the even
// CTA's empty barrier (10 arrivals).  Units in flight across the GPU are then
// about 74 consecutive ids -- a few consecutive row slices -- so the rows of a
// slice are read from HBM about once and from L2 by its 16 query tiles, which
// static round-robin dealing lost as pairs drifted apart.  Id -1 ends the loops.
__device__ __forceinline__ int take_unit(uint64_t* unit_full, const int* ring, uint32_t lead_unit_empty, int& ui,
                                         bool warp_release, int* err) {
  const int r = ui & (UNIT_RING - 1);
  const uint32_t ph = (uint32_t)(ui / UNIT_RING) & 1u;
  ++ui;
  const bool got = tc::mbar_wait_cluster(&unit_full[r], ph, err, ERR_TIMEOUT_FULL);
  const int u = got ? *reinterpret_cast<const volatile int*>(ring + r) : -1;
  if (warp_release) __syncwarp();
  if (!warp_release || (threadIdx.x & 31) == 0) tc::mbar_arrive_cluster(lead_unit_empty + 8u * (uint32_t)r);
  return u;
}

// KB > 0: per-thread top-KB epilogue (k <= KB); KB == 0: slot thresholds (any
// k) kept published by the threshold warp (warp 6, BATCH_THREADS_SLOTS threads).
template <int KB>
__global__ void __launch_bounds__(KB == 0 ? BATCH_THREADS_SLOTS : BATCH_THREADS, 1)
    k_batch_scan(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap xmap,
                 BatchScanParams P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  // full / acc_empty are used in the even CTA only; empty / acc_full in both
  // (the even CTA's MMA thread commits to its own and to the odd CTA's copy).
  __shared__ uint64_t full[BATCH_MAX_STAGES], empty[BATCH_MAX_STAGES], acc_full[2], acc_empty[2], drain;
  __shared__ uint64_t unit_full[UNIT_RING], unit_empty[UNIT_RING];
  __shared__ int unit_ring[UNIT_RING];
  __shared__ uint32_t tmem_base;
  __shared__ int s_err;
  __shared__ int s_done;  // set once this CTA's epilogue has left its loop
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();
  const bool leader = rank == 0;
  const int S = P.stages;
  float* stash = reinterpret_cast<float*>(smem + (size_t)S * STAGE_BYTES);  // [64][BQ] scores

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // one lane of each epilogue warp of both CTAs
    }
    mbar_init(&drain, 1);
    s_done = 0;
    for (int r = 0; r < UNIT_RING; ++r) {
      mbar_init(&unit_full[r], 1);
      mbar_init(&unit_empty[r], 10);  // odd producer + MMA warp + 8 epilogue warps
    }
    tc::fence_mbar_init_cluster();
  }
  if (warp == 5) tc::tmem_alloc_pair(&tmem_base, 512);
  tc::fence_before();
  tc::cluster_sync();  // barriers and the pair's TMEM exist before any remote access
  tc::fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t lead_full = tc::mapa_shared(smem_u32(&full[0]), 0);
  const uint32_t lead_acc_empty = tc::mapa_shared(smem_u32(&acc_empty[0]), 0);
  const uint32_t empty0 = tc::mapa_shared(smem_u32(&empty[0]), 0), empty1 = tc::mapa_shared(smem_u32(&empty[0]), 1);
  const uint32_t accf0 = tc::mapa_shared(smem_u32(&acc_full[0]), 0), accf1 = tc::mapa_shared(smem_u32(&acc_full[0]), 1);
  const uint32_t lead_unit_empty = tc::mapa_shared(smem_u32(&unit_empty[0]), 0);

  if (warp == 4) {
    // ---------------------------------------------------------- TMA producer (both CTAs)
    // The stage index and its phase advance incrementally (no division in the loop).
    if (lane == 0) {
      int s = 0, c = 0, ui = 0;
      uint32_t ph = 0;
      bool ok = true;
      const uint32_t peer_ring = tc::mapa_shared(smem_u32(&unit_ring[0]), 1);
      const uint32_t peer_unit_full = tc::mapa_shared(smem_u32(&unit_full[0]), 1);
      while (ok) {
        int u;
        if (leader) {
          // publish the next unit into both CTAs' rings (-1: none left)
          const int r = ui & (UNIT_RING - 1), round = ui / UNIT_RING;
          ++ui;
          const bool free_slot =
              round == 0 || tc::mbar_wait_cluster(&unit_empty[r], (uint32_t)(round - 1) & 1u, P.err, ERR_TIMEOUT_EMPTY);
          const int n = free_slot ? atomicAdd(P.unit_counter, 1) : P.units;
          u = n < P.units ? n : -1;
          *reinterpret_cast<volatile int*>(&unit_ring[r]) = u;
          tc::st_cluster_s32(peer_ring + 4u * (uint32_t)r, u);
          mbar_arrive(&unit_full[r]);
          tc::mbar_arrive_cluster(peer_unit_full + 8u * (uint32_t)r);
        } else {
          u = take_unit(unit_full, unit_ring, lead_unit_empty, ui, false, P.err);
        }
        if (u < 0) break;
        const int qp = u % P.QP, slice = u / P.QP;
        const int qrow = qp * (2 * BQ) + (int)rank * BQ;
        const int r0 = slice * P.slice_rows, r1 = min(P.N, r0 + P.slice_rows);
        for (int row0 = r0; row0 < r1 && ok; row0 += BN) {
          const int xrow = row0 + (int)rank * HALF_N;
          for (int j = 0; j < P.kb; ++j, ++c) {
            if (c >= S && !mbar_wait(&empty[s], ph ^ 1u, P.err, ERR_TIMEOUT_EMPTY)) { ok = false; break; }
            if (leader) mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * STAGE_BYTES));
            unsigned char* dst = smem + (size_t)s * STAGE_BYTES;
            const uint32_t bar = lead_full + 8u * (uint32_t)s;
            tc::tma_load_2d_pair(dst, &qmap, 32 * j, qrow, bar);
            tc::tma_load_2d_pair(dst + A_BYTES, &xmap, 32 * j, xrow, bar);
            if (++s == S) { s = 0; ph ^= 1u; }
          }
        }
      }
      // the last commits to this CTA's empty barriers have landed before it exits
      for (int t = c > S ? c - S : 0; t < c && ok; ++t)
        ok = mbar_wait(&empty[t % S], (t / S) & 1, P.err, ERR_TIMEOUT_EMPTY);
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issuer (even CTA)
    // The whole warp runs the loop and one elected lane issues: a lean issue
    // loop matters, since one 2-SM MMA (M = N = 256, K = 8) takes only ~70 ns.
    // Descriptors are formed once and advanced by adding (byte offset >> 4) to
    // their start-address field (shared-memory addresses stay below 256 KB,
    // so the 14-bit field never carries).
    if (leader) {
      const uint32_t idesc = tc::idesc_tf32(2 * BQ, BN);
      const uint32_t sbase = smem_u32(smem);
      const uint64_t dA0 = tc::sdesc_k_sw128(sbase), dB0 = tc::sdesc_k_sw128(sbase + A_BYTES);
      int s = 0, it = 0, ui = 0;
      uint32_t ph = 0;
      bool ok = true;
      while (ok) {
        const int u = __shfl_sync(FULL_MASK, take_unit(unit_full, unit_ring, lead_unit_empty, ui, true, P.err), 0);
        if (u < 0) break;
        const int slice = u / P.QP;
        const int r0 = slice * P.slice_rows, r1 = min(P.N, r0 + P.slice_rows);
        for (int row0 = r0; row0 < r1 && ok; row0 += BN, ++it) {
          const int b = it & 1, fb = it >> 1;
          // wait results are made warp-uniform: elect.sync needs every lane
          if (fb > 0 &&
              !__all_sync(FULL_MASK, tc::mbar_wait_cluster(&acc_empty[b], (fb - 1) & 1, P.err, ERR_TIMEOUT_EMPTY))) {
            ok = false;
            break;
          }
          tc::fence_after();
          const uint32_t acc = tmem + (uint32_t)(b * BN);
          for (int j = 0; j < P.kb; ++j) {
            if (!__all_sync(FULL_MASK, mbar_wait(&full[s], ph, P.err, ERR_TIMEOUT_FULL))) { ok = false; break; }
            tc::fence_after();
            if (tc::elect_one()) {
              const uint64_t off = (uint64_t)(((uint32_t)s * (uint32_t)STAGE_BYTES) >> 4);
              const uint64_t a = dA0 + off, bq = dB0 + off;
              tc::mma_tf32_ss_pair(acc, a, bq, idesc, j != 0 ? 1u : 0u);
              tc::mma_tf32_ss_pair(acc, a + 2, bq + 2, idesc, 1u);
              tc::mma_tf32_ss_pair(acc, a + 4, bq + 4, idesc, 1u);
              tc::mma_tf32_ss_pair(acc, a + 6, bq + 6, idesc, 1u);
              // both CTAs' stage s refills once these MMAs have read it
              tc::commit_pair(empty0 + 8u * (uint32_t)s);
              tc::commit_pair(empty1 + 8u * (uint32_t)s);
            }
            __syncwarp();
            if (++s == S) { s = 0; ph ^= 1u; }
          }
          if (ok && tc::elect_one()) {
            tc::commit_pair(accf0 + 8u * (uint32_t)b);
            tc::commit_pair(accf1 + 8u * (uint32_t)b);
          }
          __syncwarp();
        }
      }
    }
  } else if (warp == 6) {
    // ---------------------------------------------------------- threshold warp (k > 32 only)
    if constexpr (KB == 0) {
      const volatile int* done = &s_done;
      if (P.nslots <= 8 * 32) threshold_sweeps<8>(P, done);
      else if (P.nslots <= 16 * 32) threshold_sweeps<16>(P, done);
      else threshold_sweeps<32>(P, done);
    }
  } else {
    // ---------------------------------------------------------- epilogue (one query per thread)
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    int it = 0, ui = 0;
    bool ok = true;
    while (ok) {
      const int u = __shfl_sync(FULL_MASK, take_unit(unit_full, unit_ring, lead_unit_empty, ui, true, P.err), 0);
      if (u < 0) break;
      const int qp = u % P.QP, slice = u / P.QP;
      const int q = qp * (2 * BQ) + (int)rank * BQ + 32 * warp + lane;
      const bool qv = q < P.B;
      if constexpr (KB > 0) {
      const float band = qv ? __ldg(P.qband + q) : 0.f;
      float top[KB];
#pragma unroll
      for (int i = 0; i < KB; ++i) top[i] = -INFINITY;
      float theta_local = -INFINITY;
      uint32_t g_key = qv ? ld_volatile_u32(P.theta + q) : 0u;
      uint32_t g_pending = g_key;
      float theta = g_key ? key2f(g_key) : -INFINITY;
      uint32_t published = 0;
      const int r0 = slice * P.slice_rows, r1 = min(P.N, r0 + P.slice_rows);
      int tiles = 0;
      for (int row0 = r0; row0 < r1; row0 += BN, ++it, ++tiles) {
        const int b = it & 1, fb = it >> 1;
        if (!mbar_wait(&acc_full[b], fb & 1, P.err, ERR_TIMEOUT_FULL)) { ok = false; break; }
        tc::fence_after();
        if (qv) {
          // global threshold read one tile ahead (its latency overlaps this tile)
          if (g_pending) theta = fmaxf(theta, key2f(g_pending));
          g_pending = ld_volatile_u32(P.theta + q);
        }
        // two halves of 128 columns: all four loads of a half issued before one
        // wait; the common case is one max per score and one compare per half
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          uint32_t sa[32], sb[32], sc[32], sd[32];
          const uint32_t col = tmem + lane_base + (uint32_t)(b * BN + half * 128);
          tc::ld_32x32b_x32(col, sa);
          tc::ld_32x32b_x32(col + 32, sb);
          tc::ld_32x32b_x32(col + 64, sc);
          tc::ld_32x32b_x32(col + 96, sd);
          tc::wait_ld();
          if (half == 1) {
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive_remote(lead_acc_empty + 8u * (uint32_t)b);
          }
          if (!qv) continue;
          float mx[32];
#pragma unroll
          for (int i = 0; i < 32; ++i)
            mx[i] = fmaxf(fmaxf(__uint_as_float(sa[i]), __uint_as_float(sb[i])),
                          fmaxf(__uint_as_float(sc[i]), __uint_as_float(sd[i])));
#pragma unroll
          for (int w = 16; w > 0; w >>= 1)
#pragma unroll
            for (int i = 0; i < w; ++i) mx[i] = fmaxf(mx[i], mx[i + w]);
          if (mx[0] >= theta - band) {
            const int rb = row0 + half * 128;
            epi_pass_topk<KB>(sa, sb, rb, r1 - rb, band, theta, theta_local, top, q, stash, P);
            epi_pass_topk<KB>(sc, sd, rb + 64, r1 - rb - 64, band, theta, theta_local, top, q, stash, P);
          }
        }
        if (qv && (tiles & 1) == 1 && theta_local > -INFINITY) {
          const uint32_t key = f2key(theta_local);
          if (key > published) {
            atomicMax(P.theta + q, key);
            published = key;
          }
        }
      }
      if (qv && theta_local > -INFINITY) {
        const uint32_t key = f2key(theta_local);
        if (key > published) atomicMax(P.theta + q, key);
        published = key > published ? key : published;
      }
      if (qv && !P.seed_only) {
        // Rotated publication: this unit's i-th best goes into slot (i + u) mod k
        // by atomicMax.  Every slot then holds the score of one real row, and
        // two slots never hold the same row (main-pass units scan disjoint
        // rows; each (unit, rank) pair writes one slot), so the smallest slot
        // is the k-th best of k distinct rows: a valid threshold, and one that
        // climbs towards the global k-th best as units finish, unlike any
        // single unit's k-th best.  (The threshold pass, whose sampled rows are
        // scanned again here, stays out of the slots.)
        uint32_t* sl = P.slots + (size_t)q * P.k;
        int j = u % P.k;
#pragma unroll 1
        for (int i = 0; i < P.k && top[i] > -INFINITY; ++i) {
          atomicMax(sl + j, f2key(top[i]));
          if (++j == P.k) j = 0;
        }
        uint32_t mn = 0xffffffffu;
        for (int i = 0; i < P.k; ++i) mn = min(mn, ld_volatile_u32(sl + i));
        if (mn != 0u && mn > published) atomicMax(P.theta + q, mn);  // 0: a slot not yet filled
      }
      } else {
      const float band = qv ? __ldg(P.qband + q) : 0.f;
      uint32_t g_key = qv ? ld_volatile_u32(P.theta + q) : 0u;
      uint32_t g_pending = g_key;
      float theta = g_key ? key2f(g_key) : -INFINITY;
      const int r0 = slice * P.slice_rows, r1 = min(P.N, r0 + P.slice_rows);
      for (int row0 = r0; row0 < r1; row0 += BN, ++it) {
        const int b = it & 1, fb = it >> 1;
        if (!mbar_wait(&acc_full[b], fb & 1, P.err, ERR_TIMEOUT_FULL)) { ok = false; break; }
        tc::fence_after();
        if (qv) {
          // the query's published threshold, read one tile ahead (its latency
          // overlaps this tile)
          if (g_pending) theta = fmaxf(theta, key2f(g_pending));
          g_pending = ld_volatile_u32(P.theta + q);
        }
        // two halves of 128 columns: all four loads of a half issued before one
        // wait; the common case is one max per score and one compare per half
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          uint32_t sa[32], sb[32], sc[32], sd[32];
          const uint32_t col = tmem + lane_base + (uint32_t)(b * BN + half * 128);
          tc::ld_32x32b_x32(col, sa);
          tc::ld_32x32b_x32(col + 32, sb);
          tc::ld_32x32b_x32(col + 64, sc);
          tc::ld_32x32b_x32(col + 96, sd);
          tc::wait_ld();
          if (half == 1) {
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive_remote(lead_acc_empty + 8u * (uint32_t)b);
          }
          if (!qv) continue;
          float mx[32];
#pragma unroll
          for (int i = 0; i < 32; ++i)
            mx[i] = fmaxf(fmaxf(__uint_as_float(sa[i]), __uint_as_float(sb[i])),
                          fmaxf(__uint_as_float(sc[i]), __uint_as_float(sd[i])));
#pragma unroll
          for (int w = 16; w > 0; w >>= 1)
#pragma unroll
            for (int i = 0; i < w; ++i) mx[i] = fmaxf(mx[i], mx[i + w]);
          if (mx[0] >= theta - band) {
            const int rb = row0 + half * 128;
            epi_pass(sa, sb, rb, r1 - rb, band, theta, q, stash, P);
            epi_pass(sc, sd, rb + 64, r1 - rb - 64, band, theta, q, stash, P);
          }
        }
      }
      }
    }
    // the threshold warp stops with this CTA's epilogue (error path included)
    if (threadIdx.x == 0) *reinterpret_cast<volatile int*>(&s_done) = 1;
  }
  // Normally every MMA has completed here (each epilogue waited for its last
  // accumulator).  On the error path a wait gave up: the even CTA waits
  // (bounded) for the MMAs it issued, and both CTAs give in-flight TMA copies a
  // bounded grace period, before TMEM is freed and shared memory released.
  tc::fence_before();
  tc::cluster_sync();
  if (threadIdx.x == 0) s_err = ld_volatile_u32(reinterpret_cast<const uint32_t*>(P.err)) != 0u;
  __syncthreads();
  if (s_err) {
    if (warp == 5 && leader) {
      if (tc::elect_one()) tc::commit_pair(tc::mapa_shared(smem_u32(&drain), 0));
      __syncwarp();
      mbar_wait(&drain, 0, nullptr, 0);
    }
    if (threadIdx.x == 0) grace_period();
  }
  tc::fence_before();
  tc::cluster_sync();  // no CTA touches its peer after this point
  tc::fence_after();
  if (warp == 5) tc::tmem_dealloc_pair(tmem, 512);
}

// One CTA per query.  The candidate list was appended against running
// thresholds; the query's final threshold (the larger of the scan's and the
// k-th best tf32 score among the candidates themselves -- k real rows either
// way) is tighter, so candidates whose tf32 score is below it minus the band are
// dropped.  The rest are scored exactly in fp32 (the single-query scan's
// arithmetic: per-lane float4 FMAs, xor-tree reduction 16..1) in rounds of up
// to 8,192 candidates, each round merged with the running exact top-k, so any
// number of candidates fits.
constexpr int RESCORE_CHUNK = 8192;

template <int VPL>
__global__ void __launch_bounds__(256) k_batch_rescore(const float* __restrict__ Q, const float* __restrict__ leaf,
                                                       const int* __restrict__ original_ids, int D, int k, int cap,
                                                       const float* __restrict__ qband,
                                                       const uint32_t* __restrict__ theta,
                                                       const int* __restrict__ cand_count,
                                                       const unsigned long long* __restrict__ cand_in,
                                                       float* __restrict__ out_s, int* __restrict__ out_i,
                                                       int* __restrict__ overflow) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem);  // [RESCORE_CHUNK + BATCH_MAX_K]
  unsigned long long* sel = cand + RESCORE_CHUNK + BATCH_MAX_K;            // [BATCH_MAX_K]
  unsigned long long* run = sel + BATCH_MAX_K;                             // [BATCH_MAX_K] running top-k
  SelectScratch* scratch = reinterpret_cast<SelectScratch*>(run + BATCH_MAX_K);
  __shared__ int s_n;
  const int q = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int total = cand_count[q];
  if (total > cap) {  // the appended list overflowed: this query must be answered another way
    if (threadIdx.x == 0) atomicAdd(overflow, 1);
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
      out_s[(size_t)q * k + i] = -INFINITY;
      out_i[(size_t)q * k + i] = -2;
    }
    return;
  }
  const unsigned long long* in = cand_in + (size_t)q * cap;
  const int D4 = D >> 2;
  const float4* q4 = reinterpret_cast<const float4*>(Q + (size_t)q * D);
  float4 qv[VPL];
#pragma unroll
  for (int v = 0; v < VPL; ++v) {
    const int c = lane + 32 * v;
    qv[v] = c < D4 ? __ldg(q4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  int selN = 1;
  while (selN < k) selN <<= 1;
  uint32_t tk = theta[q];
  if (total >= k) {
    block_select_topk<true>(in, total, k, sel, selN, scratch);
    const uint32_t ck = (uint32_t)(sel[k - 1] >> 32);
    tk = ck > tk ? ck : tk;
  }
  const float lim = tk ? key2f(tk) - qband[q] : -INFINITY;
  int run_n = 0;
  for (int base = 0; base < total; base += RESCORE_CHUNK) {
    if (threadIdx.x == 0) s_n = 0;
    __syncthreads();
    const int end = min(total, base + RESCORE_CHUNK);
    for (int i = base + threadIdx.x; i < end; i += blockDim.x) {
      const unsigned long long e = in[i];
      if (key2f((uint32_t)(e >> 32)) >= lim) cand[atomicAdd(&s_n, 1)] = e & 0xFFFFFFFFull;
    }
    __syncthreads();
    const int n = s_n;
    for (int i = warp; i < n; i += nw) {
      const int row = (int)(uint32_t)cand[i];
      const float4* x4 = reinterpret_cast<const float4*>(leaf + (size_t)row * D);
      float acc = 0.f;
#pragma unroll
      for (int v = 0; v < VPL; ++v) {
        const int c = lane + 32 * v;
        if (c < D4) {
          const float4 x = __ldg(x4 + c);
          acc = fmaf(x.x, qv[v].x, acc);
          acc = fmaf(x.y, qv[v].y, acc);
          acc = fmaf(x.z, qv[v].z, acc);
          acc = fmaf(x.w, qv[v].w, acc);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(FULL_MASK, acc, o);
      __syncwarp();
      if (lane == 0) cand[i] = pack_cand(f2key(acc), (uint32_t)row);
    }
    for (int i = threadIdx.x; i < run_n; i += blockDim.x) cand[n + i] = run[i];  // merge the running top-k
    __syncthreads();
    run_n = block_select_topk<false>(cand, n + run_n, k, sel, selN, scratch);
    for (int i = threadIdx.x; i < run_n; i += blockDim.x) run[i] = sel[i];
    __syncthreads();
  }
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const unsigned long long c = i < run_n ? run[i] : 0ull;
    out_s[(size_t)q * k + i] = c ? key2f(cand_key(c)) : -INFINITY;
    out_i[(size_t)q * k + i] = c ? original_ids[cand_row(c)] : -1;
  }
}

// Error band of each query, 2 eps = band_scale ||q|| (padded): one warp per query.
__global__ void k_query_bands(const float* __restrict__ Q, int B, int D, float band_scale, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int q = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  if (q >= B) return;
  const float* row = Q + (size_t)q * D;
  float s = 0.f;
  for (int d = lane; d < D; d += 32) s = fmaf(row[d], row[d], s);
  s = warp_sum(s);
  if (lane == 0) out[q] = band_scale * sqrtf(s) * 1.0001f;
}

// Max row norm (upper bound) of the leaf matrix: one warp per row, grid-stride.
__global__ void k_max_row_norm(const float* __restrict__ leaf, int N, int D, unsigned int* __restrict__ out_key) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  float mx = 0.f;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < N; r += warps) {
    const float* x = leaf + r * D;
    float s = 0.f;
    for (int d = lane; d < D; d += 32) s = fmaf(x[d], x[d], s);
    s = warp_sum(s);
    mx = fmaxf(mx, s);
  }
  if (lane == 0) atomicMax(out_key, __float_as_uint(mx));  // non-negative floats order as their bits
}

// ---------------------------------------------------------------- host
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// [rows, D] fp32 -> boxes of 128 rows x 32 columns, 128-byte swizzle; row r of
// the map is row r * row_step of the buffer.
static bool make_rows_tensor_map(const float* base, int rows, int D, void* out_map, int row_step = 1) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)D * 4 * (cuuint64_t)row_step};
  cuuint32_t box[2] = {32, 128};
  cuuint32_t estr[2] = {1, 1};
  return enc(reinterpret_cast<CUtensorMap*>(out_map), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base),
             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_leaf_tensor_map(const float* leaf, int N, int D, void* out_map) {
  return make_rows_tensor_map(leaf, N, D, out_map);
}

// rows r * step, step = max(16, N / 32768), r < sample_rows_for(N) <= 32768:
// all inside the corpus
static int sample_step(int N) { return N / SEED_ROWS > 16 ? N / SEED_ROWS : 16; }
int sample_rows_for(int N) {
  if (N < BATCH_SEED_MIN_N) return 0;
  const int n = (N - 1) / sample_step(N) + 1;
  return n < SEED_ROWS ? n : SEED_ROWS;
}

bool make_sample_tensor_map(const float* leaf, int N, int D, void* out_map) {
  return make_rows_tensor_map(leaf, sample_rows_for(N), D, out_map, sample_step(N));
}

cudaError_t launch_max_row_norm(const float* leaf, int N, int D, unsigned int* out_key, int sms, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(out_key, 0, sizeof(unsigned int), st);
  if (e != cudaSuccess) return e;
  k_max_row_norm<<<sms * 8, 256, 0, st>>>(leaf, N, D, out_key);
  return cudaGetLastError();
}

// Ring depth from the shared-memory budget; at least 120 KB is requested so that
// one CTA (and one 512-column TMEM allocation) occupies each SM.
static constexpr int BATCH_SMEM_BUDGET = 227 * 1024 - 1024;
static int batch_stages() {
  const int s = (BATCH_SMEM_BUDGET - EPI_COLS * BQ * 4 - 1024) / STAGE_BYTES;
  return s < BATCH_MAX_STAGES ? s : BATCH_MAX_STAGES;
}
static int batch_scan_smem(int stages) {
  const int b = stages * STAGE_BYTES + EPI_COLS * BQ * 4 + 1024;
  return b < 120 * 1024 ? 120 * 1024 : b;
}

template <int KB>
static cudaError_t launch_batch_scan(const void* qmap, const void* xmap, const BatchScanParams& P, int max_pairs,
                                       cudaStream_t st) {
  const int smem = batch_scan_smem(P.stages);
  static SmemOptIn opt_in;
  cudaError_t e = opt_in.ensure(reinterpret_cast<const void*>(k_batch_scan<KB>), smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(KB == 0 ? BATCH_THREADS_SLOTS : BATCH_THREADS);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // pairs that can be resident at once: a persistent grid larger than that
  // would leave late pairs a second wave.  Cached per device (the shared-memory
  // size is a constant of the build, so it needs no key of its own).
  static std::atomic<int> resident_by_dev[SmemOptIn::kMaxDevices] = {};
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  int resident = (dev >= 0 && dev < SmemOptIn::kMaxDevices) ? resident_by_dev[dev].load() : 0;
  if (resident < 1) {
    cfg.gridDim = dim3(2 * max_pairs);
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, k_batch_scan<KB>, &cfg);
    if (e != cudaSuccess) return e;
    if (n < 1) return cudaErrorInvalidConfiguration;
    resident = n;
    if (dev >= 0 && dev < SmemOptIn::kMaxDevices) resident_by_dev[dev].store(n);
  }
  const int pairs = std::min(std::min(P.units, max_pairs), resident);
  cfg.gridDim = dim3(2 * pairs);
  return cudaLaunchKernelEx(&cfg, k_batch_scan<KB>, *reinterpret_cast<const CUtensorMap*>(qmap),
                            *reinterpret_cast<const CUtensorMap*>(xmap), P);
}

template <int VPL>
static cudaError_t launch_rescore_t(const float* Q, const IndexView& ix, const BatchWorkspace& bw, int B, int k,
                                    int cap, float* out_s, int* out_i, cudaStream_t st) {
  const size_t smem = (size_t)(RESCORE_CHUNK + 3 * BATCH_MAX_K) * 8 + sizeof(SelectScratch) + 16;
  static SmemOptIn opt_in;
  cudaError_t e = opt_in.ensure(reinterpret_cast<const void*>(k_batch_rescore<VPL>), (int)smem);
  if (e != cudaSuccess) return e;
  k_batch_rescore<VPL><<<B, 256, smem, st>>>(Q, ix.leaf, ix.original_ids, ix.D, k, cap, bw.qband, bw.theta,
                                             bw.cand_count, bw.cand, out_s, out_i, bw.overflow);
  return cudaGetLastError();
}

cudaError_t launch_batch_search(const IndexView& ix, const BatchWorkspace& bw, const float* Q, int B, int k,
                                float* out_scores, int* out_ids, cudaStream_t st, cudaEvent_t ev_scan_begin,
                                cudaEvent_t ev_scan_end) {
  cudaError_t e;
  if ((e = cudaMemsetAsync(bw.theta, 0, sizeof(uint32_t) * B, st)) != cudaSuccess) return e;
  if ((e = cudaMemsetAsync(bw.cand_count, 0, sizeof(int) * B, st)) != cudaSuccess) return e;
  if ((e = cudaMemsetAsync(bw.overflow, 0, sizeof(int), st)) != cudaSuccess) return e;
  // a wait that gave up in an earlier batch must not send this one down the error path
  if ((e = cudaMemsetAsync(bw.err, 0, sizeof(int), st)) != cudaSuccess) return e;
  const int nslots = batch_slot_count(k);
  if ((e = cudaMemsetAsync(bw.slots, 0, sizeof(uint32_t) * (size_t)B * nslots, st)) != cudaSuccess) return e;
  if ((e = cudaMemsetAsync(bw.unit_counter, 0, 2 * sizeof(int), st)) != cudaSuccess) return e;
  BatchScanParams P{};
  P.Q = Q;
  P.B = B;
  P.D = ix.D;
  P.N = ix.N;
  P.k = k;
  P.kb = (ix.D + 31) / 32;
  P.stages = batch_stages();
  if (P.stages < 2 || ix.D % 4 != 0 || ix.D > BATCH_MAX_DIM || k < 1 || k > BATCH_MAX_K) return cudaErrorInvalidValue;
  P.QP = (B + 2 * BQ - 1) / (2 * BQ);
  const int slices = (ix.N + SLICE_ROWS - 1) / SLICE_ROWS;
  P.units = P.QP * slices;
  // eps = (2^-9 + 2^-20 + 2 D 2^-23 + gamma_D) ||q|| max||x||, padded; band = 2 eps
  const double u = 5.9604644775390625e-08;
  const double gD = ix.D * u / (1.0 - ix.D * u);
  const double eps_rel = 1.953125e-3 + 9.5367431640625e-07 + 2.0 * ix.D * 1.1920928955078125e-07 + gD;
  P.band_scale = (float)(2.0 * eps_rel * 1.01 * bw.xmax);
  P.qband = bw.qband;
  k_query_bands<<<(B + 7) / 8, 256, 0, st>>>(Q, B, ix.D, P.band_scale, bw.qband);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  P.theta = bw.theta;
  P.slots = bw.slots;
  P.nslots = nslots;
  P.cand_count = bw.cand_count;
  P.cand = bw.cand;
  // candidate entries per query: the workspace's fixed pool shared by the batch
  // (16,384 per query at full capacity, up to 65,536 for smaller batches)
  P.cap = (int)std::min<int64_t>(BATCH_CAND_MAX, bw.cand_entries / B);
  P.err = bw.err;
  P.seed_only = 0;
  P.slice_rows = SLICE_ROWS;
  P.row_step = 1;
  P.unit_counter = bw.unit_counter;
  alignas(64) unsigned char qmap[128];
  if (!make_rows_tensor_map(Q, B, ix.D, qmap)) return cudaErrorInvalidValue;
  const int max_pairs = bw.sms / 2;
  // k <= 32: per-thread top-k in registers (its threshold rises on every
  // insertion); larger k: slot thresholds, no per-thread list
  auto scan = [&](const void* xmap, const BatchScanParams& PP) -> cudaError_t {
    if (k <= 16) return launch_batch_scan<16>(qmap, xmap, PP, max_pairs, st);
    if (k <= 32) return launch_batch_scan<32>(qmap, xmap, PP, max_pairs, st);
    return launch_batch_scan<0>(qmap, xmap, PP, max_pairs, st);
  };
  if (ev_scan_begin && (e = cudaEventRecord(ev_scan_begin, st)) != cudaSuccess) return e;
  if (bw.sample_rows > 0) {
    // threshold pass over up to 32,768 rows spread evenly through the corpus,
    // one unit per query tile: it fills every query's slots, so the main pass
    // starts from the k-th best of k distinct sampled rows instead of -inf,
    // which removes most cold-start candidates and rare-path epilogue work
    BatchScanParams S = P;
    S.N = bw.sample_rows;
    S.seed_only = 1;
    // k <= 32: one unit per query tile (a unit's own k best set the threshold);
    // k > 32: the slots are keyed by row, so the sample is cut into slices of
    // 2,048 rows and spread over 16x as many CTA pairs
    S.slice_rows = k > 32 ? SEED_ROWS / 16 : SEED_ROWS;
    S.units = P.QP * ((S.N + S.slice_rows - 1) / S.slice_rows);
    S.row_step = sample_step(ix.N);
    S.unit_counter = bw.unit_counter + 1;
    if ((e = scan(bw.smap, S)) != cudaSuccess) return e;
  }
  if ((e = scan(bw.tmap, P)) != cudaSuccess) return e;
  if (ev_scan_end && (e = cudaEventRecord(ev_scan_end, st)) != cudaSuccess) return e;
  // float4 registers per lane for the query (the per-lane FMA order does not
  // depend on this bucket, so scores match the single-query scan bit for bit)
  const int v = (ix.D / 4 + 31) / 32;
  switch (v <= 1 ? 1 : v <= 2 ? 2 : v <= 3 ? 3 : v <= 4 ? 4 : v <= 6 ? 6 : v <= 8 ? 8 : v <= 12 ? 12 : 16) {
    case 1: return launch_rescore_t<1>(Q, ix, bw, B, k, P.cap, out_scores, out_ids, st);
    case 2: return launch_rescore_t<2>(Q, ix, bw, B, k, P.cap, out_scores, out_ids, st);
    case 3: return launch_rescore_t<3>(Q, ix, bw, B, k, P.cap, out_scores, out_ids, st);
    case 4: return launch_rescore_t<4>(Q, ix, bw, B, k, P.cap, out_scores, out_ids, st);
    case 6: return launch_rescore_t<6>(Q, ix, bw, B, k, P.cap, out_scores, out_ids, st);
    case 8: return launch_rescore_t<8>(Q, ix, bw, B, k, P.cap, out_scores, out_ids, st);
    case 12: return launch_rescore_t<12>(Q, ix, bw, B, k, P.cap, out_scores, out_ids, st);
    default: return launch_rescore_t<16>(Q, ix, bw, B, k, P.cap, out_scores, out_ids, st);
  }
}

}  // namespace cb
