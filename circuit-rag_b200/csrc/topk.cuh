// Block- and warp-level top-k building blocks over packed 64-bit candidates
// (key << 32 | ~row, see common.cuh): bitonic sorts in shared memory and an
// 8 x 8-bit radix select.  Used by the leaf scan (per-CTA and grid merges) and
// by the cross-shard merge.
#pragma once

#include "common.cuh"

namespace cb {

// ============================================================ block top-k select
struct SelectScratch {
  uint32_t hist[256];
  unsigned long long prefix;
  uint32_t need;
  uint32_t count;
  uint32_t done;
  uint32_t kk;
};

template <bool GLOBAL>
__device__ __forceinline__ unsigned long long ld_cand(const unsigned long long* p) {
  if constexpr (GLOBAL) return __ldcg(p);
  else return *p;
}

// Block-wide descending bitonic sort of a[0..n) (n a power of two) in shared memory.
static __device__ void block_bitonic_desc(unsigned long long* a, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < (n >> 1); i += blockDim.x) {
        const int lo = ((i & ~(stride - 1)) << 1) | (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const unsigned long long x = a[lo], y = a[hi];
        if ((x < y) == up) { a[lo] = y; a[hi] = x; }
      }
      __syncthreads();
    }
  }
}

// Warp-wide descending bitonic sort of a[0..n) (n a power of two) in shared memory.
static __device__ void warp_bitonic_desc(unsigned long long* a, int n, int lane) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = lane; i < (n >> 1); i += 32) {
        const int lo = ((i & ~(stride - 1)) << 1) | (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const unsigned long long x = a[lo], y = a[hi];
        if ((x < y) == up) { a[lo] = y; a[hi] = x; }
      }
      __syncwarp();
    }
  }
}

// Warp-wide descending bitonic sort of 32 * R values held in registers: lane l
// holds elements l*R .. l*R + R-1 in v[0..R).  Strides below R pair registers of
// one lane; the others pair lanes through shuffles.
template <int R>
__device__ __forceinline__ void warp_sort_regs_desc(unsigned long long (&v)[R], int lane) {
  constexpr int N = 32 * R;
#pragma unroll
  for (int size = 2; size <= N; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride < R) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int pr = r ^ stride;
          if (pr > r) {
            const bool desc = ((lane * R + r) & size) == 0;  // the lower element keeps the max
            const unsigned long long a = v[r], b = v[pr];
            if (desc ? (a < b) : (a > b)) {
              v[r] = b;
              v[pr] = a;
            }
          }
        }
      } else {
        const int lx = stride / R;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const unsigned long long b = __shfl_xor_sync(FULL_MASK, v[r], lx);
          const bool desc = ((lane * R + r) & size) == 0;
          const bool lower = (lane & lx) == 0;
          v[r] = (lower == desc) ? (v[r] > b ? v[r] : b) : (v[r] < b ? v[r] : b);
        }
      }
    }
  }
}

// Top 32 of two sorted 32-value lists held one value per lane: a descending,
// b ascending.  max(a[j], b[j]) is a bitonic sequence holding exactly the top 32
// of the union; five half-cleaner steps sort it (descending or ascending).
__device__ __forceinline__ unsigned long long warp_merge_top32(unsigned long long a_desc, unsigned long long b_asc,
                                                               bool desc, int lane) {
  unsigned long long c = a_desc > b_asc ? a_desc : b_asc;
#pragma unroll
  for (int st = 16; st > 0; st >>= 1) {
    const unsigned long long o = __shfl_xor_sync(FULL_MASK, c, st);
    const bool keep_max = ((lane & st) == 0) == desc;
    c = keep_max ? (c > o ? c : o) : (c < o ? c : o);
  }
  return c;
}

// Top-k by direct ranking, for merges with few survivors: the non-empty
// candidates of src[0..M) (shared memory) whose key is not below min_key are
// compacted into tmp[0..CAP); each one's rank is the number of larger ones
// (candidates are unique) and ranks below k land in sel.  Returns min(k,
// survivors) with sel[0..ret) sorted descending and sel[ret..selN) zero, or -1
// when more than CAP survive (sel is then undefined: use block_select_topk).
// `count` is a shared word of the caller.  All threads of the block call it.
template <int CAP>
static __device__ int block_rank_topk(const unsigned long long* src, int M, int k, unsigned long long* sel, int selN,
                                      unsigned long long* tmp, uint32_t* count, uint32_t min_key) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthreads = blockDim.x;
  const unsigned long long floor_v = (unsigned long long)min_key << 32;
  if (tid == 0) *count = 0;
  for (int i = tid; i < selN; i += nthreads) sel[i] = 0ull;
  __syncthreads();
  for (int base = warp * 32; base < M; base += nthreads) {
    const int i = base + lane;
    const unsigned long long v = i < M ? src[i] : 0ull;
    const bool pass = v != 0ull && v >= floor_v;
    const uint32_t bal = __ballot_sync(FULL_MASK, pass);
    uint32_t pos = 0;
    if (lane == 0 && bal) pos = atomicAdd(count, (uint32_t)__popc(bal));
    pos = __shfl_sync(FULL_MASK, pos, 0) + __popc(bal & lanemask_lt());
    if (pass && pos < (uint32_t)CAP) tmp[pos] = v;
  }
  __syncthreads();
  const int n = (int)*count;
  if (n > CAP) {
    __syncthreads();  // every thread has read *count before the caller reuses it
    return -1;
  }
  for (int t = tid; t < n; t += nthreads) {
    const unsigned long long v = tmp[t];
    int r = 0, j = 0;
    for (; j + 8 <= n; j += 8) {  // eight independent loads in flight
#pragma unroll
      for (int u = 0; u < 8; ++u) r += tmp[j + u] > v;
    }
    for (; j < n; ++j) r += tmp[j] > v;
    if (r < k) sel[r] = v;
  }
  __syncthreads();
  return n < k ? n : k;
}

// Selects the k largest non-zero packed candidates of src[0..M) (unique when
// non-zero; zero = empty slot) by a most-significant-digit-first radix select
// over the 64-bit packed value, 8 bits per pass, then sorts them.
//   - zeros never enter a histogram; the first pass also counts the non-zeros,
//     so fewer than k of them select them all;
//   - one shared atomic per distinct bin per warp (lanes with the same bin are
//     grouped by match.any), so runs of equal digits do not serialise;
//   - the passes stop as soon as the bin that holds the k-th value holds exactly
//     the number still needed: the selection is then "everything with this
//     prefix or above", usually after 2-4 of the 8 digits.
// Candidates whose key (upper 32 bits) is below min_key count as empty (the
// caller knows they cannot be among the k best); min_key must be the same in
// every thread.  sel must hold selN >= k entries (power of 2).  Returns the
// number selected (min(k, non-empty)); sel[0..ret) is sorted descending and
// sel[ret..selN) is zero.  All threads of the block call it; blockDim.x is a
// multiple of 32.
template <bool GLOBAL>
static __device__ int block_select_topk(const unsigned long long* src, int M, int k, unsigned long long* sel,
                                        int selN, SelectScratch* s, uint32_t min_key = 0u) {
  const unsigned long long floor_v = (unsigned long long)min_key << 32;  // v >= floor_v <=> key >= min_key
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthreads = blockDim.x;
  for (int i = tid; i < 256; i += nthreads) s->hist[i] = 0;
  for (int i = tid; i < selN; i += nthreads) sel[i] = 0ull;
  if (tid == 0) { s->count = 0; s->kk = 0; s->done = 0; }
  __syncthreads();
  unsigned long long prefix = 0ull;
  uint32_t need = (uint32_t)k;  // the first pass lowers it to min(k, non-zeros)
  for (int shift = 56;; shift -= 8) {
    const unsigned long long hmask = (shift == 56) ? 0ull : (~0ull << (shift + 8));
    for (int base = warp * 32; base < M; base += nthreads) {
      const int i = base + lane;
      const unsigned long long v = (i < M) ? ld_cand<GLOBAL>(src + i) : 0ull;
      const bool in = v != 0ull && v >= floor_v && (v & hmask) == prefix;
      const uint32_t bin = in ? (uint32_t)(v >> shift) & 255u : 256u;
      const uint32_t peers = __match_any_sync(FULL_MASK, bin);
      if (in && lane == __ffs(peers) - 1) atomicAdd(&s->hist[bin], (uint32_t)__popc(peers));
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins 255-8l .. 248-8l (descending digit order); the warp
      // clears them for the next pass while it reads them
      uint32_t c[8], sum = 0;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        c[t] = s->hist[255 - (lane * 8 + t)];
        s->hist[255 - (lane * 8 + t)] = 0;
        sum += c[t];
      }
      uint32_t incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t x = __shfl_up_sync(FULL_MASK, incl, o);
        if (lane >= o) incl += x;
      }
      if (shift == 56) {
        const uint32_t nnz = __shfl_sync(FULL_MASK, incl, 31);
        need = need < nnz ? need : nnz;
        if (lane == 0) {
          s->kk = need;
          if (need == 0) s->done = 1;
        }
      }
      const uint32_t excl = incl - sum;
      if (need > 0 && excl < need && incl >= need) {
        uint32_t acc = excl;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          if (acc + c[t] >= need) {
            const uint32_t d = 255 - (lane * 8 + t);
            s->prefix = prefix | ((unsigned long long)d << shift);
            s->need = need - acc;
            s->done = (c[t] == need - acc) || shift == 0;
            break;
          }
          acc += c[t];
        }
      }
    }
    __syncthreads();
    const bool done = s->done != 0;
    prefix = s->prefix;
    need = s->need;
    if (done) break;
  }
  const int kk = (int)s->kk;
  if (kk == 0) return 0;
  // everything at or above the k-th value's resolved prefix: exactly kk entries
  for (int i = tid; i < M; i += nthreads) {
    const unsigned long long v = ld_cand<GLOBAL>(src + i);
    if (v != 0ull && v >= floor_v && v >= prefix) {
      const uint32_t pos = atomicAdd(&s->count, 1u);
      if (pos < (uint32_t)selN) sel[pos] = v;
    }
  }
  __syncthreads();
  const int n = min((int)s->count, selN);
  if (n <= nthreads) {
    // rank sort: each selected value's rank is the number of larger values
    // (ties broken by position), then one scatter
    unsigned long long v = 0ull;
    int r = 0;
    if (tid < n) {
      v = sel[tid];
      for (int j = 0; j < n; ++j) {
        const unsigned long long u = sel[j];
        r += (u > v) || (u == v && j < tid);
      }
    }
    __syncthreads();
    if (tid < n) sel[r] = v;
    __syncthreads();
  } else {
    block_bitonic_desc(sel, selN);
  }
  return kk;
}

}  // namespace cb
