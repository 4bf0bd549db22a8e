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
  uint32_t nnz;
  uint32_t pad;
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
        const int lo = 2 * stride * (i / stride) + (i % stride);
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
        const int lo = 2 * stride * (i / stride) + (i % stride);
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const unsigned long long x = a[lo], y = a[hi];
        if ((x < y) == up) { a[lo] = y; a[hi] = x; }
      }
      __syncwarp();
    }
  }
}

// Selects the k largest non-zero packed candidates of src[0..M) (unique when
// non-zero; zero = empty slot) by an 8 x 8-bit radix select over the 64-bit
// packed value, then sorts them.  sel must hold selN >= k entries (power of 2).
// Returns the number of selected candidates (min(k, non-zeros)); sel[0..ret) is
// sorted descending and sel[ret..selN) is zero.  All threads of the block call it.
template <bool GLOBAL>
static __device__ int block_select_topk(const unsigned long long* src, int M, int k, unsigned long long* sel,
                                 int selN, SelectScratch* s) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) { s->nnz = 0; s->count = 0; s->prefix = 0; }
  __syncthreads();
  uint32_t local = 0;
  for (int i = tid; i < M; i += blockDim.x) local += (ld_cand<GLOBAL>(src + i) != 0ull);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(FULL_MASK, local, o);
  if (lane == 0 && local) atomicAdd(&s->nnz, local);
  __syncthreads();
  const int kk = min((int)s->nnz, k);
  for (int i = tid; i < selN; i += blockDim.x) sel[i] = 0ull;
  if (kk == 0) { __syncthreads(); return 0; }
  if (tid == 0) s->need = (uint32_t)kk;
  __syncthreads();
  for (int shift = 56; shift >= 0; shift -= 8) {
    const unsigned long long prefix = s->prefix;
    const uint32_t need = s->need;
    const unsigned long long hmask = (shift == 56) ? 0ull : (~0ull << (shift + 8));
    for (int i = tid; i < 256; i += blockDim.x) s->hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < M; i += blockDim.x) {
      const unsigned long long v = ld_cand<GLOBAL>(src + i);
      if ((v & hmask) == prefix) atomicAdd(&s->hist[(v >> shift) & 255ull], 1u);
    }
    __syncthreads();
    if (warp == 0) {
      uint32_t c[8], sum = 0;
#pragma unroll
      for (int t = 0; t < 8; ++t) { c[t] = s->hist[255 - (lane * 8 + t)]; sum += c[t]; }
      uint32_t incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        uint32_t x = __shfl_up_sync(FULL_MASK, incl, o);
        if (lane >= o) incl += x;
      }
      const uint32_t excl = incl - sum;
      if (excl < need && incl >= need) {
        uint32_t acc = excl;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          if (acc + c[t] >= need) {
            const uint32_t d = 255 - (lane * 8 + t);
            s->prefix = prefix | ((unsigned long long)d << shift);
            s->need = need - acc;
            break;
          }
          acc += c[t];
        }
      }
    }
    __syncthreads();
  }
  const unsigned long long kth = s->prefix;
  for (int i = tid; i < M; i += blockDim.x) {
    const unsigned long long v = ld_cand<GLOBAL>(src + i);
    if (v != 0ull && v >= kth) {
      const uint32_t pos = atomicAdd(&s->count, 1u);
      if (pos < (uint32_t)selN) sel[pos] = v;
    }
  }
  __syncthreads();
  block_bitonic_desc(sel, selN);
  return kk;
}

}  // namespace cb
