// Shared device helpers for the circuit-b200 search kernels (sm_100a only).
//
// * mbarrier + 1-D bulk TMA (cp.async.bulk) wrappers used to stage leaf tiles,
//   centroids and rank-r bases into shared memory.  Every copy reads this
//   GPU's own memory into the issuing CTA's shared memory (the batched scan's
//   CTA-pair loads only route their completion to the even CTA's barrier).
// * bounded waits: every spin on an mbarrier gives up after WAIT_LIMIT_NS of
//   %globaltimer time, records an error bit in the per-query control block and
//   returns false, so a stuck copy can never hang the GPU.
// * order-preserving float <-> uint32 keys and the packed 64-bit candidate
//   (key << 32 | ~row) used by every top-k structure: larger packed value means
//   larger score, ties broken towards the smaller leaf row.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "circuit-b200 kernels target sm_100a only"
#endif

namespace cb {

constexpr uint32_t FULL_MASK = 0xffffffffu;
constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;  // 2 s per wait

// Error bits written to SearchCtrl::error by device code.
enum : int {
  ERR_TIMEOUT_FULL = 1,    // consumer waited too long for a staged tile
  ERR_TIMEOUT_EMPTY = 2,   // producer waited too long for a free stage
  ERR_TIMEOUT_BASIS = 4,   // bounds kernel waited too long for a basis chunk
  ERR_BAD_RANGE = 8,       // a range / row index failed its bounds check
};

// ---------------------------------------------------------------- ordering keys
__device__ __forceinline__ uint32_t f2key(float f) {
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(b);
}
__host__ __device__ __forceinline__ unsigned long long pack_cand(uint32_t key, uint32_t row) {
  return ((unsigned long long)key << 32) | (unsigned long long)(~row);
}
__host__ __device__ __forceinline__ uint32_t cand_key(unsigned long long c) { return (uint32_t)(c >> 32); }
__host__ __device__ __forceinline__ uint32_t cand_row(unsigned long long c) { return ~(uint32_t)(c & 0xffffffffull); }

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: true when the phase with `parity` completed, false after the
// time limit (the error bit is then or-ed into *err, if err is non-null).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > WAIT_LIMIT_NS) {
      if (err) atomicOr(err, code);
      return false;
    }
  }
}
// Error path only: a bounded wait gave up while bulk copies (or MMAs) may still
// be in flight into this CTA's shared memory.  They complete within
// microseconds unless the memory system is stuck, so the CTA waits a fixed,
// bounded grace period before it reuses that memory or exits.
constexpr unsigned long long GRACE_NS = 1000000ull;  // 1 ms
__device__ __forceinline__ void grace_period() {
  const unsigned long long t0 = globaltimer();
  while (globaltimer() - t0 < GRACE_NS) __nanosleep(1000);
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned: callers check this on the host).
__device__ __forceinline__ void tma_load_1d(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Same, with an L2 evict-first policy for data streamed exactly once (leaf rows).
__device__ __forceinline__ void tma_load_1d_stream(void* dst_smem, const void* src, uint32_t bytes,
                                                   uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// Bulk prefetch of [src, src + bytes) into L2 (no shared memory, no completion
// to wait for): keeps DRAM busy ahead of the shared-memory ring.
__device__ __forceinline__ void prefetch_l2_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// Brings the 128-byte line holding p into L2 (no completion to wait for).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}
__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
  return *reinterpret_cast<const volatile unsigned long long*>(p);
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialisation may start while the kernel before it on the stream is still
// running; griddep_wait() blocks until that kernel has completed and its
// memory is visible, so everything before it must only read data that existed
// before that kernel was launched.  griddep_launch() lets the next kernel of
// the stream start early (it still waits for this one's completion before it
// reads any result).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- warp helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL_MASK, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL_MASK, v, o);
  return v;
}
__device__ __forceinline__ int warp_incl_scan(int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(FULL_MASK, v, o);
    if (lane >= o) v += t;
  }
  return v;
}
__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

}  // namespace cb
