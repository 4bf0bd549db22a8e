// circuit_flat_search_noalloc: exact top-k over a raw device corpus that never
// allocates device memory.
//
// Some callers cannot call cudaMalloc: an inference-engine plugin whose host
// framework owns every byte of device memory and forbids stray allocations, a
// serving loop that must not touch the allocator (or its lock) after start-up,
// code running while another library holds the device allocator.  They pass
// the corpus, the query and the outputs; the per-CTA candidate lists and the
// control words the scan needs live in the file-scope array below instead of
// the per-handle workspace the other entry points allocate.
//
// The array is part of the library's device image: every GPU on which the
// library's kernels are loaded holds NOALLOC_SCRATCH_BYTES of it until the
// process exits.  All calls on a device share it and each call leaves its
// contents behind, so every call clears the control words it needs, and calls
// that overlap on the GPU (e.g. issued on two streams without ordering) race
// on it and must be serialised by the caller.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/circuit.h"
#include "common.cuh"
#include "engine.h"
#include "index_internal.h"

namespace cb {
namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = 256 * 1024;
constexpr size_t NOALLOC_CTRL_BYTES = 2304;                    // SearchCtrl, rounded up to 256
constexpr size_t NOALLOC_RANGE_OFF = NOALLOC_CTRL_BYTES;       // int4 range + u64 packed count
constexpr size_t NOALLOC_LISTS_OFF = NOALLOC_CTRL_BYTES + 256;  // per-CTA candidate lists
constexpr int NOALLOC_LIST_CAP = (int)((NOALLOC_SCRATCH_BYTES - NOALLOC_LISTS_OFF) / 8);
constexpr int NOALLOC_MAX_K = 128;
constexpr int NOALLOC_MAX_DEVICES = 64;
static_assert(sizeof(SearchCtrl) <= NOALLOC_CTRL_BYTES, "control block does not fit");

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

std::mutex g_setup_mutex;
void* g_scratch_addr[NOALLOC_MAX_DEVICES] = {};

// Clears the control words of the previous call and writes the single leaf range.
__global__ void k_noalloc_prepare(int n) {
  uint32_t* ctrl = reinterpret_cast<uint32_t*>(g_noalloc_scratch);
  for (int i = threadIdx.x; i < (int)(CTRL_RESET_BYTES / 4); i += blockDim.x) ctrl[i] = 0u;
  if (threadIdx.x == 0) {
    *reinterpret_cast<int4*>(g_noalloc_scratch + NOALLOC_RANGE_OFF) = make_int4(0, 0, n, -1);
    *reinterpret_cast<unsigned long long*>(g_noalloc_scratch + NOALLOC_RANGE_OFF + 16) =
        (1ull << 32) | (unsigned long long)(uint32_t)n;
  }
}

// Device address of the scratch array for the current device, looked up once
// per device (with that device current) and cached.
int scratch_address(int device, unsigned char** out) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_error(std::string("cudaGetSymbolAddress(no-alloc scratch): ") + cudaGetErrorString(e));
      return CIRCUIT_ERR_CUDA;
    }
    g_scratch_addr[device] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_addr[device]);
  return CIRCUIT_OK;
}

}  // namespace
}  // namespace cb

extern "C" int circuit_flat_search_noalloc(const float* dev_corpus, int64_t n, int dim, const float* dev_query, int k,
                                           float* dev_out_scores, int* dev_out_ids, void* stream) {
  using namespace cb;
  if (!dev_corpus || !dev_query || !dev_out_scores || !dev_out_ids) {
    set_error("flat_search_noalloc: null pointer");
    return CIRCUIT_ERR_ARG;
  }
  if (n < 1 || n >= (int64_t)0x7fffffff) {
    set_error("flat_search_noalloc: n must be in [1, 2^31 - 1)");
    return CIRCUIT_ERR_ARG;
  }
  if (dim < 4 || dim % 4 != 0 || dim > MAX_DIM) {
    set_error("flat_search_noalloc: dim must be a multiple of 4 in [4, 2048]");
    return CIRCUIT_ERR_UNSUPPORTED;
  }
  if (k < 1 || k > NOALLOC_MAX_K) {
    set_error("flat_search_noalloc: k must be in [1, 128] (the fixed scratch holds 128 candidates per CTA)");
    return CIRCUIT_ERR_ARG;
  }
  if (((uintptr_t)dev_corpus | (uintptr_t)dev_query) & 15) {
    set_error("flat_search_noalloc: corpus and query must be 16-byte aligned");
    return CIRCUIT_ERR_ARG;
  }
  int device = 0;
  if (!cuda_ok(cudaGetDevice(&device), "cudaGetDevice")) return CIRCUIT_ERR_CUDA;
  if (device < 0 || device >= NOALLOC_MAX_DEVICES) {
    set_error("flat_search_noalloc: device ordinal above 63");
    return CIRCUIT_ERR_UNSUPPORTED;
  }
  unsigned char* scratch = nullptr;
  int rc = scratch_address(device, &scratch);
  if (rc != CIRCUIT_OK) return rc;
  int grid = sm_count(device);
  if ((grid + 1) * k > NOALLOC_LIST_CAP) grid = NOALLOC_LIST_CAP / k - 1;
  cudaStream_t st = (cudaStream_t)stream;
  k_noalloc_prepare<<<1, 32, 0, st>>>((int)n);
  if (!cuda_ok(cudaGetLastError(), "flat_search_noalloc prepare")) return CIRCUIT_ERR_CUDA;
  const cudaError_t e = launch_flat_scan(
      dev_corpus, dim, (int)n, dev_query, k, grid, reinterpret_cast<SearchCtrl*>(scratch),
      reinterpret_cast<const int4*>(scratch + NOALLOC_RANGE_OFF),
      reinterpret_cast<const unsigned long long*>(scratch + NOALLOC_RANGE_OFF + 16),
      reinterpret_cast<unsigned long long*>(scratch + NOALLOC_LISTS_OFF), dev_out_scores, dev_out_ids, st);
  return cuda_ok(e, "flat_search_noalloc scan") ? CIRCUIT_OK : CIRCUIT_ERR_CUDA;
}
