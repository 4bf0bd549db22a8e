// Cross-shard top-k merge (multi-GPU search): the k candidates of each of the
// W shards, gathered on every rank by one NCCL all-gather, are reduced to the
// global top-k on the device.  Ordering is (score desc, original id asc), the
// same total order every shard used locally, so the merged result does not
// depend on the number of shards.  Also the root-to-rank shard plan (host).
#include <algorithm>
#include <numeric>
#include <string>
#include <vector>

#include "../../include/circuit_shard.h"
#include "common.cuh"
#include "engine.h"
#include "index_internal.h"
#include "topk.cuh"

namespace cb {

constexpr int MERGE_THREADS = 256;
constexpr int MERGE_MAX_N = 16384;

__global__ void __launch_bounds__(MERGE_THREADS) k_merge_topk(const float* __restrict__ scores,
                                                                const int* __restrict__ ids, int n, int k,
                                                                int selN, float* __restrict__ out_scores,
                                                                int* __restrict__ out_ids) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem);
  unsigned long long* sel = cand + n;
  SelectScratch* scratch = reinterpret_cast<SelectScratch*>(sel + selN);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int id = ids[i];
    cand[i] = id >= 0 ? pack_cand(f2key(scores[i]), (uint32_t)id) : 0ull;
  }
  __syncthreads();
  block_select_topk<false>(cand, n, k, sel, selN, scratch);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const unsigned long long c = sel[i];
    out_scores[i] = c ? key2f(cand_key(c)) : -INFINITY;
    out_ids[i] = c ? (int)cand_row(c) : -1;
  }
}

// One CTA per query; candidate j of query q is at [(j / k_in) * qstride + q * k_in + j % k_in].
__global__ void __launch_bounds__(MERGE_THREADS) k_merge_topk_batch(const float* __restrict__ scores,
                                                                      const int* __restrict__ ids, int world, int k_in,
                                                                      size_t qstride, int k, int selN,
                                                                      float* __restrict__ out_scores,
                                                                      int* __restrict__ out_ids) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int n = world * k_in;
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem);
  unsigned long long* sel = cand + n;
  SelectScratch* scratch = reinterpret_cast<SelectScratch*>(sel + selN);
  const int q = blockIdx.x;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const size_t at = (size_t)(j / k_in) * qstride + (size_t)q * k_in + (size_t)(j % k_in);
    const int id = ids[at];
    cand[j] = id >= 0 ? pack_cand(f2key(scores[at]), (uint32_t)id) : 0ull;
  }
  __syncthreads();
  block_select_topk<false>(cand, n, k, sel, selN, scratch);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const unsigned long long c = sel[i];
    out_scores[(size_t)q * k + i] = c ? key2f(cand_key(c)) : -INFINITY;
    out_ids[(size_t)q * k + i] = c ? (int)cand_row(c) : -1;
  }
}

// One thread waits on an mbarrier that nothing arrives on: the bounded wait
// gives up after WAIT_LIMIT_NS and records ERR_TIMEOUT_FULL.
__global__ void k_selftest_wait(int* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_wait(&bar, 0, err, ERR_TIMEOUT_FULL);
  }
}

cudaError_t launch_selftest_wait(int* err, cudaStream_t stream) {
  k_selftest_wait<<<1, 32, 0, stream>>>(err);
  return cudaGetLastError();
}

}  // namespace cb

extern "C" {

int circuit_selftest_wait_timeout(int device_id, int* out_error_bits) {
  if (!out_error_bits) { cb::set_error("null out_error_bits"); return CIRCUIT_ERR_ARG; }
  if (!cb::cuda_ok(cudaSetDevice(device_id), "cudaSetDevice")) return CIRCUIT_ERR_CUDA;
  int* d = nullptr;
  if (!cb::cuda_ok(cudaMalloc(&d, sizeof(int)), "cudaMalloc")) return CIRCUIT_ERR_CUDA;
  int rc = CIRCUIT_OK;
  if (!cb::cuda_ok(cudaMemset(d, 0, sizeof(int)), "memset")) rc = CIRCUIT_ERR_CUDA;
  if (rc == CIRCUIT_OK) {
    cb::k_selftest_wait<<<1, 32>>>(d);
    if (!cb::cuda_ok(cudaGetLastError(), "selftest launch") || !cb::cuda_ok(cudaDeviceSynchronize(), "selftest sync") ||
        !cb::cuda_ok(cudaMemcpy(out_error_bits, d, sizeof(int), cudaMemcpyDeviceToHost), "selftest D2H"))
      rc = CIRCUIT_ERR_CUDA;
  }
  cudaFree(d);
  return rc;
}

int circuit_merge_topk_batch(const float* scores, const int* ids, int num_queries, int world, int k_in, int k,
                             float* out_scores, int* out_ids, void* stream) {
  if (!scores || !ids || !out_scores || !out_ids) {
    cb::set_error("merge_topk_batch: null pointer");
    return CIRCUIT_ERR_ARG;
  }
  if (num_queries < 1 || world < 1 || k_in < 1 || (int64_t)world * k_in > cb::MERGE_MAX_N || k < 1 ||
      k > cb::KMAX) {
    cb::set_error("merge_topk_batch: need num_queries >= 1, 1 <= world * k_in <= 16384, 1 <= k <= 256");
    return CIRCUIT_ERR_ARG;
  }
  int selN = 1;
  while (selN < k) selN <<= 1;
  const int n = world * k_in;
  const size_t smem = sizeof(unsigned long long) * (size_t)(n + selN) + sizeof(cb::SelectScratch) + 16;
  static cb::SmemOptIn opt_in;
  if (smem > 48 * 1024 &&
      !cb::cuda_ok(opt_in.ensure(reinterpret_cast<const void*>(cb::k_merge_topk_batch), (int)smem), "merge batch smem"))
    return CIRCUIT_ERR_CUDA;
  cb::k_merge_topk_batch<<<num_queries, cb::MERGE_THREADS, smem, (cudaStream_t)stream>>>(
      scores, ids, world, k_in, (size_t)num_queries * k_in, k, selN, out_scores, out_ids);
  return cb::cuda_ok(cudaGetLastError(), "merge_topk_batch launch") ? CIRCUIT_OK : CIRCUIT_ERR_CUDA;
}

int circuit_merge_topk(const float* scores, const int* ids, int n, int k, float* out_scores, int* out_ids,
                       void* stream) {
  if (!scores || !ids || !out_scores || !out_ids) {
    cb::set_error("merge_topk: null pointer");
    return CIRCUIT_ERR_ARG;
  }
  if (n < 1 || n > cb::MERGE_MAX_N || k < 1 || k > cb::KMAX) {
    cb::set_error("merge_topk: need 1 <= n <= 16384 and 1 <= k <= 256");
    return CIRCUIT_ERR_ARG;
  }
  int selN = 1;
  while (selN < k) selN <<= 1;
  const size_t smem = sizeof(unsigned long long) * (size_t)(n + selN) + sizeof(cb::SelectScratch) + 16;
  static cb::SmemOptIn opt_in;
  if (smem > 48 * 1024 &&
      !cb::cuda_ok(opt_in.ensure(reinterpret_cast<const void*>(cb::k_merge_topk), (int)smem), "merge smem"))
    return CIRCUIT_ERR_CUDA;
  cb::k_merge_topk<<<1, cb::MERGE_THREADS, smem, (cudaStream_t)stream>>>(scores, ids, n, k, selN, out_scores, out_ids);
  return cb::cuda_ok(cudaGetLastError(), "merge_topk launch") ? CIRCUIT_OK : CIRCUIT_ERR_CUDA;
}

int circuit_plan_shards(const int64_t* root_rows, int num_roots, int world, int* root_to_rank, int64_t* rank_rows) {
  if (!root_rows || !root_to_rank || num_roots < 1 || world < 1) {
    cb::set_error("plan_shards: bad arguments");
    return CIRCUIT_ERR_ARG;
  }
  // longest-processing-time first: heaviest root to the currently lightest rank
  std::vector<int> order(num_roots);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return root_rows[a] > root_rows[b]; });
  std::vector<int64_t> load(world, 0);
  for (int r : order) {
    int best = 0;
    for (int w = 1; w < world; ++w)
      if (load[w] < load[best]) best = w;
    root_to_rank[r] = best;
    load[best] += root_rows[r];
  }
  if (rank_rows)
    for (int w = 0; w < world; ++w) rank_rows[w] = load[w];
  return CIRCUIT_OK;
}

}  // extern "C"
