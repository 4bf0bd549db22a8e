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

int circuit_plan_shard_parts(const int64_t* atom_rows, const int64_t* root_atom_ptr, int num_roots, int world,
                             double max_imbalance, int* part_root, int64_t* part_atom_begin, int64_t* part_atom_end,
                             int* part_rank, int max_parts, int* num_parts, int64_t* rank_rows) {
  if (!atom_rows || !root_atom_ptr || !part_root || !part_atom_begin || !part_atom_end || !part_rank || !num_parts ||
      num_roots < 1 || world < 1 || max_parts < 1 || !(max_imbalance >= 1.0)) {
    cb::set_error("plan_shard_parts: bad arguments");
    return CIRCUIT_ERR_ARG;
  }
  struct Item {
    int64_t rows;
    int root;
    int64_t a0, a1;  // atom range
  };
  std::vector<Item> items;
  int64_t total = 0;
  for (int p = 0; p < num_roots; ++p) {
    const int64_t a0 = root_atom_ptr[p], a1 = root_atom_ptr[p + 1];
    if (a0 < 0 || a1 < a0) {
      cb::set_error("plan_shard_parts: root_atom_ptr must be non-decreasing from 0");
      return CIRCUIT_ERR_ARG;
    }
    int64_t r = 0;
    for (int64_t a = a0; a < a1; ++a) {
      if (atom_rows[a] < 0) {
        cb::set_error("plan_shard_parts: negative atom size");
        return CIRCUIT_ERR_ARG;
      }
      r += atom_rows[a];
    }
    if (r > 0) items.push_back({r, p, a0, a1});
    total += r;
  }
  const double allowed = max_imbalance * (double)total / (double)world;
  // largest first; ties by root (deterministic on every rank)
  const auto before = [](const Item& x, const Item& y) { return x.rows != y.rows ? x.rows > y.rows : x.root < y.root; };
  std::sort(items.begin(), items.end(), before);
  std::vector<int64_t> load(world, 0);
  struct Part {
    int rank, root;
    int64_t a0, a1;
  };
  std::vector<Part> parts;
  size_t head = 0;
  while (head < items.size()) {
    const Item it = items[head++];
    int r = 0;
    for (int w = 1; w < world; ++w)
      if (load[w] < load[r]) r = w;
    if ((double)(load[r] + it.rows) <= allowed || it.a1 - it.a0 == 1) {
      parts.push_back({r, it.root, it.a0, it.a1});
      load[r] += it.rows;
      continue;
    }
    // the longest prefix of atoms that fits (at least one atom)
    int64_t a = it.a0, taken = 0;
    while (a < it.a1 && (double)(load[r] + taken + atom_rows[a]) <= allowed) taken += atom_rows[a++];
    if (a == it.a0) taken += atom_rows[a++];
    parts.push_back({r, it.root, it.a0, a});
    load[r] += taken;
    Item rest{it.rows - taken, it.root, a, it.a1};
    if (rest.rows > 0 || rest.a1 > rest.a0) {
      // keep the pending items sorted: insert the remainder at its place
      auto pos = std::lower_bound(items.begin() + head, items.end(), rest, before);
      items.insert(pos, rest);
    }
  }
  std::sort(parts.begin(), parts.end(), [](const Part& x, const Part& y) {
    if (x.rank != y.rank) return x.rank < y.rank;
    if (x.root != y.root) return x.root < y.root;
    return x.a0 < y.a0;
  });
  *num_parts = (int)parts.size();
  if ((int)parts.size() > max_parts) {
    cb::set_error("plan_shard_parts: more parts than max_parts");
    return CIRCUIT_ERR_ARG;
  }
  for (size_t i = 0; i < parts.size(); ++i) {
    part_root[i] = parts[i].root;
    part_atom_begin[i] = parts[i].a0;
    part_atom_end[i] = parts[i].a1;
    part_rank[i] = parts[i].rank;
  }
  if (rank_rows)
    for (int w = 0; w < world; ++w) rank_rows[w] = load[w];
  return CIRCUIT_OK;
}

}  // extern "C"
