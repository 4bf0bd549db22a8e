// Per-stage operators with the reference torch extension's semantics
// (include/circuit_ops.h).  These evaluate the reference's formulas without
// rounding margins; they are the op-level surface of `circuit_cuda`, not the
// fused search path (search_kernels.cu).
//
// Design: warp-per-root for root bounds and projection (rank up to 64, lanes
// over basis columns, grid-stride over any number of survivors), thread-per-
// child for child bounds, warp-per-row for leaf scoring.  Dot products use
// 128-bit loads when the row pointer allows it and scalar loads otherwise, so
// any dim works.
#include <cmath>
#include <string>

#include "../../include/circuit_ops.h"
#include "common.cuh"
#include "engine.h"
#include "index_internal.h"

namespace cb {
namespace ops {

__device__ __forceinline__ float dot_row(const float* __restrict__ q, const float* __restrict__ x, int dim, int lane) {
  float acc = 0.f;
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(x)) & 15) == 0) {
    const int d4 = dim >> 2;
    const float4* q4 = reinterpret_cast<const float4*>(q);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int c = lane; c < d4; c += 32) {
      const float4 a = __ldg(q4 + c), b = __ldg(x4 + c);
      acc = fmaf(a.x, b.x, acc);
      acc = fmaf(a.y, b.y, acc);
      acc = fmaf(a.z, b.z, acc);
      acc = fmaf(a.w, b.w, acc);
    }
    for (int d = (d4 << 2) + lane; d < dim; d += 32) acc = fmaf(__ldg(q + d), __ldg(x + d), acc);
  } else {
    for (int d = lane; d < dim; d += 32) acc = fmaf(__ldg(q + d), __ldg(x + d), acc);
  }
  return warp_sum(acc);
}

__global__ void k_root_bounds(const float* __restrict__ q, const float* __restrict__ centers,
                              const float* __restrict__ radii, float threshold, float qnorm, int R, int dim,
                              int* __restrict__ mask, int* __restrict__ idx, int* __restrict__ count,
                              float* __restrict__ dots) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int p = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < R; p += warps) {
    const float dot = dot_row(q, centers + (size_t)p * dim, dim, lane);
    if (lane == 0) {
      dots[p] = dot;
      const float bound = dot + qnorm * radii[p];
      if (bound >= threshold) {
        mask[p] = 1;
        idx[atomicAdd(count, 1)] = p;
      } else {
        mask[p] = 0;
      }
    }
  }
}

// count_dev != nullptr: survivor count read from device memory (fused chain).
__global__ void k_project(const float* __restrict__ q, float qn2, const float* __restrict__ bases,
                          const int* __restrict__ surv, int n_surv_host, const int* __restrict__ count_dev, int dim,
                          int rank, float* __restrict__ proj, float* __restrict__ perp) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int n_surv = count_dev ? *count_dev : n_surv_host;
  for (int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < n_surv; s += warps) {
    const int p = surv[s];
    const float* B = bases + (size_t)p * dim * rank;
    float a0 = 0.f, a1 = 0.f;
    const bool c0 = lane < rank, c1 = lane + 32 < rank;
    for (int d = 0; d < dim; ++d) {
      const float qd = __ldg(q + d);
      if (c0) a0 = fmaf(qd, __ldg(B + (size_t)d * rank + lane), a0);
      if (c1) a1 = fmaf(qd, __ldg(B + (size_t)d * rank + lane + 32), a1);
    }
    if (c0) proj[(size_t)p * rank + lane] = a0;
    if (c1) proj[(size_t)p * rank + lane + 32] = a1;
    float n2 = (c0 ? a0 * a0 : 0.f) + (c1 ? a1 * a1 : 0.f);
    n2 = warp_sum(n2);
    if (lane == 0) {
      const float ps = qn2 - n2;
      perp[p] = ps > 0.f ? sqrtf(ps) : 0.f;
    }
  }
}

__global__ void k_child_bounds(const float* __restrict__ proj, const float* __restrict__ perp,
                               const float* __restrict__ dots, const float* __restrict__ L, const float* __restrict__ U,
                               const float* __restrict__ rho, const int* __restrict__ parent,
                               const int* __restrict__ root_mask, float threshold, int C, int rank,
                               int* __restrict__ mask, int* __restrict__ idx, int* __restrict__ count) {
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < C; c += gridDim.x * blockDim.x) {
    const int P = parent[c];
    if (root_mask[P] == 0) { mask[c] = 0; continue; }
    const float* qp = proj + (size_t)P * rank;
    const float* l = L + (size_t)c * rank;
    const float* u = U + (size_t)c * rank;
    float box = 0.f;
    for (int j = 0; j < rank; ++j) {
      const float qj = qp[j];
      box += fmaxf(qj * l[j], qj * u[j]);
    }
    const float ub = dots[P] + box + perp[P] * rho[c];
    if (ub >= threshold) {
      mask[c] = 1;
      idx[atomicAdd(count, 1)] = c;
    } else {
      mask[c] = 0;
    }
  }
}

__global__ void k_fill(float* __restrict__ x, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) x[i] = v;
}

// Block per surviving child (grid-stride), warps over its rows.
__global__ void k_score_children(const float* __restrict__ q, const float* __restrict__ leaf,
                                 const int* __restrict__ offsets, const int* __restrict__ sizes,
                                 const int* __restrict__ surv, int n_surv_host, const int* __restrict__ count_dev,
                                 int dim, float* __restrict__ scores) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int n_surv = count_dev ? *count_dev : n_surv_host;
  for (int s = blockIdx.x; s < n_surv; s += gridDim.x) {
    const int c = surv[s];
    const int off = offsets[c], size = sizes[c];
    for (int i = warp; i < size; i += nw) {
      const int64_t v = (int64_t)off + i;
      const float d = dot_row(q, leaf + v * dim, dim, lane);
      if (lane == 0) scores[v] = d;
    }
  }
}

__global__ void k_flat(const float* __restrict__ q, const float* __restrict__ corpus, int64_t n, int dim,
                       float* __restrict__ scores) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t v = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; v < n; v += warps) {
    const float d = dot_row(q, corpus + v * dim, dim, lane);
    if (lane == 0) scores[v] = d;
  }
}

static int grid_for(int64_t work, int per_block, int cap) {
  int64_t g = (work + per_block - 1) / per_block;
  if (g < 1) g = 1;
  return (int)(g > cap ? cap : g);
}

static int check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return CIRCUIT_OK;
  set_error(std::string(what) + ": " + cudaGetErrorString(e));
  return CIRCUIT_ERR_CUDA;
}

static int bad(const char* msg) {
  set_error(msg);
  return CIRCUIT_ERR_ARG;
}

}  // namespace ops
}  // namespace cb

using namespace cb::ops;

extern "C" {

int circuit_op_evaluate_root_bounds(const float* query, const float* root_centers, const float* root_radii,
                                    float threshold, float query_norm, int num_roots, int dim, int* survivor_mask,
                                    int* survivor_indices, int* num_survivors, float* root_dot_products,
                                    void* stream) {
  if (!query || !root_centers || !root_radii || !survivor_mask || !survivor_indices || !num_survivors ||
      !root_dot_products)
    return bad("evaluate_root_bounds: null pointer");
  if (num_roots <= 0 || dim <= 0) return bad("evaluate_root_bounds: num_roots and dim must be positive");
  cudaStream_t st = (cudaStream_t)stream;
  int rc = check(cudaMemsetAsync(num_survivors, 0, sizeof(int), st), "memset count");
  if (rc) return rc;
  k_root_bounds<<<grid_for(num_roots, 8, 4096), 256, 0, st>>>(query, root_centers, root_radii, threshold, query_norm,
                                                             num_roots, dim, survivor_mask, survivor_indices,
                                                             num_survivors, root_dot_products);
  return check(cudaGetLastError(), "evaluate_root_bounds launch");
}

int circuit_op_project_parents(const float* query, const float* bases, const int* survivor_indices,
                               int num_survivors, int num_bases, int dim, int rank, float query_norm_sq,
                               float* projected_queries, float* perp_norms, void* stream) {
  if (!query || !bases || !projected_queries || !perp_norms) return bad("project_parents: null pointer");
  if (rank < 1 || rank > CIRCUIT_MAX_RANK) return bad("project_parents: rank must be in [1, 64]");
  if (num_bases <= 0 || dim <= 0 || num_survivors < 0 || num_survivors > num_bases)
    return bad("project_parents: bad sizes");
  cudaStream_t st = (cudaStream_t)stream;
  int rc = check(cudaMemsetAsync(projected_queries, 0, sizeof(float) * (size_t)num_bases * rank, st), "memset proj");
  if (!rc) rc = check(cudaMemsetAsync(perp_norms, 0, sizeof(float) * (size_t)num_bases, st), "memset perp");
  if (rc) return rc;
  if (num_survivors == 0) return CIRCUIT_OK;
  if (!survivor_indices) return bad("project_parents: null survivor_indices");
  k_project<<<grid_for(num_survivors, 8, 4096), 256, 0, st>>>(query, query_norm_sq, bases, survivor_indices,
                                                             num_survivors, nullptr, dim, rank, projected_queries,
                                                             perp_norms);
  return check(cudaGetLastError(), "project_parents launch");
}

int circuit_op_evaluate_child_bounds(const float* projected_queries, const float* perp_norms,
                                     const float* root_dot_products, const float* child_intervals_l,
                                     const float* child_intervals_u, const float* child_radii,
                                     const int* child_parent_ids, const int* root_survivor_mask, float threshold,
                                     int num_total_children, int rank, int* child_survivor_mask,
                                     int* child_survivor_indices, int* num_child_survivors, void* stream) {
  if (!projected_queries || !perp_norms || !root_dot_products || !child_intervals_l || !child_intervals_u ||
      !child_radii || !child_parent_ids || !root_survivor_mask || !child_survivor_mask || !child_survivor_indices ||
      !num_child_survivors)
    return bad("evaluate_child_bounds: null pointer");
  if (num_total_children <= 0 || rank < 1) return bad("evaluate_child_bounds: bad sizes");
  cudaStream_t st = (cudaStream_t)stream;
  int rc = check(cudaMemsetAsync(num_child_survivors, 0, sizeof(int), st), "memset count");
  if (rc) return rc;
  k_child_bounds<<<grid_for(num_total_children, 256, 8192), 256, 0, st>>>(
      projected_queries, perp_norms, root_dot_products, child_intervals_l, child_intervals_u, child_radii,
      child_parent_ids, root_survivor_mask, threshold, num_total_children, rank, child_survivor_mask,
      child_survivor_indices, num_child_survivors);
  return check(cudaGetLastError(), "evaluate_child_bounds launch");
}

int circuit_op_score_surviving_leaves(const float* query, const float* leaf_vectors, const int* leaf_offsets,
                                      const int* leaf_sizes, const int* child_survivor_indices, int num_survivors,
                                      int64_t n, int dim, float* vector_scores, void* stream) {
  if (!query || !leaf_vectors || !leaf_offsets || !leaf_sizes || !vector_scores)
    return bad("score_surviving_leaves: null pointer");
  if (n <= 0 || dim <= 0 || num_survivors < 0) return bad("score_surviving_leaves: bad sizes");
  cudaStream_t st = (cudaStream_t)stream;
  k_fill<<<grid_for(n, 256, 4096), 256, 0, st>>>(vector_scores, n, -1e9f);
  int rc = check(cudaGetLastError(), "fill launch");
  if (rc || num_survivors == 0) return rc;
  if (!child_survivor_indices) return bad("score_surviving_leaves: null survivor list");
  k_score_children<<<grid_for(num_survivors, 1, 8192), 256, 0, st>>>(
      query, leaf_vectors, leaf_offsets, leaf_sizes, child_survivor_indices, num_survivors, nullptr, dim,
      vector_scores);
  return check(cudaGetLastError(), "score_surviving_leaves launch");
}

int circuit_op_flat_exact_score(const float* query, const float* corpus, int64_t n, int dim, float* scores,
                                void* stream) {
  if (!query || !corpus || !scores) return bad("flat_exact_score: null pointer");
  if (n <= 0 || dim <= 0) return bad("flat_exact_score: bad sizes");
  cudaStream_t st = (cudaStream_t)stream;
  k_flat<<<grid_for(n, 8, 148 * 16), 256, 0, st>>>(query, corpus, n, dim, scores);
  return check(cudaGetLastError(), "flat_exact_score launch");
}

int circuit_op_hierarchical_search(const float* query, const float* root_centers, const float* root_radii,
                                   const float* bases, const float* child_intervals_l,
                                   const float* child_intervals_u, const float* child_radii,
                                   const int* child_parent_ids, const float* leaf_vectors, const int* leaf_offsets,
                                   const int* leaf_sizes, int* survivor_mask, int* survivor_indices,
                                   int* num_survivors, float* root_dot_products, float* projected_queries,
                                   float* perp_norms, int* child_survivor_mask, int* child_survivor_indices,
                                   int* num_child_survivors, float* vector_scores, int num_roots,
                                   int num_total_children, int64_t n, int dim, float threshold, int rank,
                                   float query_norm, void* stream) {
  if (!query || !root_centers || !root_radii || !bases || !child_intervals_l || !child_intervals_u ||
      !child_radii || !child_parent_ids || !leaf_vectors || !leaf_offsets || !leaf_sizes || !survivor_mask ||
      !survivor_indices || !num_survivors || !root_dot_products || !projected_queries || !perp_norms ||
      !child_survivor_mask || !child_survivor_indices || !num_child_survivors || !vector_scores)
    return bad("hierarchical_search: null pointer");
  if (rank < 1 || rank > CIRCUIT_MAX_RANK) return bad("hierarchical_search: rank must be in [1, 64]");
  if (num_roots <= 0 || num_total_children <= 0 || n <= 0 || dim <= 0) return bad("hierarchical_search: bad sizes");
  cudaStream_t st = (cudaStream_t)stream;
  int rc = check(cudaMemsetAsync(num_survivors, 0, sizeof(int), st), "memset");
  if (!rc) rc = check(cudaMemsetAsync(num_child_survivors, 0, sizeof(int), st), "memset");
  if (rc) return rc;
  k_fill<<<grid_for(n, 256, 4096), 256, 0, st>>>(vector_scores, n, -1e9f);
  k_root_bounds<<<grid_for(num_roots, 8, 4096), 256, 0, st>>>(query, root_centers, root_radii, threshold, query_norm,
                                                             num_roots, dim, survivor_mask, survivor_indices,
                                                             num_survivors, root_dot_products);
  k_project<<<grid_for(num_roots, 8, 4096), 256, 0, st>>>(query, query_norm * query_norm, bases, survivor_indices, 0,
                                                         num_survivors, dim, rank, projected_queries, perp_norms);
  k_child_bounds<<<grid_for(num_total_children, 256, 8192), 256, 0, st>>>(
      projected_queries, perp_norms, root_dot_products, child_intervals_l, child_intervals_u, child_radii,
      child_parent_ids, survivor_mask, threshold, num_total_children, rank, child_survivor_mask,
      child_survivor_indices, num_child_survivors);
  k_score_children<<<grid_for(num_total_children, 1, 8192), 256, 0, st>>>(
      query, leaf_vectors, leaf_offsets, leaf_sizes, child_survivor_indices, 0, num_child_survivors, dim,
      vector_scores);
  return check(cudaGetLastError(), "hierarchical_search launch");
}

}  // extern "C"
