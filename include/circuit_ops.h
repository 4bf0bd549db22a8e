/*
 * circuit-b200 per-stage operators: the C ABI behind the Python `circuit_cuda`
 * module, one function per op of the reference torch extension
 * (reference native/bindings/torch_extension.cpp:236-257).  Same argument
 * meaning and output semantics as the reference op; tensors are passed as raw
 * device pointers plus sizes, and every call is asynchronous on `stream`
 * (a cudaStream_t; NULL = legacy default stream).
 *
 * These ops evaluate the reference's bound formulas exactly as written there
 * (no rounding margin) so they can be compared element by element with the
 * reference kernels; the fused search of include/circuit.h is the path that
 * inflates every bound by a rigorous fp32 margin.
 *
 * Output buffers are fully written by each op (masks, counts, zero / -1e9
 * fills), so callers may pass uninitialised memory.
 * Like the reference ops, these take the index tables as given: the sizes and
 * pointers are checked on the host, but survivor lists, parent ids and leaf
 * offsets / sizes are used as indices on the device without a range check, so
 * they must describe a valid index (one that circuit_load_index or
 * circuit_index_from_device accepts: those validate every table once).
 * Return value: 0 on success, a negative CIRCUIT_ERR_* code otherwise
 * (description in circuit_last_error()).
 */
#ifndef CIRCUIT_OPS_H
#define CIRCUIT_OPS_H

#include <stdint.h>

#include "circuit.h"

#ifdef __cplusplus
extern "C" {
#endif

/* reference evaluate_root_bounds_cuda (torch_extension.cpp:10-47, root_bounds.cu:11-56):
 * dots[r] = q.c_r; mask[r] = (dots[r] + query_norm * radii[r] >= threshold);
 * indices[0..count) = surviving roots (unspecified order); *count written. */
int circuit_op_evaluate_root_bounds(const float* query, const float* root_centers, const float* root_radii,
                                    float threshold, float query_norm, int num_roots, int dim, int* survivor_mask,
                                    int* survivor_indices, int* num_survivors, float* root_dot_products,
                                    void* stream);

/* reference project_parents_cuda (torch_extension.cpp:49-81, parent_projection.cu:11-65):
 * for each of the first num_survivors entries p of survivor_indices:
 *   projected[p, j] = sum_d q[d] * bases[p, d, j]     (j < rank <= 64)
 *   perp[p] = sqrt(max(query_norm_sq - ||projected[p]||^2, 0))
 * every other row of projected / perp is zero.  No survivor limit (the
 * reference device-count kernel projects at most 512 roots, dispatch.cu:284). */
int circuit_op_project_parents(const float* query, const float* bases, const int* survivor_indices,
                               int num_survivors, int num_bases, int dim, int rank, float query_norm_sq,
                               float* projected_queries, float* perp_norms, void* stream);

/* reference evaluate_child_bounds_cuda (torch_extension.cpp:83-119, child_bounds.cu:11-83):
 * child c of a surviving parent P survives iff
 *   dots[P] + sum_j max(qP_j l_cj, qP_j u_cj) + perp[P] * rho_c >= threshold. */
int circuit_op_evaluate_child_bounds(const float* projected_queries, const float* perp_norms,
                                     const float* root_dot_products, const float* child_intervals_l,
                                     const float* child_intervals_u, const float* child_radii,
                                     const int* child_parent_ids, const int* root_survivor_mask, float threshold,
                                     int num_total_children, int rank, int* child_survivor_mask,
                                     int* child_survivor_indices, int* num_child_survivors, void* stream);

/* reference score_surviving_leaves_cuda (torch_extension.cpp:121-149, dense_score.cu:9-59):
 * vector_scores[0..n) = -1e9, then q.x_v for every row v of the listed children. */
int circuit_op_score_surviving_leaves(const float* query, const float* leaf_vectors, const int* leaf_offsets,
                                      const int* leaf_sizes, const int* child_survivor_indices, int num_survivors,
                                      int64_t n, int dim, float* vector_scores, void* stream);

/* reference flat_exact_score_cuda (torch_extension.cpp:224-234, dense_score.cu:169-212):
 * scores[v] = q.x_v for v < n. */
int circuit_op_flat_exact_score(const float* query, const float* corpus, int64_t n, int dim, float* scores,
                                void* stream);

/* reference hierarchical_search_cuda (torch_extension.cpp:151-222, dispatch.cu:244-307):
 * in place on the caller's workspaces: vector_scores = -1e9, counters = 0, then
 * root bounds -> projection of every surviving root -> child bounds -> scores of
 * every surviving child's rows, with survivor counts read on the device. */
int circuit_op_hierarchical_search(const float* query, const float* root_centers, const float* root_radii,
                                   const float* bases, const float* child_intervals_l,
                                   const float* child_intervals_u, const float* child_radii,
                                   const int* child_parent_ids, const float* leaf_vectors, const int* leaf_offsets,
                                   const int* leaf_sizes, int* survivor_mask, int* survivor_indices,
                                   int* num_survivors, float* root_dot_products, float* projected_queries,
                                   float* perp_norms, int* child_survivor_mask, int* child_survivor_indices,
                                   int* num_child_survivors, float* vector_scores, int num_roots,
                                   int num_total_children, int64_t n, int dim, float threshold, int rank,
                                   float query_norm, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CIRCUIT_OPS_H */
