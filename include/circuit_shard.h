/*
 * circuit-b200 multi-GPU helpers (no reference counterpart: the reference is
 * single-GPU, reference wiki/Limits-and-FAQ.md:9).
 *
 * The corpus is sharded by root cluster across the GPUs of one node: each GPU
 * holds complete roots (centre, basis, children, leaf rows, original ids) and
 * searches them with circuit_search_async; the per-GPU top-k lists are
 * all-gathered (NCCL, by the host layer) and merged on every rank with
 * circuit_merge_topk.
 */
#ifndef CIRCUIT_SHARD_H
#define CIRCUIT_SHARD_H

#include <stdint.h>

#include "circuit.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Global top-k of n device candidates (scores[n] float32, ids[n] int32 original
 * ids; id < 0 marks an empty slot), ordered by (score desc, id asc).  Writes
 * out_scores[k] / out_ids[k] (-inf / -1 past the last candidate).
 * 1 <= n <= 16384, 1 <= k <= CIRCUIT_MAX_K.  Asynchronous on `stream`. */
int circuit_merge_topk(const float* scores, const int* ids, int n, int k, float* out_scores, int* out_ids,
                       void* stream);

/* Batched form for circuit_search_batch results: scores / ids hold `world`
 * blocks of [num_queries, k_in] (the rank-major layout of an all-gather of each
 * rank's [num_queries, k_in] result); writes out_scores / out_ids
 * [num_queries, k], each row ordered by (score desc, id asc).  One CTA per
 * query.  1 <= world * k_in <= 16384, 1 <= k <= CIRCUIT_MAX_K. */
int circuit_merge_topk_batch(const float* scores, const int* ids, int num_queries, int world, int k_in, int k,
                             float* out_scores, int* out_ids, void* stream);

/* Host-only: assign roots to `world` ranks by longest-processing-time on their
 * leaf rows (heaviest root to the lightest rank).  root_to_rank[num_roots] is
 * written; rank_rows[world] (optional) receives each rank's total rows. */
int circuit_plan_shards(const int64_t* root_rows, int num_roots, int world, int* root_to_rank, int64_t* rank_rows);

#ifdef __cplusplus
}
#endif

#endif /* CIRCUIT_SHARD_H */
