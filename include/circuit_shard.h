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

/* Host-only shard plan that splits oversized roots (no reference counterpart).
 * Root p's rows come as the ordered atoms atom_rows[root_atom_ptr[p] ..
 * root_atom_ptr[p + 1]) -- its children in leaf order, or fixed blocks of rows
 * for a builder that has not clustered children yet; root_atom_ptr has
 * num_roots + 1 entries.  Roots are taken largest first and placed whole on the
 * least-loaded rank when that keeps it within max_imbalance x (total rows /
 * world); otherwise the root is cut between atoms: the least-loaded rank takes
 * the longest prefix that fits (at least one atom) and the rest is planned
 * again.  Every part is a contiguous atom range of one root; a split root's
 * centre and basis are shared by its parts.  A rank exceeds the limit only by
 * less than one atom.  Writes up to max_parts parts (part_root, part_atom_begin,
 * part_atom_end, part_rank), ordered by (rank, root, first atom); *num_parts
 * receives the count; rank_rows[world] (optional) each rank's rows.  With
 * max_imbalance > 1 every split fills a rank, so there are about num_roots +
 * world parts; when max_parts is too small the call returns CIRCUIT_ERR_ARG
 * with *num_parts set to the number needed (num_roots + total atoms always
 * suffices). */
int circuit_plan_shard_parts(const int64_t* atom_rows, const int64_t* root_atom_ptr, int num_roots, int world,
                             double max_imbalance, int* part_root, int64_t* part_atom_begin, int64_t* part_atom_end,
                             int* part_rank, int max_parts, int* num_parts, int64_t* rank_rows);

/* Load rank `rank` of `world`'s shard of a .circuit file onto `device_id`
 * (NULL on failure, circuit_last_error() says why).  The plan is
 * circuit_plan_shard_parts over each root's children in leaf order with the
 * given max_imbalance (e.g. 1.05), identical on every rank; every part the
 * rank owns becomes a root of the returned index with the file root's centre,
 * radius and basis and a contiguous range of its children.  Only those parts'
 * byte ranges of the file are read (mmap + pinned double-buffered staging;
 * adjacent children are copied as one range); original ids stay global, so
 * per-shard results merge with circuit_merge_topk.  Search it like any index.
 * Multi-GPU counterpart of circuit_load_index (reference gpu_index.cpp:50-141
 * loads the whole file). */
circuit_index_t circuit_load_shard(const char* filepath, int rank, int world, int device_id, double max_imbalance);

/* circuit_search_finish_async with a running threshold shared by the shards
 * that search the same query, exchanged while their scans run to tighten each
 * shard's pruning (no reference counterpart: the reference is single-GPU).  Each shard owns
 * one 64-bit word in its GPU's memory, dev_shared_word (8-byte aligned); its
 * main scan raises that word and every peer's (dev_peer_words: a device array
 * of num_peers pointers to the other shards' words, e.g. opened with
 * circuit_ipc_import) with query_tag << 32 | key whenever it finds a higher
 * k-th best, and prunes with the largest key carrying query_tag that it reads
 * from its own word.  Every key is the k-th best score of k real rows of some
 * shard, so it never exceeds the global k-th best and the merged top-k stays
 * exact.  query_tag must be the same on every shard for one query and differ
 * from the previous queries' (a counter); words carrying another tag are
 * ignored, so the words need no clearing between queries.  The peers' words are
 * written with remote atomics while their scans run (no TMA, no multicast).
 * Other arguments and the order of calls as in circuit_search_finish_async. */
int circuit_search_finish_shared_async(circuit_index_t index, const float* dev_query, int k,
                                       const float* dev_threshold_in, unsigned long long* dev_shared_word,
                                       unsigned long long* const* dev_peer_words, int num_peers, uint32_t query_tag,
                                       float* dev_out_scores, int* dev_out_ids, int64_t* dev_out_rows, void* stream,
                                       void* ev_scan_begin, void* ev_scan_end);

/* CUDA IPC for the shared threshold words of shards in separate processes:
 * circuit_ipc_export writes the 64-byte handle of the allocation holding
 * dev_ptr (device memory from cudaMalloc or a caching allocator block; the
 * handle names the start of that allocation, *offset_out the byte offset of
 * dev_ptr in it); circuit_ipc_import opens a handle from another process on
 * device_id (with peer access to the exporter's GPU enabled) and returns the
 * mapped allocation start; circuit_ipc_close unmaps it.  Not for handles of the
 * same process. */
int circuit_ipc_export(const void* dev_ptr, void* handle_out, int64_t* offset_out);
int circuit_ipc_import(const void* handle, int device_id, void** dev_ptr_out);
int circuit_ipc_close(void* dev_ptr);

#ifdef __cplusplus
}
#endif

#endif /* CIRCUIT_SHARD_H */
