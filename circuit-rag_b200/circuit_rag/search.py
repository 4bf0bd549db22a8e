"""circuit_search: exact top-k inner-product search (reference
circuit_rag/search.py:45-84), same signature, same results as brute force.

The whole search is one call into libcircuit.so on the current torch stream:
root scan -> on-device seed threshold -> rigorous root / child bounds -> fused
leaf scan + top-k -> original ids.  Unlike the reference there is no host
synchronisation inside a search (the reference syncs 7 times, search.py:26-41,
:75, :78-83), no O(N) score buffer, and no torch.topk over N.

SearchTrace keeps the reference's fields; the device-side ones
(seed_threshold, surviving_children, total_gpu_time_us, ...) are captured
asynchronously and resolved on first access, so tracing costs no sync per query.
"""
import ctypes
from typing import Tuple

import torch

from circuit_rag import _native
from circuit_rag.hierarchy.build import CircuitIndex


class SearchTrace:
    """Per-search statistics (reference search.py:12-19 fields plus
    vectors_scored, surviving_roots, pruned_fraction, best_root, rows_streamed).

    vectors_scored / pruned_fraction describe the bounds: the rows of the
    children whose rigorous bound is not below the seed threshold.
    rows_streamed counts the rows the main scan read; it runs beside the bounds
    kernel, so it streams children whose bound is not known yet (a small
    corpus streams whole before the bounds are ready) and skips children whose
    bound is below the threshold it has raised by then."""

    _LAZY = ("seed_threshold", "surviving_children", "surviving_roots", "vectors_scored", "best_root",
             "total_gpu_time_us", "pruned_fraction", "rows_streamed")

    def __init__(self):
        self.corpus_size = 0
        self.path = ""
        self.total_children = 0
        self._pending = None
        self._values = {"seed_threshold": -1e9, "surviving_children": -1, "surviving_roots": -1,
                        "vectors_scored": -1, "best_root": -1, "total_gpu_time_us": 0.0, "pruned_fraction": 0.0,
                        "rows_streamed": -1}

    def _resolve(self):
        if self._pending is None:
            return
        index, snap, path, ev0, ev1, ev2 = self._pending
        self._pending = None
        ev2.synchronize()
        host = snap.cpu()
        tx = _native.TraceEx()
        rc = _native.lib().circuit_trace_decode(index.native_handle(), host.data_ptr(), path, ctypes.byref(tx))
        _native.check(rc, "search (device-side error)")
        v = self._values
        v["total_gpu_time_us"] = ev0.elapsed_time(ev1) * 1000.0
        v["vectors_scored"] = int(tx.vectors_scored)
        v["pruned_fraction"] = 1.0 - tx.vectors_scored / max(1, tx.vectors_total)
        v["rows_streamed"] = int(tx.rows_streamed)
        if path:
            v["seed_threshold"] = float(tx.seed_threshold) if tx.seed_threshold > float("-inf") else -1e9
            v["surviving_children"] = int(tx.surviving_children)
            v["surviving_roots"] = int(tx.surviving_roots)
            v["best_root"] = int(tx.best_root)

    def __getattr__(self, name):
        if name in SearchTrace._LAZY:
            self._resolve()
            return self._values[name]
        raise AttributeError(name)

    def __setattr__(self, name, value):
        if name in SearchTrace._LAZY:
            self._resolve()
            self._values[name] = value
        else:
            object.__setattr__(self, name, value)

    def as_dict(self):
        self._resolve()
        d = {"corpus_size": self.corpus_size, "path": self.path, "total_children": self.total_children}
        d.update(self._values)
        return d


def _launch(handle, query, k, min_hierarchy_n, out_scores, out_ids, out_rows, stream, ev0=None, ev1=None):
    rc = _native.lib().circuit_search_async(
        handle, query.data_ptr(), int(k), int(min_hierarchy_n), out_scores.data_ptr(),
        out_ids.data_ptr() if out_ids is not None else None,
        out_rows.data_ptr() if out_rows is not None else None,
        stream.cuda_stream, ev0.cuda_event if ev0 is not None else None,
        ev1.cuda_event if ev1 is not None else None)
    _native.check(rc, "circuit_search")


def circuit_search(query: torch.Tensor, index: CircuitIndex, k: int = 10,
                   min_hierarchy_n: int = 10000) -> Tuple[torch.Tensor, torch.Tensor, SearchTrace]:
    """Exact top-k by inner product.  Returns (scores [k] float32 descending,
    original ids [k] int32, SearchTrace).  Raises ValueError on a bad query
    shape (reference search.py:48-49) or k outside [1, 256]."""
    if query.ndim != 1 or query.numel() != index.dim:
        raise ValueError("query must have shape [index.dim]")
    if not index.is_cuda:
        raise RuntimeError("circuit-b200 searches run on a CUDA device (no CPU path); load or build the index "
                           "with device='cuda'")
    k = min(int(k), index.N)
    if k < 1 or k > _native.CIRCUIT_MAX_K:
        raise ValueError(f"k must be in [1, {_native.CIRCUIT_MAX_K}]")
    dev = index.leaf_vectors.device
    query = query.to(device=dev, dtype=torch.float32).contiguous()
    if query.data_ptr() % 16:
        query = query.clone()
    handle = index.native_handle()
    trace = SearchTrace()
    trace.corpus_size = index.N
    trace.total_children = index.num_total_children
    hier = index.N >= min_hierarchy_n
    trace.path = "hierarchical" if hier else "flat"
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream()
        scores = torch.empty(k, dtype=torch.float32, device=dev)
        ids = torch.empty(k, dtype=torch.int32, device=dev)
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        _launch(handle, query, k, min_hierarchy_n, scores, ids, None, stream)
        ev1.record(stream)
        snap = torch.empty(_native.TRACE_SNAPSHOT_BYTES, dtype=torch.uint8, device=dev)
        _native.check(_native.lib().circuit_trace_snapshot_async(handle, snap.data_ptr(), stream.cuda_stream),
                      "trace snapshot")
        ev2 = torch.cuda.Event()
        ev2.record(stream)
        trace._pending = (index, snap, 1 if hier else 0, ev0, ev1, ev2)
    return scores, ids, trace


def circuit_search_batch(queries: torch.Tensor, index: CircuitIndex, k: int = 10) -> Tuple[torch.Tensor, torch.Tensor]:
    """Exact top-k for a batch of queries [B, dim] on the tensor cores.

    No reference counterpart (the reference answers one query per call); the
    results equal B calls of circuit_search: a tf32 tcgen05 pass over every
    leaf row keeps each query's rows within a rigorous error band of its running
    k-th best, and those rows are rescored exactly in fp32.  Returns (scores
    [B, k] float32 descending, original ids [B, k] int32), 1 <= k <= 256.
    A query whose candidate list overflows
    (more rows inside the error band than the batch's candidate pool holds:
    16,384 per query for 4,096 queries, up to 65,536 for smaller batches) is
    answered by circuit_search."""
    if queries.ndim != 2 or queries.shape[1] != index.dim:
        raise ValueError("queries must have shape [B, index.dim]")
    if not index.is_cuda:
        raise RuntimeError("circuit-b200 searches run on a CUDA device (no CPU path); load or build the index "
                           "with device='cuda'")
    k = min(int(k), index.N)
    if k < 1 or k > _native.CIRCUIT_MAX_K:
        raise ValueError(f"k must be in [1, {_native.CIRCUIT_MAX_K}]")
    B = queries.shape[0]
    dev = index.leaf_vectors.device
    queries = queries.to(device=dev, dtype=torch.float32).contiguous()
    if queries.data_ptr() % 16:
        queries = queries.clone()
    handle = index.native_handle()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream()
        scores = torch.empty(B, k, dtype=torch.float32, device=dev)
        ids = torch.empty(B, k, dtype=torch.int32, device=dev)
        if B == 0:
            return scores, ids
        rc = _native.lib().circuit_search_batch_async(handle, queries.data_ptr(), B, k, scores.data_ptr(),
                                                      ids.data_ptr(), stream.cuda_stream, None, None)
        _native.check(rc, "circuit_search_batch")
        n_over = ctypes.c_int(0)
        if k <= _native.CIRCUIT_BATCH_MAX_K:
            _native.check(_native.lib().circuit_batch_overflow(handle, ctypes.byref(n_over)),
                          "circuit_batch_overflow")
        if n_over.value:
            for q in torch.nonzero(ids[:, 0] == -2).flatten().tolist():
                s1, i1, _ = circuit_search(queries[q], index, k)
                scores[q] = s1
                ids[q] = i1
    return scores, ids
