"""circuit_cuda: the six per-stage ops of the reference torch extension
(reference native/bindings/torch_extension.cpp:236-257), same op names,
argument names, defaults and output semantics, implemented over the C ABI of
include/circuit_ops.h (libcircuit.so).  Every op runs on the current torch
stream (the reference's first four ops used stream 0) and raises RuntimeError
when an argument is not a CUDA tensor (reference TORCH_CHECKs,
torch_extension.cpp:17-19, :57-58, :225).
"""
from typing import List

import torch

from circuit_rag import _native

__all__ = ["evaluate_root_bounds", "project_parents", "evaluate_child_bounds", "score_surviving_leaves",
           "flat_exact_score", "hierarchical_search"]


def _cuda(t: torch.Tensor, name: str, dtype) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be CUDA tensor")
    if t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def evaluate_root_bounds(query, root_centers, root_radii, threshold, query_norm=1.0) -> List[torch.Tensor]:
    q = _cuda(query, "query", torch.float32)
    c = _cuda(root_centers, "root_centers", torch.float32)
    r = _cuda(root_radii, "root_radii", torch.float32)
    R, dim = c.shape[0], q.shape[0]
    o_i = dict(dtype=torch.int32, device=q.device)
    mask = torch.zeros(R, **o_i)
    idx = torch.zeros(R, **o_i)
    count = torch.zeros(1, **o_i)
    dots = torch.empty(R, dtype=torch.float32, device=q.device)
    rc = _native.lib().circuit_op_evaluate_root_bounds(
        q.data_ptr(), c.data_ptr(), r.data_ptr(), float(threshold), float(query_norm), R, dim, mask.data_ptr(),
        idx.data_ptr(), count.data_ptr(), dots.data_ptr(), _stream(q))
    _native.check(rc, "evaluate_root_bounds")
    return [mask, idx, count, dots]


def project_parents(query, bases, survivor_indices, num_survivors, rank, query_norm_sq=1.0) -> List[torch.Tensor]:
    q = _cuda(query, "query", torch.float32)
    b = _cuda(bases, "bases", torch.float32)
    s = survivor_indices.to(device=q.device, dtype=torch.int32).contiguous()
    nb = b.shape[0]
    proj = torch.zeros((nb, int(rank)), dtype=torch.float32, device=q.device)
    perp = torch.zeros(nb, dtype=torch.float32, device=q.device)
    rc = _native.lib().circuit_op_project_parents(
        q.data_ptr(), b.data_ptr(), s.data_ptr(), int(num_survivors), nb, q.shape[0], int(rank),
        float(query_norm_sq), proj.data_ptr(), perp.data_ptr(), _stream(q))
    _native.check(rc, "project_parents")
    return [proj, perp]


def evaluate_child_bounds(projected_queries, perp_norms, root_dot_products, child_intervals_l, child_intervals_u,
                          child_radii, child_parent_ids, root_survivor_mask, threshold, rank) -> List[torch.Tensor]:
    pq = _cuda(projected_queries, "projected_queries", torch.float32)
    pn = _cuda(perp_norms, "perp_norms", torch.float32)
    rd = _cuda(root_dot_products, "root_dot_products", torch.float32)
    lo = _cuda(child_intervals_l, "child_intervals_l", torch.float32)
    up = _cuda(child_intervals_u, "child_intervals_u", torch.float32)
    cr = _cuda(child_radii, "child_radii", torch.float32)
    cp = _cuda(child_parent_ids, "child_parent_ids", torch.int32)
    rm = _cuda(root_survivor_mask, "root_survivor_mask", torch.int32)
    C = cr.shape[0]
    o_i = dict(dtype=torch.int32, device=pq.device)
    mask = torch.zeros(C, **o_i)
    idx = torch.zeros(C, **o_i)
    count = torch.zeros(1, **o_i)
    rc = _native.lib().circuit_op_evaluate_child_bounds(
        pq.data_ptr(), pn.data_ptr(), rd.data_ptr(), lo.data_ptr(), up.data_ptr(), cr.data_ptr(), cp.data_ptr(),
        rm.data_ptr(), float(threshold), C, int(rank), mask.data_ptr(), idx.data_ptr(), count.data_ptr(),
        _stream(pq))
    _native.check(rc, "evaluate_child_bounds")
    return [mask, idx, count]


def score_surviving_leaves(query, leaf_vectors, leaf_offsets, leaf_sizes, child_survivor_indices,
                           num_survivors) -> List[torch.Tensor]:
    q = _cuda(query, "query", torch.float32)
    x = _cuda(leaf_vectors, "leaf_vectors", torch.float32)
    off = _cuda(leaf_offsets, "leaf_offsets", torch.int32)
    sz = _cuda(leaf_sizes, "leaf_sizes", torch.int32)
    s = child_survivor_indices.to(device=q.device, dtype=torch.int32).contiguous()
    N = x.shape[0]
    scores = torch.empty(N, dtype=torch.float32, device=q.device)
    rc = _native.lib().circuit_op_score_surviving_leaves(
        q.data_ptr(), x.data_ptr(), off.data_ptr(), sz.data_ptr(), s.data_ptr(), int(num_survivors), N, q.shape[0],
        scores.data_ptr(), _stream(q))
    _native.check(rc, "score_surviving_leaves")
    return [scores]


def flat_exact_score(query, corpus) -> torch.Tensor:
    if not (isinstance(query, torch.Tensor) and isinstance(corpus, torch.Tensor) and query.is_cuda and corpus.is_cuda):
        raise RuntimeError("query and corpus must be CUDA tensors")
    q = query.to(torch.float32).contiguous()
    x = corpus.to(torch.float32).contiguous()
    N, dim = x.shape
    scores = torch.empty(N, dtype=torch.float32, device=q.device)
    rc = _native.lib().circuit_op_flat_exact_score(q.data_ptr(), x.data_ptr(), N, dim, scores.data_ptr(), _stream(q))
    _native.check(rc, "flat_exact_score")
    return scores


def hierarchical_search(query, root_centers, root_radii, bases, child_intervals_l, child_intervals_u, child_radii,
                        child_parent_ids, leaf_vectors, leaf_offsets, leaf_sizes, survivor_mask, survivor_indices,
                        num_survivors, root_dot_products, projected_queries, perp_norms, child_survivor_mask,
                        child_survivor_indices, num_child_survivors, vector_scores, threshold, rank,
                        query_norm=1.0) -> torch.Tensor:
    """In place on the workspaces, like the reference (torch_extension.cpp:151-222); returns vector_scores."""
    ins = [_cuda(query, "query", torch.float32), _cuda(root_centers, "root_centers", torch.float32),
           _cuda(root_radii, "root_radii", torch.float32), _cuda(bases, "bases", torch.float32),
           _cuda(child_intervals_l, "child_intervals_l", torch.float32),
           _cuda(child_intervals_u, "child_intervals_u", torch.float32),
           _cuda(child_radii, "child_radii", torch.float32), _cuda(child_parent_ids, "child_parent_ids", torch.int32),
           _cuda(leaf_vectors, "leaf_vectors", torch.float32), _cuda(leaf_offsets, "leaf_offsets", torch.int32),
           _cuda(leaf_sizes, "leaf_sizes", torch.int32)]
    ws = [survivor_mask, survivor_indices, num_survivors, root_dot_products, projected_queries, perp_norms,
          child_survivor_mask, child_survivor_indices, num_child_survivors, vector_scores]
    want = [torch.int32, torch.int32, torch.int32, torch.float32, torch.float32, torch.float32, torch.int32,
            torch.int32, torch.int32, torch.float32]
    for t, dt in zip(ws, want):
        if not t.is_cuda or t.dtype != dt or not t.is_contiguous():
            raise RuntimeError("workspace tensors must be contiguous CUDA tensors of the reference dtypes")
    q = ins[0]
    rc = _native.lib().circuit_op_hierarchical_search(
        *[t.data_ptr() for t in ins], *[t.data_ptr() for t in ws], ins[1].shape[0], ins[6].shape[0],
        ins[8].shape[0], q.shape[0], float(threshold), int(rank), float(query_norm), _stream(q))
    _native.check(rc, "hierarchical_search")
    return vector_scores
