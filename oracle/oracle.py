"""circuit oracle -- TEST INFRASTRUCTURE ONLY (the checker, never the product).

CPU restatement of the reference's exact top-k search path, used only by
tests/, __graft_entry__.smoke() and the CPU-baseline leg of bench.py:

* brute force, exactly the reference's own oracle: ``topk(X @ q)``
  (reference tests/test_exact.py:26, circuit_rag/search.py:58-61), in float64
  for truth and in torch float32 for the timed CPU baseline;
* the reference's seed threshold (circuit_rag/search.py:26-41), bound kernels
  (native/kernels/root_bounds.cu:31-54, parent_projection.cu:34-64,
  child_bounds.cu:30-82) and hierarchical pipeline, in plain C
  (oracle/circuit_oracle.c, built to oracle/_build/liboracle.so);
* a .circuit reader restating the reference format
  (circuit_rag/storage/format.py:82-142);
* ``check_topk``: the parity rule -- ids identical to brute force except among
  scores tied within 1e-6 absolute, scores within 1e-5 relative.

Pinned against the reference: tests/test_oracle_golden.py checks this module
against fixtures produced by the reference package itself
(tests/golden/make_golden.py).
"""
import ctypes
import json
import os
import struct
import subprocess
from typing import Dict, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "liboracle.so")

TIE_ABS = 1e-6
SCORE_REL = 1e-5

_lib = None


def lib():
    """ctypes handle of liboracle.so (compiled with gcc on first use if missing)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            subprocess.run(["make", "-C", HERE, "oracle"], check=True, capture_output=True)
        L = ctypes.CDLL(LIB)
        P, I, I64, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_double
        L.oracle_root_bounds.restype = I
        L.oracle_root_bounds.argtypes = [P, P, P, I, I, D, D, I, P, P]
        L.oracle_project.restype = None
        L.oracle_project.argtypes = [P, P, P, I, I, I, D, I, P, P]
        L.oracle_child_bounds.restype = I
        L.oracle_child_bounds.argtypes = [P, P, P, P, P, P, P, P, I, I, D, P, P]
        L.oracle_brute_topk.restype = I
        L.oracle_brute_topk.argtypes = [P, I64, I, P, I, P, P]
        L.oracle_seed_threshold.restype = D
        L.oracle_seed_threshold.argtypes = [P, P, I, I, P, P, I, P, I, I, P]
        L.oracle_hierarchical_search.restype = I
        L.oracle_hierarchical_search.argtypes = [P] * 12 + [I, I, I64, I, I, I, P, P, P, P]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


# ------------------------------------------------------------------ .circuit reader
TENSORS = ("root_centers", "root_radii", "bases", "child_intervals_l", "child_intervals_u", "child_radii",
           "child_parent_ids", "leaf_offsets", "leaf_sizes", "leaf_vectors", "original_ids")


def read_circuit(path: str) -> Dict[str, object]:
    """numpy arrays of a .circuit file + its header ints (reference format.py:82-142)."""
    with open(path, "rb") as f:
        if f.read(8) != b"CIRCUIT1":
            raise ValueError("bad magic")
        hlen = struct.unpack("<I", f.read(4))[0]
        meta = json.loads(f.read(hlen).decode("utf-8").rstrip("\x00"))
        out: Dict[str, object] = {k: int(meta[k]) for k in ("dim", "rank", "num_roots", "num_total_children", "N")}
        for name in TENSORS:
            info = meta["tensor_meta"][name]
            f.seek(int(info["offset"]))
            arr = np.frombuffer(f.read(int(info["nbytes"])), dtype=np.dtype(info["dtype"]))
            out[name] = arr.reshape(tuple(info["shape"])).copy()
    return out


def corpus_from_index(ix: Dict[str, object]) -> np.ndarray:
    """The original corpus X (rows by original id) recovered from an index."""
    X = np.empty_like(ix["leaf_vectors"])
    X[ix["original_ids"]] = ix["leaf_vectors"]
    return X


# ------------------------------------------------------------------ brute force
def exact_scores(X: np.ndarray, q: np.ndarray) -> np.ndarray:
    """float64 X q (products of float32 values are exact in float64)."""
    return X.astype(np.float64) @ q.astype(np.float64)


def brute_topk(X: np.ndarray, q: np.ndarray, k: int) -> Tuple[np.ndarray, np.ndarray]:
    """(scores desc, rows) by (score desc, row asc), float64."""
    s = exact_scores(X, q)
    k = min(k, len(s))
    part = np.argpartition(-s, k - 1)[:k] if k < len(s) else np.arange(len(s))
    order = np.lexsort((part, -s[part]))
    rows = part[order]
    return s[rows], rows


def brute_topk_c(X: np.ndarray, q: np.ndarray, k: int) -> Tuple[np.ndarray, np.ndarray]:
    """Same as brute_topk, through the C restatement."""
    X, q = _f32(X), _f32(q)
    out_s = np.empty(k, np.float64)
    out_r = np.empty(k, np.int64)
    m = lib().oracle_brute_topk(_p(X), X.shape[0], X.shape[1], _p(q), k, _p(out_s), _p(out_r))
    return out_s[:m], out_r[:m]


def torch_flat_search(X, q, k):
    """The reference's CPU path, verbatim formulation (circuit_rag/search.py:58-61):
    ``topk(leaf_vectors @ query, k)`` in float32 torch.  Used for the timed CPU baseline."""
    import torch

    return torch.topk(X @ q, k)


def torch_batch_flat_search(X, Q, k):
    """Batched form of the same brute force, ``topk(Q @ X.T, k, dim=1)`` (the
    reference's exactness test computes its truth this way per query,
    tests/test_exact.py:26).  Used for the timed CPU baseline of batches."""
    import torch

    return torch.topk(Q @ X.T, k, dim=1)


# ------------------------------------------------------------------ reference pipeline pieces
def seed_threshold(ix, q: np.ndarray, k: int, f64: bool = False) -> Tuple[float, int]:
    """reference search.py:26-41 -> (T, best_root)."""
    q = _f32(q)
    best = ctypes.c_int(-1)
    T = lib().oracle_seed_threshold(_p(q), _p(_f32(ix["root_centers"])), ix["num_roots"], ix["dim"],
                                    _p(_i32(ix["leaf_offsets"])), _p(_i32(ix["leaf_sizes"])),
                                    ix["num_total_children"], _p(_f32(ix["leaf_vectors"])), k, int(f64),
                                    ctypes.byref(best))
    return T, best.value


def root_bounds(q, centers, radii, query_norm, threshold, f64=True):
    q, centers, radii = _f32(q), _f32(centers), _f32(radii)
    R, D = centers.shape
    mask = np.zeros(R, np.int32)
    dots = np.zeros(R, np.float64)
    lib().oracle_root_bounds(_p(q), _p(centers), _p(radii), R, D, float(query_norm), float(threshold), int(f64),
                             _p(mask), _p(dots))
    return mask, dots


def project(q, bases, roots, query_norm_sq, f64=True):
    q, bases = _f32(q), _f32(bases)
    roots = _i32(roots)
    R, D, r = bases.shape
    proj = np.zeros((R, r), np.float64)
    perp = np.zeros(R, np.float64)
    lib().oracle_project(_p(q), _p(bases), _p(roots), len(roots), D, r, float(query_norm_sq), int(f64), _p(proj),
                         _p(perp))
    return proj, perp


def child_bounds(proj, perp, dots, L, U, rho, parent, root_mask, threshold):
    proj = np.ascontiguousarray(proj, np.float64)
    perp = np.ascontiguousarray(perp, np.float64)
    dots = np.ascontiguousarray(dots, np.float64)
    L, U, rho = _f32(L), _f32(U), _f32(rho)
    parent, root_mask = _i32(parent), _i32(root_mask)
    C, r = L.shape
    mask = np.zeros(C, np.int32)
    ub = np.zeros(C, np.float64)
    lib().oracle_child_bounds(_p(proj), _p(perp), _p(dots), _p(L), _p(U), _p(rho), _p(parent), _p(root_mask), C, r,
                              float(threshold), _p(mask), _p(ub))
    return mask, ub


def hierarchical_search(ix, q, k):
    """The reference hierarchical pipeline on CPU -> (scores, ids, rows_scored, child_mask)."""
    q = _f32(q)
    out_s = np.empty(k, np.float64)
    out_i = np.empty(k, np.int32)
    scored = ctypes.c_int64(0)
    cmask = np.zeros(ix["num_total_children"], np.int32)
    m = lib().oracle_hierarchical_search(
        _p(q), _p(_f32(ix["root_centers"])), _p(_f32(ix["root_radii"])), _p(_f32(ix["bases"])),
        _p(_f32(ix["child_intervals_l"])), _p(_f32(ix["child_intervals_u"])), _p(_f32(ix["child_radii"])),
        _p(_i32(ix["child_parent_ids"])), _p(_i32(ix["leaf_offsets"])), _p(_i32(ix["leaf_sizes"])),
        _p(_f32(ix["leaf_vectors"])), _p(_i32(ix["original_ids"])), ix["num_roots"], ix["num_total_children"],
        ix["N"], ix["dim"], ix["rank"], k, _p(out_s), _p(out_i), ctypes.byref(scored), _p(cmask))
    return out_s[:m], out_i[:m], scored.value, cmask


# ------------------------------------------------------------------ parity rule
def check_topk(exact: np.ndarray, k: int, got_scores, got_ids, tie_abs: float = TIE_ABS,
               score_rel: float = SCORE_REL) -> None:
    """Raise AssertionError unless (got_scores, got_ids) is the exact top-k of
    ``exact`` (float64 scores indexed by id): ids identical to brute force except
    among scores within ``tie_abs`` of the k-th; every score within
    ``score_rel`` relative (plus tie_abs absolute) of the exact score; scores
    sorted descending."""
    got_scores = np.asarray(got_scores, np.float64)
    got_ids = np.asarray(got_ids, np.int64)
    k = min(k, len(exact))
    assert got_ids.shape == (k,), f"expected {k} ids, got {got_ids.shape}"
    assert len(set(got_ids.tolist())) == k, "duplicate ids"
    assert got_ids.min() >= 0 and got_ids.max() < len(exact), "id out of range"
    assert np.all(np.diff(got_scores) <= 0), "scores not sorted descending"
    kth = np.partition(exact, len(exact) - k)[len(exact) - k]
    ex = exact[got_ids]
    assert np.all(ex >= kth - tie_abs), f"id below the k-th score: {ex.min()} < {kth}"
    must = np.nonzero(exact > kth + tie_abs)[0]
    missing = set(must.tolist()) - set(got_ids.tolist())
    assert not missing, f"missing top-k ids {sorted(missing)[:8]}"
    err = np.abs(got_scores - ex)
    assert np.all(err <= score_rel * np.abs(ex) + tie_abs), f"score error {err.max()}"
