"""GPU tests of the hierarchical main scan running beside the bounds kernel.

The scan reads each child's bound as the bounds kernel publishes it (tagged
with the search's epoch) and skips a child only when that bound is below the
running threshold; a child whose bound is not published yet is streamed.
These tests check exactness where that matters: a corpus large enough that the
bounds arrive while the scan streams (so it prunes mid-scan), the bounds of the
previous search left in the same workspace (queries alternating with their
negation, whose pruned children are each other's best), the external threshold
of the sharded path, and the trace's two row counts.  Parity rule:
oracle.check_topk against float64 brute force."""
import ctypes
import dataclasses

import numpy as np
import pytest
import torch

from circuit_rag import _native, build_circuit_index, circuit_search
from circuit_rag.synthetic import WORKLOADS
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _exact(X, q):
    return (X.double() @ q.double()).cpu().numpy()


def _check(X, q, k, s, i):
    oracle.check_topk(_exact(X, q), k, s.cpu().numpy(), i.cpu().numpy())


@pytest.fixture(scope="module")
def clustered_2m():
    # the clustered-50k law at 2,000,000 rows (1 GB): the bounds are ready after
    # a small part of it has streamed
    w = dataclasses.replace(WORKLOADS["clustered-50k"], name="clustered-2m", n=2_000_000)
    X = w.corpus(device=DEV)
    idx = build_circuit_index(X, num_roots=w.num_roots, children_per_root=w.children_per_root, rank=w.rank,
                              device=DEV)
    yield w, X, idx
    idx.close()


def test_prunes_while_streaming(clustered_2m):
    w, X, idx = clustered_2m
    streamed, pruned = [], []
    for q in w.query_batch(20, device=DEV):
        s, i, tr = circuit_search(q, idx, k=w.k)
        _check(X, q, w.k, s, i)
        assert tr.path == "hierarchical"
        assert 0 < tr.rows_streamed <= w.n
        streamed.append(tr.rows_streamed)
        pruned.append(tr.pruned_fraction)
    # (the hierarchy comes from a GPU k-means, so the fractions vary a little from build to build)
    assert np.mean(pruned) > 0.85, np.mean(pruned)
    assert np.mean(streamed) < 0.5 * w.n, np.mean(streamed)


@pytest.mark.parametrize("k", [1, 10, 100])
def test_bounds_of_the_previous_search_are_not_used(clustered_2m, k):
    """q, -q, q, -q on one workspace: the children pruned for one are the best
    for the other, so a bound of the previous search read as current would
    drop true results."""
    w, X, idx = clustered_2m
    for q in w.query_batch(4, device=DEV):
        for qq in (q, -q, q, -q):
            s, i, _ = circuit_search(qq, idx, k=k)
            _check(X, qq, k, s, i)


def test_blocking_calls_alternate_directions(clustered_2m):
    """The same through the C ABI's graph-replayed blocking call (host buffers)."""
    w, X, idx = clustered_2m
    L = _native.lib()
    h = idx.native_handle()
    k = 10
    for q in w.query_batch(3, device=DEV):
        for qq in (q, -q) * 3:
            qh = qq.cpu().numpy().copy()
            sh = np.zeros(k, np.float32)
            ih = np.zeros(k, np.int32)
            tr = _native.Trace()
            assert L.circuit_search(h, qh.ctypes.data, k, sh.ctypes.data, ih.ctypes.data, ctypes.byref(tr)) == 0
            oracle.check_topk(_exact(X, qq), k, sh, ih)


def test_external_threshold_prunes_and_stays_exact(clustered_2m):
    """seed -> T_ext just below the exact k-th best score (the tightest valid
    external threshold) -> finish: the top-k stays exact."""
    w, X, idx = clustered_2m
    L = _native.lib()
    h = idx.native_handle()
    st = torch.cuda.current_stream().cuda_stream
    k = w.k
    for q in w.query_batch(5, device=DEV):
        exact = _exact(X, q)
        s = torch.empty(k, device=DEV)
        i = torch.empty(k, dtype=torch.int32, device=DEV)
        T = torch.empty(1, device=DEV)
        assert L.circuit_search_seed_async(h, q.data_ptr(), k, T.data_ptr(), st) == 0
        Tx = torch.tensor([float(np.sort(exact)[-k]) - 1e-4], device=DEV)
        assert L.circuit_search_finish_async(h, q.data_ptr(), k, Tx.data_ptr(), s.data_ptr(), i.data_ptr(), None,
                                             st, None, None) == 0
        tx = _native.TraceEx()
        assert L.circuit_last_trace(h, ctypes.byref(tx)) == 0 and tx.device_error == 0
        _check(X, q, k, s, i)
        assert tx.vectors_scored <= w.n and 0 < tx.rows_streamed <= w.n


def test_trace_counts_small_corpus():
    """clustered-50k: the bounds prune > 90 % of the rows (vectors_scored), while
    the scan, which streams beside them, reads between the survivors' rows and
    all N (rows_streamed); the flat path reads N."""
    w = WORKLOADS["clustered-50k"]
    X = w.corpus(device=DEV)
    idx = build_circuit_index(X, num_roots=w.num_roots, children_per_root=w.children_per_root, rank=w.rank,
                              device=DEV)
    for q in w.query_batch(10, device=DEV):
        s, i, tr = circuit_search(q, idx, k=w.k)
        _check(X, q, w.k, s, i)
        assert tr.pruned_fraction > 0.9
        assert 0 < tr.rows_streamed <= w.n
        s2, i2, tr2 = circuit_search(q, idx, k=w.k, min_hierarchy_n=10 ** 9)
        assert tr2.path == "flat" and tr2.rows_streamed == w.n
        assert torch.equal(i, i2)
    idx.close()


@pytest.mark.parametrize("law,n,roots,cpr", [
    ("clustered-50k", 200, 1, 4),       # fewer rows than one chunk, one root
    ("clustered-50k", 20_000, 400, 2),  # many roots of ~50 rows: most chunks span several roots
    ("clustered-50k", 60_000, 16, 64),  # small children, chunks inside roots
    ("spread-200k", 200_000, 1, 64),    # one root holding ~1,500 live chunks (more than one CTA stages)
])
def test_chunk_and_list_shapes(law, n, roots, cpr):
    """Index shapes that exercise the claim/list edge cases: a single chunk, a single
    root, chunks shared by several roots, a CTA listing more chunks than it stages in
    shared memory; k = 1, 10, 256; the pipelined search and the one that starts the
    scan after the bounds (scan events) must both be exact and agree."""
    w = dataclasses.replace(WORKLOADS[law], name="shape", n=n)
    X = w.corpus(device=DEV)
    idx = build_circuit_index(X, num_roots=roots, children_per_root=cpr, rank=8, device=DEV)
    L = _native.lib()
    h = idx.native_handle()
    st = torch.cuda.current_stream().cuda_stream
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for e in (ev0, ev1):
        e.record()
    for q in w.query_batch(4, device=DEV):
        for k in (1, 10, 256):
            kk = min(k, n)
            s, i, tr = circuit_search(q, idx, k=kk, min_hierarchy_n=0)
            assert tr.path == "hierarchical"
            _check(X, q, kk, s, i)
            s2 = torch.empty(kk, device=DEV)
            i2 = torch.empty(kk, dtype=torch.int32, device=DEV)
            assert L.circuit_search_async(h, q.data_ptr(), kk, 0, s2.data_ptr(), i2.data_ptr(), None, st,
                                          ev0.cuda_event, ev1.cuda_event) == 0
            _check(X, q, kk, s2, i2)
            assert torch.equal(i, i2) and torch.equal(s, s2)
            tx = _native.TraceEx()
            assert L.circuit_last_trace(h, ctypes.byref(tx)) == 0
            assert tx.device_error == 0  # (a list or range bounds check would set a bit)
    idx.close()
