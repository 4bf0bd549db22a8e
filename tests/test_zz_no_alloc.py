"""circuit_flat_search_noalloc: the entry point for callers that cannot
allocate device memory (engine plugins whose framework owns all device memory,
serving loops that must not touch the allocator).  Its scratch is a fixed array
inside the library, so this test calls it through the C ABI twice in a row and
checks each result against the existing flat search entry point
(circuit_search_async over a handle with its own workspace) and against the
oracle.  Collected last so that a stop-at-first-failure run has already run
everything else; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

from circuit_rag import CircuitIndex
from circuit_rag import _native
from circuit_rag.synthetic import WORKLOADS
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _one_child_index(X: torch.Tensor) -> CircuitIndex:
    """An index whose single child holds every row (original id = row), so the
    existing entry point's flat scan covers exactly the same corpus."""
    n, d = X.shape
    bases = torch.zeros(1, d, 1)
    bases[0, 0, 0] = 1.0
    return CircuitIndex(root_centers=torch.zeros(1, d), root_radii=torch.full((1,), 1e9), bases=bases,
                        child_intervals_l=torch.full((1, 1), -1e9), child_intervals_u=torch.full((1, 1), 1e9),
                        child_radii=torch.full((1,), 1e9), child_parent_ids=torch.zeros(1, dtype=torch.int32),
                        leaf_offsets=torch.zeros(1, dtype=torch.int32),
                        leaf_sizes=torch.full((1,), n, dtype=torch.int32), leaf_vectors=X,
                        original_ids=torch.arange(n, dtype=torch.int32), dim=d, rank=1, device=DEV)


def _noalloc(L, X, q, k, stream):
    s = torch.empty(k, device=DEV)
    i = torch.empty(k, dtype=torch.int32, device=DEV)
    rc = L.circuit_flat_search_noalloc(X.data_ptr(), X.shape[0], X.shape[1], q.data_ptr(), k, s.data_ptr(),
                                       i.data_ptr(), stream.cuda_stream)
    assert rc == 0, _native.last_error()
    return s, i


@pytest.mark.parametrize("k", [10, 128])
def test_noalloc_matches_existing_entry_point_twice(k):
    L = _native.lib()
    w = WORKLOADS["spread-200k"]
    X = w.corpus(0, 60000, device=DEV)
    Q = w.query_batch(2, device=DEV)
    idx = _one_child_index(X)
    h = idx.native_handle()
    stream = torch.cuda.current_stream()
    for q in Q:  # two calls in a row; the second reuses the scratch the first left behind
        s_new, i_new = _noalloc(L, X, q, k, stream)
        s_ref = torch.empty(k, device=DEV)
        i_ref = torch.empty(k, dtype=torch.int32, device=DEV)
        rc = L.circuit_search_async(h, q.data_ptr(), k, 1 << 62, s_ref.data_ptr(), i_ref.data_ptr(), None,
                                    stream.cuda_stream, None, None)
        assert rc == 0, _native.last_error()
        torch.cuda.synchronize()
        exact = (X.double() @ q.double()).cpu().numpy()
        oracle.check_topk(exact, k, s_new.cpu().numpy(), i_new.cpu().numpy())
        oracle.check_topk(exact, k, s_ref.cpu().numpy(), i_ref.cpu().numpy())
        np.testing.assert_allclose(s_new.cpu().numpy(), s_ref.cpu().numpy(), rtol=oracle.SCORE_REL,
                                   atol=oracle.TIE_ABS)
        kth = np.sort(exact)[-k]
        differ = set(i_new.tolist()) ^ set(i_ref.tolist())
        assert all(abs(exact[j] - kth) <= oracle.TIE_ABS for j in differ)
    idx.close()


def test_noalloc_rejects_sizes_beyond_its_limit():
    L = _native.lib()
    X = torch.zeros(64, 32, device=DEV)
    q = torch.zeros(32, device=DEV)
    s = torch.empty(256, device=DEV)
    i = torch.empty(256, dtype=torch.int32, device=DEV)
    assert L.circuit_flat_search_noalloc(X.data_ptr(), 64, 32, q.data_ptr(), 129, s.data_ptr(), i.data_ptr(),
                                         None) == -2
    assert "128" in _native.last_error()
    assert L.circuit_flat_search_noalloc(X.data_ptr(), 64, 30, q.data_ptr(), 5, s.data_ptr(), i.data_ptr(),
                                         None) != 0


@pytest.mark.parametrize("n,k", [(1, 10), (5, 10), (100, 10), (148, 128), (3000, 128)])
def test_noalloc_small_corpora_match_existing_entry_point(n, k):
    """Fewer rows than k (the slots past n hold -inf / -1, as for every entry
    point) and fewer rows than SMs: two calls in a row, each equal to the
    existing entry point's result and to the oracle."""
    L = _native.lib()
    w = WORKLOADS["spread-5k"]
    X = w.corpus(0, n, device=DEV)
    Q = w.query_batch(2, device=DEV)
    idx = _one_child_index(X)
    h = idx.native_handle()
    stream = torch.cuda.current_stream()
    for q in Q:
        s_new, i_new = _noalloc(L, X, q, k, stream)
        s_ref = torch.empty(k, device=DEV)
        i_ref = torch.empty(k, dtype=torch.int32, device=DEV)
        assert L.circuit_search_async(h, q.data_ptr(), k, 1 << 62, s_ref.data_ptr(), i_ref.data_ptr(), None,
                                      stream.cuda_stream, None, None) == 0, _native.last_error()
        torch.cuda.synchronize()
        m = min(n, k)
        exact = (X.double() @ q.double()).cpu().numpy()
        oracle.check_topk(exact, m, s_new[:m].cpu().numpy(), i_new[:m].cpu().numpy())
        assert torch.equal(s_new, s_ref) and torch.equal(i_new, i_ref)
        if n < k:
            assert torch.all(torch.isneginf(s_new[n:])) and torch.all(i_new[n:] == -1)
    idx.close()


def test_noalloc_long_stream_matches_existing_entry_point():
    """2,000,000 rows: long enough for the scan to hand out chunks from the
    counter kept in the fixed scratch (cleared by each call); two calls in a
    row equal the existing entry point's results."""
    L = _native.lib()
    w = WORKLOADS["mixed-100m"]
    X = w.corpus(0, 2_000_000, device=DEV)
    Q = w.query_batch(2, device=DEV)
    idx = _one_child_index(X)
    h = idx.native_handle()
    stream = torch.cuda.current_stream()
    for q in Q:
        s_new, i_new = _noalloc(L, X, q, 10, stream)
        s_ref = torch.empty(10, device=DEV)
        i_ref = torch.empty(10, dtype=torch.int32, device=DEV)
        assert L.circuit_search_async(h, q.data_ptr(), 10, 1 << 62, s_ref.data_ptr(), i_ref.data_ptr(), None,
                                      stream.cuda_stream, None, None) == 0, _native.last_error()
        torch.cuda.synchronize()
        exact = (X.double() @ q.double()).cpu().numpy()
        oracle.check_topk(exact, 10, s_new.cpu().numpy(), i_new.cpu().numpy())
        assert torch.equal(s_new, s_ref) and torch.equal(i_new, i_ref)
    idx.close()
