"""GPU tests of C-ABI edge behaviour: k above the row count (every call pads the
slots past N with score -inf and id -1), the batched path's device-error
reporting (a bounded wait that gave up is reported and cleared), and one
process searching on two GPUs (per-device kernel configuration)."""
import ctypes
import math

import numpy as np
import pytest
import torch

from circuit_rag import build_circuit_index, circuit_search_batch
from circuit_rag import _native
from circuit_rag.synthetic import WORKLOADS
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
ERR_TIMEOUT = -4


def _exact(X, q):
    return (X.double() @ q.double()).cpu().numpy()


def _check_padded(X, q, k, scores, ids):
    """All N rows first (oracle rule), then k - N empty slots."""
    n = X.shape[0]
    scores, ids = np.asarray(scores), np.asarray(ids)
    oracle.check_topk(_exact(X, q), n, scores[:n], ids[:n])
    assert sorted(ids[:n].tolist()) == list(range(n))
    assert np.all(np.isneginf(scores[n:])), scores
    assert np.all(ids[n:] == -1), ids


@pytest.mark.parametrize("n", [1, 7, 40])
def test_k_above_row_count_every_entry_point(tmp_path, n):
    L = _native.lib()
    w = WORKLOADS["spread-5k"]
    X = w.corpus(0, n, device=DEV)
    idx = build_circuit_index(X, num_roots=1, children_per_root=2, rank=2, device=DEV)
    h = idx.native_handle()
    k = 50
    q = w.query_batch(1, device=DEV)[0]
    # blocking host buffers (graph replay from the second call) and device buffers
    for _ in range(3):
        hs = np.zeros(k, np.float32)
        hi = np.zeros(k, np.int32)
        assert L.circuit_search(h, np.ascontiguousarray(q.cpu().numpy()).ctypes.data, k, hs.ctypes.data,
                                hi.ctypes.data, None) == 0, _native.last_error()
        _check_padded(X, q, k, hs, hi)
        ds = torch.empty(k, device=DEV)
        di = torch.empty(k, dtype=torch.int32, device=DEV)
        assert L.circuit_search_device(h, q.data_ptr(), k, ds.data_ptr(), di.data_ptr(), None) == 0
        _check_padded(X, q, k, ds.cpu().numpy(), di.cpu().numpy())
    # asynchronous, both routes
    st = torch.cuda.current_stream()
    for mh in (0, 1 << 62):
        ds = torch.full((k,), 7.0, device=DEV)
        di = torch.full((k,), 7, dtype=torch.int32, device=DEV)
        assert L.circuit_search_async(h, q.data_ptr(), k, mh, ds.data_ptr(), di.data_ptr(), None, st.cuda_stream,
                                      None, None) == 0
        torch.cuda.synchronize()
        _check_padded(X, q, k, ds.cpu().numpy(), di.cpu().numpy())
    # a file loaded by the native loader
    path = str(tmp_path / "tiny.circuit")
    idx.save(path)
    fh = L.circuit_load_index(path.encode(), 0)
    assert fh, _native.last_error()
    hs = np.zeros(k, np.float32)
    hi = np.zeros(k, np.int32)
    assert L.circuit_search(fh, np.ascontiguousarray(q.cpu().numpy()).ctypes.data, k, hs.ctypes.data,
                            hi.ctypes.data, None) == 0
    _check_padded(X, q, k, hs, hi)
    L.circuit_destroy_index(fh)
    # batched: host buffers and device buffers
    Q = w.query_batch(3, device=DEV)
    hq = np.ascontiguousarray(Q.cpu().numpy())
    bs = np.zeros((3, k), np.float32)
    bi = np.zeros((3, k), np.int32)
    assert L.circuit_search_batch(h, hq.ctypes.data, 3, k, bs.ctypes.data, bi.ctypes.data) == 0
    for b in range(3):
        _check_padded(X, Q[b], k, bs[b], bi[b])
    ds = torch.empty(3, k, device=DEV)
    di = torch.empty(3, k, dtype=torch.int32, device=DEV)
    assert L.circuit_search_batch_device(h, Q.data_ptr(), 3, k, ds.data_ptr(), di.data_ptr()) == 0
    for b in range(3):
        _check_padded(X, Q[b], k, ds[b].cpu().numpy(), di[b].cpu().numpy())
    # the Python API shortens the result to N instead (reference circuit_rag/search.py:51)
    s, i = circuit_search_batch(Q, idx, k)
    assert s.shape == (3, n)
    idx.close()


def test_batch_timeout_is_reported_and_then_cleared():
    """A batched-scan wait that gave up leaves error bits in the batch workspace:
    the status call reports CIRCUIT_ERR_TIMEOUT, and the next batch starts with
    the bits cleared and returns exact results."""
    L = _native.lib()
    w = WORKLOADS["clustered-50k"]
    X = w.corpus(0, 6000, device=DEV)
    idx = build_circuit_index(X, num_roots=8, children_per_root=4, rank=4, device=DEV)
    h = idx.native_handle()
    Q = w.query_batch(16, device=DEV)
    k = 10
    s = torch.empty(16, k, device=DEV)
    i = torch.empty(16, k, dtype=torch.int32, device=DEV)
    assert L.circuit_search_batch_device(h, Q.data_ptr(), 16, k, s.data_ptr(), i.data_ptr()) == 0
    bits = ctypes.c_int(0)
    assert L.circuit_selftest_batch_wait_timeout(h, ctypes.byref(bits)) == 0
    assert bits.value == 1
    over = ctypes.c_int(-1)
    assert L.circuit_batch_overflow(h, ctypes.byref(over)) == ERR_TIMEOUT
    assert "timed out" in _native.last_error()
    # the next batch clears the bits and is exact again
    assert L.circuit_search_batch_device(h, Q.data_ptr(), 16, k, s.data_ptr(), i.data_ptr()) == 0
    assert L.circuit_batch_overflow(h, ctypes.byref(over)) == 0 and over.value == 0
    exact = (Q.double() @ X.double().T).cpu().numpy()
    for b in range(16):
        oracle.check_topk(exact[b], k, s[b].cpu().numpy(), i[b].cpu().numpy())
    # the blocking host-buffer call reports the same error after an injected timeout
    assert L.circuit_selftest_batch_wait_timeout(h, ctypes.byref(bits)) == 0
    hq = np.ascontiguousarray(Q.cpu().numpy())
    hs = np.zeros((16, k), np.float32)
    hi = np.zeros((16, k), np.int32)
    assert L.circuit_search_batch(h, hq.ctypes.data, 16, k, hs.ctypes.data, hi.ctypes.data) == 0  # cleared first
    idx.close()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_searches_on_two_devices_in_one_process():
    """Kernels that opt into more than 48 KB of shared memory are configured on
    each device before their first launch there."""
    w = WORKLOADS["spread-200k"]
    for dev in ("cuda:0", "cuda:1", "cuda:0"):
        X = w.corpus(0, 30000, device=dev)
        idx = build_circuit_index(X, num_roots=16, children_per_root=8, rank=8, device=dev)
        Q = w.query_batch(4, device=dev)
        from circuit_rag import circuit_search

        with torch.cuda.device(torch.device(dev)):
            for q in Q:
                s1, i1, _ = circuit_search(q, idx, 10)
                oracle.check_topk(_exact(X, q), 10, s1.cpu().numpy(), i1.cpu().numpy())
            s, i = circuit_search_batch(Q, idx, 10)
            exact = (Q.double() @ X.double().T).cpu().numpy()
            for b in range(4):
                oracle.check_topk(exact[b], 10, s[b].cpu().numpy(), i[b].cpu().numpy())
        idx.close()
