"""GPU parity of the batched tensor-core search (circuit_search_batch and the
C ABI circuit_search_batch_async / circuit_search_batch).

Each query of a batch must return exactly what circuit_search returns for it
(bit-identical fp32 scores: the exact rescoring uses the single-query scan's
arithmetic) and must pass the oracle's top-k rule against float64 brute force
(ids identical except among scores tied within 1e-6; scores within 1e-5
relative)."""
import ctypes

import numpy as np
import pytest
import torch

from circuit_rag import build_circuit_index, circuit_search, circuit_search_batch
from circuit_rag import _native
from circuit_rag.synthetic import WORKLOADS
from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _unit_rows(n, dim, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(n, dim, generator=g)
    return (x / x.norm(dim=1, keepdim=True)).to(DEV)


def _check_batch(X, Q, index, k, scores, ids, compare_single=True):
    exact = (Q.double() @ X.double().T).cpu().numpy()
    s_np, i_np = scores.cpu().numpy(), ids.cpu().numpy()
    for b in range(Q.shape[0]):
        oracle.check_topk(exact[b], k, s_np[b], i_np[b])
        if compare_single:
            s1, i1, _ = circuit_search(Q[b], index, k)
            assert torch.equal(scores[b], s1), (b, scores[b], s1)
            assert torch.equal(ids[b], i1), (b, ids[b], i1)


def test_batch_many_ties_within_capacity():
    """20,000 identical rows: every one is inside the band; the rescore takes
    them in rounds of 8,192 with a running top-k, no fallback."""
    base = _unit_rows(1, 64, 41)
    X = torch.cat([base.repeat(20000, 1), _unit_rows(700, 64, 42)])
    index = build_circuit_index(X, num_roots=4, children_per_root=2, rank=2, device=DEV)
    Q = torch.cat([base, _unit_rows(5, 64, 43)])
    scores, ids = circuit_search_batch(Q, index, 10)
    n_over = ctypes.c_int(-1)
    assert _native.lib().circuit_batch_overflow(index.native_handle(), ctypes.byref(n_over)) == 0
    assert n_over.value == 0
    _check_batch(X, Q, index, 10, scores, ids, compare_single=False)


@pytest.mark.parametrize("name,n,dim", [
    ("mixed-100m", 30_000, 384),
    ("clustered-50k", 20_011, 128),
    (None, 9_000, 100),
    (None, 6_000, 1028),
    (None, 3_000, 2048),
])
@pytest.mark.parametrize("k", [1, 10, 32])
def test_batch_matches_single_query_and_oracle(name, n, dim, k):
    if name is None:
        X = _unit_rows(n, dim, 5)
        Q = _unit_rows(131, dim, 6)
    else:
        w = WORKLOADS[name]
        X = w.corpus(0, n, device=DEV)
        Q = w.query_batch(131, device=DEV)
    index = build_circuit_index(X, num_roots=16, children_per_root=4, rank=8, device=DEV)
    scores, ids = circuit_search_batch(Q, index, k)
    assert scores.shape == (131, k) and ids.shape == (131, k)
    _check_batch(X, Q, index, k, scores, ids, compare_single=(k == 10 or name is None))


def test_batch_ragged_edges():
    """N smaller than one leaf tile, batch of one, k clamped to N."""
    X = _unit_rows(37, 64, 11)
    index = build_circuit_index(X, num_roots=2, children_per_root=2, rank=2, device=DEV)
    Q = _unit_rows(1, 64, 12)
    scores, ids = circuit_search_batch(Q, index, 32)
    _check_batch(X, Q, index, 32, scores, ids, compare_single=False)
    X2 = _unit_rows(20, 64, 13)
    index2 = build_circuit_index(X2, num_roots=2, children_per_root=2, rank=2, device=DEV)
    scores, ids = circuit_search_batch(Q, index2, 50)  # k > N -> N results
    assert ids.shape == (1, 20)
    assert sorted(ids[0].tolist()) == list(range(20))


def test_batch_overflow_falls_back_to_single_query():
    """70,000 identical rows all sit inside the error band of a query equal to
    them: its candidate list (at most 65,536 entries for a small batch)
    overflows, the async call marks it with id -2, and circuit_search_batch
    answers it with circuit_search."""
    base = _unit_rows(1, 64, 21)
    X = torch.cat([base.repeat(70000, 1), _unit_rows(500, 64, 22)])
    index = build_circuit_index(X, num_roots=4, children_per_root=2, rank=2, device=DEV)
    Q = torch.cat([base, _unit_rows(3, 64, 23)])
    handle = index.native_handle()
    s = torch.empty(4, 10, device=DEV)
    i = torch.empty(4, 10, dtype=torch.int32, device=DEV)
    rc = _native.lib().circuit_search_batch_async(handle, Q.data_ptr(), 4, 10, s.data_ptr(), i.data_ptr(),
                                                  torch.cuda.current_stream().cuda_stream, None, None)
    assert rc == 0
    n_over = ctypes.c_int(-1)
    assert _native.lib().circuit_batch_overflow(handle, ctypes.byref(n_over)) == 0
    assert n_over.value >= 1
    assert int(i[0, 0]) == -2
    scores, ids = circuit_search_batch(Q, index, 10)
    assert int(ids.min()) >= 0
    _check_batch(X, Q, index, 10, scores, ids, compare_single=False)
    # the blocking device-buffer call answers the overflowed row in place
    s2 = torch.full((4, 10), float("nan"), device=DEV)
    i2 = torch.full((4, 10), -7, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    rc = _native.lib().circuit_search_batch_device(handle, Q.data_ptr(), 4, 10, s2.data_ptr(), i2.data_ptr())
    assert rc == 0, _native.last_error()
    assert torch.equal(i2, ids) and torch.equal(s2, scores)


def test_batch_host_buffers_through_c_abi():
    w = WORKLOADS["spread-5k"]
    X = w.corpus(0, 5183, device=DEV)
    index = build_circuit_index(X, num_roots=8, children_per_root=4, rank=8, device=DEV)
    Qh = w.query_batch(200).contiguous()
    s = np.zeros((200, 10), np.float32)
    i = np.zeros((200, 10), np.int32)
    torch.cuda.synchronize()
    rc = _native.lib().circuit_search_batch(index.native_handle(), Qh.data_ptr(), 200, 10, s.ctypes.data,
                                            i.ctypes.data)
    assert rc == 0, _native.last_error()
    _check_batch(X, Qh.to(DEV), index, 10, torch.from_numpy(s).to(DEV), torch.from_numpy(i).to(DEV))
    Qd = Qh.to(DEV)
    sd = torch.empty(200, 10, device=DEV)
    idd = torch.empty(200, 10, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    rc = _native.lib().circuit_search_batch_device(index.native_handle(), Qd.data_ptr(), 200, 10, sd.data_ptr(),
                                                   idd.data_ptr())
    assert rc == 0, _native.last_error()
    assert np.array_equal(sd.cpu().numpy(), s) and np.array_equal(idd.cpu().numpy(), i)


def test_batch_rejects_unsupported():
    X = _unit_rows(500, 64, 31)
    index = build_circuit_index(X, num_roots=2, children_per_root=2, rank=2, device=DEV)
    Q = _unit_rows(4, 64, 32)
    with pytest.raises(ValueError):
        circuit_search_batch(Q, index, 257)
    with pytest.raises(ValueError):
        circuit_search_batch(Q[:, :32], index, 10)
    s = torch.empty(4, 257, device=DEV)
    i = torch.empty(4, 257, dtype=torch.int32, device=DEV)
    rc = _native.lib().circuit_search_batch_async(index.native_handle(), Q.data_ptr(), 4, 257, s.data_ptr(),
                                                  i.data_ptr(), None, None, None)
    assert rc == -7
    # a query pointer that is not 16-byte aligned is rejected before any launch
    rc = _native.lib().circuit_search_batch_async(index.native_handle(), Q.data_ptr() + 4, 2, 10, s.data_ptr(),
                                                  i.data_ptr(), None, None, None)
    assert rc == -2


@pytest.mark.parametrize("k", [64, 100, 128, 200])
def test_batch_large_k_host_buffers(k):
    """Host-buffer batched call at large k (all on the tensor cores); results
    identical to the single-query search."""
    w = WORKLOADS["zipf-10m"]
    X = w.corpus(0, 30_000, device=DEV)
    index = build_circuit_index(X, num_roots=32, children_per_root=8, rank=16, device=DEV)
    Qh = w.query_batch(20).contiguous()
    s = np.zeros((20, k), np.float32)
    i = np.zeros((20, k), np.int32)
    torch.cuda.synchronize()
    rc = _native.lib().circuit_search_batch(index.native_handle(), Qh.data_ptr(), 20, k, s.ctypes.data, i.ctypes.data)
    assert rc == 0, _native.last_error()
    _check_batch(X, Qh.to(DEV), index, k, torch.from_numpy(s).to(DEV), torch.from_numpy(i).to(DEV))


def test_batch_large_k_matches_single_query():
    """k = 100 (the zipf-10m configuration's k): same results as the single-query
    search."""
    w = WORKLOADS["zipf-10m"]
    X = w.corpus(0, 40_000, device=DEV)
    index = build_circuit_index(X, num_roots=32, children_per_root=8, rank=16, device=DEV)
    Q = w.query_batch(24, device=DEV)
    scores, ids = circuit_search_batch(Q, index, 100)
    assert scores.shape == (24, 100)
    _check_batch(X, Q, index, 100, scores, ids)


@pytest.mark.parametrize("k", [10, 50, 100])
def test_batch_threshold_pass_and_slots(k):
    """120K rows: the threshold pass over sampled rows runs (corpora of 65,536
    rows and more), k = 10 takes the per-thread top-k epilogue, k = 50 / 100 the
    slot thresholds; results equal the single-query search's."""
    w = WORKLOADS["mixed-100m"]
    X = w.corpus(0, 120_000, device=DEV)
    index = build_circuit_index(X, num_roots=32, children_per_root=8, rank=8, device=DEV)
    Q = w.query_batch(300, device=DEV)
    scores, ids = circuit_search_batch(Q, index, k)
    _check_batch(X, Q[:60], index, k, scores[:60], ids[:60])


@pytest.mark.parametrize("k", [33, 100, 256])
def test_batch_slot_thresholds_full_batch(k):
    """1,024 queries at k > 32 on 300K rows: every CTA's threshold warp refreshes
    several queries per sweep (the k-th largest of 4k row-keyed slots), the
    threshold pass is cut into 2,048-row slices; the first, middle and last
    queries of the batch equal the single-query search's results and pass the
    oracle's rule."""
    w = WORKLOADS["zipf-10m"]
    X = w.corpus(0, 300_000, device=DEV)
    index = build_circuit_index(X, num_roots=32, children_per_root=8, rank=16, device=DEV)
    Q = w.query_batch(1024, device=DEV)
    scores, ids = circuit_search_batch(Q, index, k)
    pick = torch.tensor(list(range(0, 16)) + list(range(500, 516)) + list(range(1008, 1024)), device=DEV)
    _check_batch(X, Q[pick], index, k, scores[pick], ids[pick])
