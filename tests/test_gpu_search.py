"""GPU parity of the fused search (circuit_search / C ABI) against the oracle.

Parity rule (oracle.check_topk): ids identical to brute force except among
scores tied within 1e-6 absolute; scores within 1e-5 relative of the exact
(float64) score of the same id."""
import ctypes
import os

import numpy as np
import pytest
import torch

from circuit_rag import CircuitIndex, build_circuit_index, circuit_search
from circuit_rag import _native
from circuit_rag.synthetic import WORKLOADS
from oracle import oracle

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = "cuda"


def _exact(X: torch.Tensor, q: torch.Tensor) -> np.ndarray:
    return (X.double() @ q.double()).cpu().numpy()


def _check(X, q, k, scores, ids):
    oracle.check_topk(_exact(X, q), k, scores.cpu().numpy(), ids.cpu().numpy())


@pytest.fixture(scope="module")
def torch_fp32():
    torch.backends.cuda.matmul.allow_tf32 = False
    return True


@pytest.mark.parametrize("fixture,circuit,ks", [
    ("ref_small_search.npz", "ref_small.circuit", (1, 5, 10)),
    ("ref_d384_search.npz", "ref_d384.circuit", (10,)),
])
@pytest.mark.parametrize("min_hier", [0, 10 ** 9])
def test_reference_built_indexes(fixture, circuit, ks, min_hier):
    g = np.load(os.path.join(GOLDEN, fixture))
    idx = CircuitIndex.load(os.path.join(GOLDEN, circuit), device=DEV)
    X = torch.empty_like(idx.leaf_vectors)
    X[idx.original_ids.long()] = idx.leaf_vectors
    for k in ks:
        for qi, qn in enumerate(g["queries"]):
            q = torch.from_numpy(qn).to(DEV)
            s, i, tr = circuit_search(q, idx, k=k, min_hierarchy_n=min_hier)
            _check(X, q, k, s, i)
            ref_ids = set(g[f"ids_k{k}"][qi].tolist())
            exact = _exact(X, q)
            kth = np.sort(exact)[-k]
            differ = set(i.tolist()) ^ ref_ids
            assert all(abs(exact[j] - kth) <= 1e-6 for j in differ)
            assert tr.path == ("hierarchical" if min_hier == 0 else "flat")


def test_reference_exactness_test_verbatim(torch_fp32):
    """tests/test_exact.py of the reference, on the GPU path."""
    rng = np.random.default_rng(0)
    centers = rng.normal(size=(64, 128))
    X = centers[rng.integers(0, 64, 40000)] + 0.3 * rng.normal(size=(40000, 128))
    X = (X / np.linalg.norm(X, axis=1, keepdims=True)).astype(np.float32)
    idx = build_circuit_index(X, num_roots=32, children_per_root=8, rank=8, device=DEV)
    corpus = torch.from_numpy(X).to(idx.device)
    rng = np.random.default_rng(1)
    for qi in rng.integers(0, len(X), 25):
        q = corpus[qi]
        scores, ids, tr = circuit_search(q, idx, k=10)
        truth = torch.topk(corpus @ q, 10)
        assert set(ids.tolist()) == set(truth.indices.tolist())
        assert torch.allclose(scores.sort(descending=True).values, truth.values, atol=1e-4)
        assert tr.path == "hierarchical"


@pytest.mark.parametrize("name,nq,min_hier", [
    ("clustered-50k", 25, 10000),
    ("spread-5k", 60, 10 ** 9),
    ("spread-5k", 60, 0),
    ("spread-200k", 30, 10000),
])
def test_workloads_exact(name, nq, min_hier):
    w = WORKLOADS[name]
    X = w.corpus(device=DEV)
    idx = build_circuit_index(X, num_roots=w.num_roots, children_per_root=w.children_per_root, rank=w.rank,
                              device=DEV)
    Q = w.query_batch(nq, device=DEV)
    pruned = []
    for q in Q:
        s, i, tr = circuit_search(q, idx, k=w.k, min_hierarchy_n=min_hier)
        _check(X, q, w.k, s, i)
        pruned.append(tr.pruned_fraction)
    if name == "clustered-50k":
        assert np.mean(pruned) > 0.9, np.mean(pruned)


@pytest.mark.parametrize("k", [1, 2, 31, 32, 33, 100, 128, 129, 256])
def test_k_range(k):
    w = WORKLOADS["clustered-50k"]
    X = w.corpus(0, 20000, device=DEV)
    idx = build_circuit_index(X, num_roots=32, children_per_root=8, rank=8, device=DEV)
    for q in w.query_batch(4, device=DEV):
        for mh in (0, 10 ** 9):
            s, i, _ = circuit_search(q, idx, k=k, min_hierarchy_n=mh)
            _check(X, q, k, s, i)


def test_k_limits_and_small_corpus():
    X = WORKLOADS["clustered-50k"].corpus(0, 200, device=DEV)
    idx = build_circuit_index(X, num_roots=4, children_per_root=4, rank=4, device=DEV)
    for mh in (0, 10 ** 9):
        # k clamps to N (reference search.py:51)
        s, i, _ = circuit_search(X[3], idx, k=1000, min_hierarchy_n=mh)
        assert len(i) == 200
        _check(X, X[3], 200, s, i)
        s, i, _ = circuit_search(X[5], idx, k=40, min_hierarchy_n=mh)
        _check(X, X[5], 40, s, i)
    big = WORKLOADS["clustered-50k"].corpus(0, 2000, device=DEV)
    idx2 = build_circuit_index(big, num_roots=4, children_per_root=4, rank=4, device=DEV)
    with pytest.raises(ValueError):
        circuit_search(big[0], idx2, k=257)
    with pytest.raises(ValueError):
        circuit_search(big[0], idx2, k=0)


def test_duplicates_and_exact_ties():
    base = WORKLOADS["spread-5k"].corpus(0, 500, device=DEV)
    X = torch.cat([base, base[:50], base[:50]])  # every one of the first 50 rows appears 3 times
    idx = build_circuit_index(X, num_roots=8, children_per_root=4, rank=4, device=DEV)
    for q in (X[7], X[499]):
        for mh in (0, 10 ** 9):
            s, i, _ = circuit_search(q, idx, k=10, min_hierarchy_n=mh)
            _check(X, q, 10, s, i)


@pytest.mark.parametrize("dim,rank", [(4, 1), (64, 3), (132, 33), (640, 64), (1024, 16), (2048, 8)])
def test_dims_and_ranks(dim, rank):
    g = torch.Generator(device=DEV)
    g.manual_seed(dim * 31 + rank)
    X = torch.randn(3000, dim, generator=g, device=DEV)
    X = X / X.norm(dim=1, keepdim=True)
    idx = build_circuit_index(X, num_roots=8, children_per_root=4, rank=min(rank, dim), device=DEV)
    for qi in (0, 1234, 2999):
        for mh in (0, 10 ** 9):
            s, i, _ = circuit_search(X[qi], idx, k=10, min_hierarchy_n=mh)
            _check(X, X[qi], 10, s, i)


def test_trace_fields():
    w = WORKLOADS["clustered-50k"]
    X = w.corpus(device=DEV)
    idx = build_circuit_index(X, num_roots=64, children_per_root=16, rank=8, device=DEV)
    q = w.query_batch(1, device=DEV)[0]
    s, i, tr = circuit_search(q, idx, k=10)
    assert tr.path == "hierarchical" and tr.corpus_size == 50000 and tr.total_children == 1024
    assert 0 < tr.vectors_scored < 50000
    assert 0 < tr.surviving_children <= 1024
    assert tr.seed_threshold > -1e9 and tr.seed_threshold <= float(s[-1]) + 1e-6
    assert tr.total_gpu_time_us > 0
    s2, i2, tr2 = circuit_search(q, idx, k=10, min_hierarchy_n=10 ** 9)
    assert tr2.path == "flat" and tr2.vectors_scored == 50000
    assert torch.equal(i, i2)


def test_c_abi_host_and_device_search(tmp_path):
    w = WORKLOADS["spread-200k"]
    X = w.corpus(0, 30000, device=DEV)
    idx = build_circuit_index(X, num_roots=32, children_per_root=8, rank=8, device=DEV)
    path = str(tmp_path / "i.circuit")
    idx.save(path)
    L = _native.lib()
    h = L.circuit_load_index(path.encode(), torch.cuda.current_device())
    assert h, _native.last_error()
    try:
        info = (ctypes.c_int64 * 8)()
        assert L.circuit_index_info(h, info) == 0 and info[4] == 30000
        Q = w.query_batch(6, device=DEV)
        for k in (10, 64):
            for q in Q:
                qh = q.cpu().numpy().copy()
                sh = np.zeros(k, np.float32)
                ih = np.zeros(k, np.int32)
                tr = _native.Trace()
                rc = L.circuit_search(h, qh.ctypes.data, k, sh.ctypes.data, ih.ctypes.data, ctypes.byref(tr))
                assert rc == 0, _native.last_error()
                oracle.check_topk(_exact(X, q), k, sh, ih)
                assert 0 < tr.vectors_scored <= 30000
                sd = torch.empty(k, device=DEV)
                idd = torch.empty(k, dtype=torch.int32, device=DEV)
                rc = L.circuit_search_device(h, q.contiguous().data_ptr(), k, sd.data_ptr(), idd.data_ptr(), None)
                assert rc == 0, _native.last_error()
                assert np.array_equal(idd.cpu().numpy(), ih) and np.array_equal(sd.cpu().numpy(), sh)
        tx = _native.TraceEx()
        assert L.circuit_last_trace(h, ctypes.byref(tx)) == 0 and tx.device_error == 0
        assert L.circuit_search(h, Q[0].cpu().numpy().ctypes.data, 0, sh.ctypes.data, ih.ctypes.data, None) == -2
    finally:
        L.circuit_destroy_index(h)


def test_blocking_search_graph_replay_paths(tmp_path):
    """Blocking calls replay a graph from the second call per (k, path, buffer kind):
    the query comes from mapped host memory or the caller's device pointer, and the
    final merge writes results and the control header directly.  Flat and
    hierarchical indexes, k = 10 and 256, device outputs that move between calls, and
    a query pointer that is not 16-byte aligned (direct path) all agree with the
    oracle and with each other, traces included."""
    w = WORKLOADS["spread-200k"]
    L = _native.lib()
    for n, flat in ((6000, True), (30000, False)):
        X = w.corpus(0, n, device=DEV)
        idx = build_circuit_index(X, num_roots=32, children_per_root=8, rank=8, device=DEV)
        path = str(tmp_path / f"g{n}.circuit")
        idx.save(path)
        h = L.circuit_load_index(path.encode(), torch.cuda.current_device())
        assert h, _native.last_error()
        try:
            Q = w.query_batch(5, device=DEV)
            qbuf = torch.empty(Q.shape[1] + 1, device=DEV)
            for k in (10, 256):
                out_s = torch.full((len(Q) * k,), float("nan"), device=DEV)
                out_i = torch.full((len(Q) * k,), -7, dtype=torch.int32, device=DEV)
                for j, q in enumerate(Q):
                    qh = q.cpu().numpy().copy()
                    sh = np.zeros(k, np.float32)
                    ih = np.zeros(k, np.int32)
                    tr = _native.Trace()
                    rc = L.circuit_search(h, qh.ctypes.data, k, sh.ctypes.data, ih.ctypes.data, ctypes.byref(tr))
                    assert rc == 0, _native.last_error()
                    oracle.check_topk(_exact(X, q), k, sh, ih)
                    if flat:
                        assert tr.vectors_scored == n
                    else:
                        assert 0 < tr.vectors_scored <= n
                    sd, idd = out_s[j * k:(j + 1) * k], out_i[j * k:(j + 1) * k]
                    tr2 = _native.Trace()
                    rc = L.circuit_search_device(h, q.contiguous().data_ptr(), k, sd.data_ptr(), idd.data_ptr(),
                                                 ctypes.byref(tr2))
                    assert rc == 0, _native.last_error()
                    assert np.array_equal(sd.cpu().numpy(), sh) and np.array_equal(idd.cpu().numpy(), ih)
                    assert tr2.vectors_scored == tr.vectors_scored
                    qbuf[1:].copy_(q)
                    sd2 = torch.empty(k, device=DEV)
                    id2 = torch.empty(k, dtype=torch.int32, device=DEV)
                    rc = L.circuit_search_device(h, qbuf[1:].data_ptr(), k, sd2.data_ptr(), id2.data_ptr(), None)
                    assert rc == 0, _native.last_error()
                    assert np.array_equal(sd2.cpu().numpy(), sh) and np.array_equal(id2.cpu().numpy(), ih)
                # earlier outputs stay untouched by later calls
                for j, q in enumerate(Q):
                    oracle.check_topk(_exact(X, q), k, out_s[j * k:(j + 1) * k].cpu().numpy(),
                                      out_i[j * k:(j + 1) * k].cpu().numpy())
            tx = _native.TraceEx()
            assert L.circuit_last_trace(h, ctypes.byref(tx)) == 0
            assert tx.device_error == 0 and tx.path == (0 if flat else 1)
        finally:
            L.circuit_destroy_index(h)


def test_cuda_graph_replay_matches():
    w = WORKLOADS["clustered-50k"]
    X = w.corpus(device=DEV)
    idx = build_circuit_index(X, num_roots=64, children_per_root=16, rank=8, device=DEV)
    for q in w.query_batch(5, device=DEV):
        v1, i1 = idx.search_graph(q, k=10)
        s, i, _ = circuit_search(q, idx, k=10, min_hierarchy_n=10001)
        assert torch.equal(i1, i) and torch.equal(v1, s)


def test_bounded_wait_gives_up_and_context_stays_usable():
    """A device wait that nothing satisfies ends after its 2 s limit with an error
    bit the host reads (no trap, no hang); the next search runs normally."""
    L = _native.lib()
    bits = ctypes.c_int(-1)
    assert L.circuit_selftest_wait_timeout(0, ctypes.byref(bits)) == 0
    assert bits.value == 1
    w = WORKLOADS["clustered-50k"]
    X = w.corpus(0, 5000, device=DEV)
    idx = build_circuit_index(X, num_roots=8, children_per_root=4, rank=4, device=DEV)
    q = w.query_batch(1, device=DEV)[0]
    s, i, _ = circuit_search(q, idx, k=10)
    _check(X, q, 10, s, i)


def test_search_after_append_is_exact():
    """An index grown with CircuitIndex.append (rows far outside the old roots
    included) searches exactly, single and batched."""
    from circuit_rag import circuit_search_batch

    w = WORKLOADS["clustered-50k"]
    X1 = w.corpus(0, 20000, device=DEV)
    idx = build_circuit_index(X1, num_roots=16, children_per_root=8, rank=8, device=DEV)
    g = torch.Generator(device="cpu").manual_seed(3)
    X2 = w.corpus(20000, 26000, device=DEV)
    X3 = (torch.randn(500, X1.shape[1], generator=g) * 2.0).to(DEV)
    idx.append(X2)
    idx.append(X3)
    X = torch.cat([X1, X2, X3])
    Q = torch.cat([w.query_batch(6, device=DEV), X3[:4] * 1.01])
    for q in Q:
        s, i, tr = circuit_search(q, idx, k=10)
        _check(X, q, 10, s, i)
    bs, bi = circuit_search_batch(Q, idx, k=10)
    for b in range(Q.shape[0]):
        _check(X, Q[b], 10, bs[b], bi[b])


def test_circuit_bench_binary_runs(tmp_path):
    """The native bench (reference command line plus an optional batch size)
    loads a .circuit file, runs host, in-VRAM and batched queries, prints JSON."""
    import json
    import subprocess

    binary = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "circuit-rag_b200", "csrc",
                          "_build", "circuit_bench")
    if not os.path.exists(binary):
        pytest.skip("circuit_bench not built")
    w = WORKLOADS["spread-5k"]
    idx = build_circuit_index(w.corpus(0, 5183, device=DEV), num_roots=16, children_per_root=4, rank=8, device=DEV)
    path = str(tmp_path / "b.circuit")
    idx.save(path)
    out = subprocess.run([binary, path, "10", "50", "256"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    line = json.loads([x for x in out.stdout.splitlines() if x.startswith("{")][-1])
    assert line["N"] == 5183 and line["batch"] == 256 and line["batch_qps"] > 0 and line["host_qps"] > 0
