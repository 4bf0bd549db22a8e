"""GPU side of the sharded search: the device merge kernel and shards loaded
from one .circuit file, searched one by one and merged, against brute force."""
import os

import numpy as np
import pytest
import torch

from circuit_rag import build_circuit_index, circuit_search, circuit_search_batch
from circuit_rag.shard import load_shard, merge_topk, merge_topk_batch, merge_topk_batch_host, merge_topk_host
from circuit_rag.synthetic import WORKLOADS
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("world,k", [(2, 10), (8, 10), (8, 100), (3, 256)])
def test_merge_kernel_matches_host_merge(world, k):
    g = torch.Generator().manual_seed(world * 1000 + k)
    s = torch.randn(world * k, generator=g)
    s[::7] = s[3]  # exact ties, broken by the smaller id
    ids = torch.randperm(10 ** 6, generator=g)[:world * k].int()
    ids[-3:] = -1  # empty slots
    hs, hi = merge_topk_host(s, ids, k)
    ds, di = merge_topk(s.to(DEV), ids.to(DEV), k)
    assert torch.equal(di.cpu(), hi)
    assert torch.equal(ds.cpu(), hs)


@pytest.mark.parametrize("world", [2, 3, 5])
def test_shards_merge_to_brute_force(tmp_path, world):
    w = WORKLOADS["zipf-10m"]
    X = w.corpus(0, 30000, device=DEV)
    idx = build_circuit_index(X, num_roots=24, children_per_root=8, rank=8, device=DEV)
    path = str(tmp_path / "z.circuit")
    idx.save(path)
    shards = [load_shard(path, r, world, device=DEV) for r in range(world)]
    assert sum(s.N for s in shards) == 30000
    for q in w.query_batch(4, device=DEV):
        for k in (10, 100):
            S, I = [], []
            for sh in shards:
                s, i, _ = circuit_search(q, sh, k=k, min_hierarchy_n=0)
                S.append(torch.cat([s, s.new_full((k - len(s),), float("-inf"))]))
                I.append(torch.cat([i, i.new_full((k - len(i),), -1)]))
            ms, mi = merge_topk(torch.cat(S), torch.cat(I), k)
            oracle.check_topk((X.double() @ q.double()).cpu().numpy(), k, ms.cpu().numpy(), mi.cpu().numpy())


@pytest.mark.parametrize("world,k_in,k", [(1, 10, 10), (3, 10, 10), (8, 32, 20)])
def test_batched_merge_kernel_matches_host_merge(world, k_in, k):
    g = torch.Generator().manual_seed(world * 100 + k)
    B = 37
    s = torch.randn(world, B, k_in, generator=g)
    s[0, :, 3] = s[0, :, 2]  # exact ties across ids
    i = torch.randint(0, 1 << 30, (world, B, k_in), generator=g, dtype=torch.int32)
    i[:, :, -1] = -1  # empty slots
    hs, hi = merge_topk_batch_host(s, i, k)
    ds, di = merge_topk_batch(s.cuda(), i.cuda(), k)
    assert torch.equal(di.cpu(), hi)
    assert torch.equal(ds.cpu(), hs)


@pytest.mark.parametrize("world", [2, 4])
def test_batched_shards_merge_to_brute_force(tmp_path, world):
    """Each shard answers the whole batch with circuit_search_batch; the
    rank-major gathered results, merged per query, are the global top-k."""
    w = WORKLOADS["spread-200k"]
    X = w.corpus(0, 30000, device="cuda")
    idx = build_circuit_index(X, num_roots=16, children_per_root=4, rank=8, device="cuda")
    path = str(tmp_path / "b.circuit")
    idx.save(path)
    Q = w.query_batch(70, device="cuda")
    S, I = [], []
    for r in range(world):
        sh = load_shard(path, r, world, device="cuda")
        s, i = circuit_search_batch(Q, sh, 10)
        S.append(s)
        I.append(i)
    ms, mi = merge_topk_batch(torch.stack(S), torch.stack(I), 10)
    exact = (Q.double() @ X.double().T).cpu().numpy()
    for b in range(Q.shape[0]):
        oracle.check_topk(exact[b], 10, ms[b].cpu().numpy(), mi[b].cpu().numpy())


@pytest.mark.parametrize("world", [2, 3])
def test_threshold_exchange_is_exact_and_prunes_no_less(tmp_path, world):
    """Seed phase on every shard, the max of the shards' seed thresholds, finish
    phase with it: the merged result is the exact global top-k, and no shard
    scans more rows than it does with its own seed alone."""
    import ctypes

    from circuit_rag import _native

    w = WORKLOADS["clustered-50k"]
    X = w.corpus(0, 40000, device="cuda")
    idx = build_circuit_index(X, num_roots=32, children_per_root=8, rank=8, device="cuda")
    path = str(tmp_path / "c.circuit")
    idx.save(path)
    shards = [load_shard(path, r, world, device="cuda") for r in range(world)]
    L = _native.lib()
    st = torch.cuda.current_stream().cuda_stream
    Q = w.query_batch(12, device="cuda")
    k = 10
    rows_plain, rows_ex = 0, 0
    tx = _native.TraceEx()
    for q in Q:
        exact = (X.double() @ q.double()).cpu().numpy()
        # plain: every shard prunes with its own seed
        for sh in shards:
            s = torch.empty(k, device="cuda")
            i = torch.empty(k, dtype=torch.int32, device="cuda")
            assert L.circuit_search_async(sh.native_handle(), q.data_ptr(), k, 0, s.data_ptr(), i.data_ptr(), None, st,
                                          None, None) == 0
            assert L.circuit_last_trace(sh.native_handle(), ctypes.byref(tx)) == 0 and tx.device_error == 0
            rows_plain += tx.vectors_scored
        # exchange: seeds -> max -> finish
        Ts = []
        for sh in shards:
            T = torch.empty(1, device="cuda")
            assert L.circuit_search_seed_async(sh.native_handle(), q.data_ptr(), k, T.data_ptr(), st) == 0
            Ts.append(T)
        Tmax = torch.stack(Ts).max().reshape(1).contiguous()
        assert float(Tmax) <= float(np.sort(exact)[-k]) + 1e-6  # never above the global k-th best
        S, I = [], []
        for sh, T in zip(shards, Ts):
            s = torch.empty(k, device="cuda")
            i = torch.empty(k, dtype=torch.int32, device="cuda")
            assert L.circuit_search_finish_async(sh.native_handle(), q.data_ptr(), k, Tmax.data_ptr(), s.data_ptr(),
                                                 i.data_ptr(), None, st, None, None) == 0
            assert L.circuit_last_trace(sh.native_handle(), ctypes.byref(tx)) == 0 and tx.device_error == 0
            rows_ex += tx.vectors_scored
            S.append(s)
            I.append(i)
        ms, mi = merge_topk(torch.cat(S), torch.cat(I), k)
        oracle.check_topk(exact, k, ms.cpu().numpy(), mi.cpu().numpy())
    assert rows_ex <= rows_plain
