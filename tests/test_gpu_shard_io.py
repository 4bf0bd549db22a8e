"""A 10M-row index written by the streaming builder, loaded whole and as
shards (native circuit_load_shard and the Python load_shard), searched, and
compared with float64 brute force; the load rates are printed."""
import ctypes
import os
import time

import numpy as np
import pytest
import torch

from circuit_rag import _native
from circuit_rag.hierarchy.build import build_circuit_index_streaming
from circuit_rag.shard import load_shard, merge_topk
from circuit_rag.synthetic import Workload
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"

# 10M rows of a Zipf(1.1) clustered corpus, D = 128 (a 5.1 GB file)
W = Workload("zipf-10m-d128", 10_000_000, 128, 64, 16, 8, 10, 64, "clustered", 2048, 0.08, 1.1)


@pytest.fixture(scope="module")
def big_index(tmp_path_factory):
    idx = build_circuit_index_streaming(lambda s, e: W.corpus(s, e, device=DEV), W.n, W.dim, W.num_roots,
                                        W.children_per_root, W.rank, device=DEV)
    path = str(tmp_path_factory.mktemp("big") / "z10m.circuit")
    t = time.perf_counter()
    idx.save(path)
    print(f"\n[shard io] wrote {os.path.getsize(path) / 1e9:.2f} GB in {time.perf_counter() - t:.1f} s")
    yield idx, path
    idx.close()
    os.remove(path)


def _exact_topk(idx, Q, k):
    """float64 top-k (scores, original ids) of every query over the whole index."""
    out = []
    leaf, ids = idx.leaf_vectors, idx.original_ids
    best_s = torch.full((Q.shape[0], k), float("-inf"), dtype=torch.float64, device=DEV)
    best_i = torch.full((Q.shape[0], k), -1, dtype=torch.int64, device=DEV)
    Qd = Q.double()
    for a in range(0, idx.N, 1 << 21):
        s = leaf[a:a + (1 << 21)].double() @ Qd.T
        v, r = torch.topk(s, k, dim=0)
        cs = torch.cat([best_s, v.T], dim=1)
        ci = torch.cat([best_i, ids[a:a + (1 << 21)].long()[r].T], dim=1)
        t, o = torch.topk(cs, k, dim=1)
        best_s, best_i = t, torch.gather(ci, 1, o)
    return best_s, best_i


def _check(res_s, res_i, ex_s, ex_i, k):
    for b in range(len(res_s)):
        s, i = np.asarray(res_s[b]), np.asarray(res_i[b])
        es, ei = ex_s[b].cpu().numpy(), ex_i[b].cpu().numpy()
        kth = es[k - 1]
        must = set(ei[es > kth + oracle.TIE_ABS].tolist())
        assert must <= set(i.tolist())
        assert len(set(i.tolist())) == k
        exact_of = dict(zip(ei.tolist(), es.tolist()))
        for sc, idv in zip(s, i):
            if int(idv) in exact_of:
                assert abs(sc - exact_of[int(idv)]) <= oracle.SCORE_REL * abs(exact_of[int(idv)]) + oracle.TIE_ABS
            else:  # a tie at the k-th score
                assert sc >= kth - 1e-5
        assert np.all(np.diff(s) <= 0)


def test_10m_index_whole_and_native_shards(big_index):
    idx, path = big_index
    L = _native.lib()
    Q = W.query_batch(8, device=DEV)
    k = 10
    ex_s, ex_i = _exact_topk(idx, Q, k)
    size = os.path.getsize(path)
    t = time.perf_counter()
    h = L.circuit_load_index(path.encode(), 0)
    t_whole = time.perf_counter() - t
    assert h, _native.last_error()
    res_s, res_i = [], []
    for q in Q.cpu().numpy():
        s = np.zeros(k, np.float32)
        i = np.zeros(k, np.int32)
        assert L.circuit_search(h, np.ascontiguousarray(q).ctypes.data, k, s.ctypes.data, i.ctypes.data, None) == 0
        res_s.append(s)
        res_i.append(i)
    L.circuit_destroy_index(h)
    _check(res_s, res_i, ex_s, ex_i, k)
    print(f"\n[shard io] circuit_load_index: {size / 1e9:.2f} GB in {t_whole:.2f} s = {size / t_whole / 1e9:.2f} GB/s")
    for world in (2, 3):
        handles, t_load, rows = [], 0.0, 0
        for r in range(world):
            t = time.perf_counter()
            hs = L.circuit_load_shard(path.encode(), r, world, 0, 1.05)
            t_load += time.perf_counter() - t
            assert hs, _native.last_error()
            info = (ctypes.c_int64 * 8)()
            assert L.circuit_index_info(hs, info) == 0
            rows += info[4]
            handles.append((hs, info[4]))
        assert rows == W.n
        assert max(n for _, n in handles) <= 1.05 * W.n / world + 200_000
        Qd = Q.contiguous()
        merged_s, merged_i = [], []
        for b in range(Q.shape[0]):
            S, I = [], []
            for hs, _ in handles:
                s = torch.empty(k, device=DEV)
                i = torch.empty(k, dtype=torch.int32, device=DEV)
                assert L.circuit_search_async(hs, Qd[b].data_ptr(), k, 0, s.data_ptr(), i.data_ptr(), None,
                                              torch.cuda.current_stream().cuda_stream, None, None) == 0
                S.append(s)
                I.append(i)
            ms, mi = merge_topk(torch.cat(S), torch.cat(I), k)
            merged_s.append(ms.cpu().numpy())
            merged_i.append(mi.cpu().numpy())
        _check(merged_s, merged_i, ex_s, ex_i, k)
        # shards and the whole index score every row with the same arithmetic
        for b in range(Q.shape[0]):
            assert np.array_equal(merged_s[b], res_s[b])
        for hs, _ in handles:
            L.circuit_destroy_index(hs)
        print(f"[shard io] circuit_load_shard x {world}: {t_load:.2f} s for the whole file "
              f"= {size / t_load / 1e9:.2f} GB/s")


def test_10m_index_python_shards(big_index):
    idx, path = big_index
    Q = W.query_batch(4, device=DEV)
    k = 10
    ex_s, ex_i = _exact_topk(idx, Q, k)
    shards = [load_shard(path, r, 2, device=DEV) for r in range(2)]
    assert sum(s.N for s in shards) == W.n
    from circuit_rag import circuit_search

    res_s, res_i = [], []
    for q in Q:
        S, I = [], []
        for sh in shards:
            s, i, _ = circuit_search(q, sh, k=k)
            S.append(s)
            I.append(i)
        ms, mi = merge_topk(torch.cat(S), torch.cat(I), k)
        res_s.append(ms.cpu().numpy())
        res_i.append(mi.cpu().numpy())
    _check(res_s, res_i, ex_s, ex_i, k)
    for sh in shards:
        sh.close()
