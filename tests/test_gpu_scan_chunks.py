"""The main scan's claimed-chunk mode (streams of about 1.8M rows and more are
cut into chunks that the CTAs take from a counter instead of equal slices):
flat and hierarchical searches over a 3M-row index with thousands of short
child ranges, k = 10 and 100, against float64 brute force; the device-buffer
blocking call on the same index; and a mid-size index that stays in
equal-slice mode, for comparison."""
import numpy as np
import pytest
import torch

from circuit_rag import _native, circuit_search
from circuit_rag.hierarchy.build import build_circuit_index_streaming
from circuit_rag.synthetic import Workload
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
W = Workload("zipf-3m-d128", 3_000_000, 128, 256, 32, 8, 10, 16, "clustered", 4096, 0.08, 1.1)


def _exact(idx, Q, k):
    """float64 top-(k + 8) (scores, original ids) per query over the index rows."""
    kk = k + 8
    best_s = torch.full((Q.shape[0], kk), float("-inf"), dtype=torch.float64, device=DEV)
    best_i = torch.full((Q.shape[0], kk), -1, dtype=torch.int64, device=DEV)
    for a in range(0, idx.N, 1 << 20):
        s = idx.leaf_vectors[a:a + (1 << 20)].double() @ Q.double().T
        v, r = torch.topk(s, kk, dim=0)
        cs = torch.cat([best_s, v.T], dim=1)
        ci = torch.cat([best_i, idx.original_ids[a:a + (1 << 20)].long()[r].T], dim=1)
        t, o = torch.topk(cs, kk, dim=1)
        best_s, best_i = t, torch.gather(ci, 1, o)
    return best_s.cpu().numpy(), best_i.cpu().numpy()


def _check(s, i, es, ei, k):
    s, i = np.asarray(s, np.float64), np.asarray(i)
    kth = es[k - 1]
    assert len(set(i.tolist())) == k and np.all(np.diff(s) <= 0)
    assert set(ei[es > kth + oracle.TIE_ABS].tolist()) <= set(i.tolist())
    exact_of = dict(zip(ei.tolist(), es.tolist()))
    for sc, idv in zip(s, i):
        e = exact_of.get(int(idv))
        if e is None:
            assert sc >= kth - 1e-5
        else:
            assert e >= kth - oracle.TIE_ABS and abs(sc - e) <= oracle.SCORE_REL * abs(e) + oracle.TIE_ABS


@pytest.fixture(scope="module")
def idx3m():
    idx = build_circuit_index_streaming(lambda s, e: W.corpus(s, e, device=DEV), W.n, W.dim, W.num_roots,
                                        W.children_per_root, W.rank, device=DEV)
    yield idx
    idx.close()


@pytest.mark.parametrize("k", [10, 100])
@pytest.mark.parametrize("flat", [True, False])
def test_claimed_chunks_exact(idx3m, k, flat):
    Q = W.query_batch(12, device=DEV)
    es, ei = _exact(idx3m, Q, k)
    for b in range(Q.shape[0]):
        s, i, tr = circuit_search(Q[b], idx3m, k=k, min_hierarchy_n=(1 << 40) if flat else 0)
        _check(s.cpu().numpy(), i.cpu().numpy(), es[b], ei[b], k)
        if not flat:
            assert tr.vectors_scored <= W.n


def test_claimed_chunks_blocking_device_buffers(idx3m):
    L = _native.lib()
    h = idx3m.native_handle()
    Q = W.query_batch(6, device=DEV).contiguous()
    es, ei = _exact(idx3m, Q, 10)
    s = torch.empty(10, device=DEV)
    i = torch.empty(10, dtype=torch.int32, device=DEV)
    for rep in range(2):  # the second call replays the captured graph
        for b in range(Q.shape[0]):
            assert L.circuit_search_device(h, Q[b].data_ptr(), 10, s.data_ptr(), i.data_ptr(), None) == 0
            _check(s.cpu().numpy(), i.cpu().numpy(), es[b], ei[b], 10)
