"""GPU tests of the running threshold shared between shards while their scans run
(circuit_search_finish_shared_async).  Each shard owns a 64-bit word holding
tag << 32 | key; its main scan raises its own word and every peer's with the
k-th best scores it finds and prunes with the largest key carrying the query's
tag.  Checked: the merged top-k of three shards in one process (their words are
plain device pointers to each other) equals float64 brute force, every word ends
with the query's tag and a key no higher than the exact k-th best, the shards
read no more rows than without sharing; and two processes on one GPU that open
each other's word through CUDA IPC end with equal words.  Parity rule:
oracle.check_topk."""
import ctypes
import multiprocessing as mp
import os

import numpy as np
import pytest
import torch

from circuit_rag import _native, build_circuit_index
from circuit_rag.shard import load_shard, merge_topk
from circuit_rag.synthetic import WORKLOADS
from oracle import oracle
from shard_worker import ipc_word_worker

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _f2key(x: float) -> int:
    b = int(np.array([x], dtype=np.float32).view(np.uint32)[0])
    return (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)


def _trace(L, h):
    tx = _native.TraceEx()
    assert L.circuit_last_trace(h, ctypes.byref(tx)) == 0 and tx.device_error == 0
    return tx


@pytest.mark.parametrize("seed", ["max", "own"])
def test_three_shards_share_the_running_threshold(tmp_path, seed):
    """seed = "max": every shard starts from the largest seed (the all-reduce);
    "own": no seed exchange, each shard starts from its own seed and learns
    the others' thresholds only through the shared words (exact either way;
    only "max" is held to reading no more rows than the unshared search)."""
    import dataclasses

    w = dataclasses.replace(WORKLOADS["clustered-50k"], name="clustered-600k", n=600_000)
    X = w.corpus(device=DEV)
    idx = build_circuit_index(X, num_roots=w.num_roots, children_per_root=w.children_per_root, rank=w.rank,
                              device=DEV)
    path = str(tmp_path / "c.circuit")
    idx.save(path)
    idx.close()
    world = 3
    shards = [load_shard(path, r, world, device=DEV) for r in range(world)]
    L = _native.lib()
    st = torch.cuda.current_stream().cuda_stream
    words = torch.zeros(world, dtype=torch.int64, device=DEV)
    peers = [torch.tensor([words[j:j + 1].data_ptr() for j in range(world) if j != r], dtype=torch.int64,
                          device=DEV) for r in range(world)]
    k = w.k
    rows_shared = rows_plain = 0
    for tag, q in enumerate(w.query_batch(12, device=DEV), start=1):
        exact = (X.double() @ q.double()).cpu().numpy()
        kth = float(np.sort(exact)[-k])
        for shared in (False, True):
            Ts = []
            for sh in shards:
                T = torch.empty(1, device=DEV)
                assert L.circuit_search_seed_async(sh.native_handle(), q.data_ptr(), k, T.data_ptr(), st) == 0
                Ts.append(T)
            Tmax = torch.stack(Ts).max().reshape(1).contiguous()
            S, I = [], []
            for r, sh in enumerate(shards):
                s = torch.empty(k, device=DEV)
                i = torch.empty(k, dtype=torch.int32, device=DEV)
                if shared:
                    T_in = Tmax if seed == "max" else Ts[r]
                    assert L.circuit_search_finish_shared_async(
                        sh.native_handle(), q.data_ptr(), k, T_in.data_ptr(), words[r:r + 1].data_ptr(),
                        peers[r].data_ptr(), world - 1, tag, s.data_ptr(), i.data_ptr(), None, st, None, None) == 0
                else:
                    assert L.circuit_search_finish_async(sh.native_handle(), q.data_ptr(), k, Tmax.data_ptr(),
                                                         s.data_ptr(), i.data_ptr(), None, st, None, None) == 0
                tx = _trace(L, sh.native_handle())
                if shared:
                    rows_shared += tx.rows_streamed
                else:
                    rows_plain += tx.rows_streamed
                S.append(s)
                I.append(i)
            ms, mi = merge_topk(torch.cat(S), torch.cat(I), k)
            oracle.check_topk(exact, k, ms.cpu().numpy(), mi.cpu().numpy())
        # every word carries this query's tag and a valid threshold key
        for wv in words.cpu().numpy().astype(np.uint64):
            assert int(wv) >> 32 == tag
            assert int(wv) & 0xFFFFFFFF <= _f2key(kth + 1e-6)
    if seed == "max":
        assert rows_shared <= rows_plain, (rows_shared, rows_plain)
    else:
        # the shards run one after another here, so the first learns nothing from
        # the others and every shard starts below the largest seed: more rows
        print(f"\n[own seeds] rows streamed {rows_shared} (with the largest seed and no words: {rows_plain})")
    for sh in shards:
        sh.close()


def test_two_processes_open_each_others_word_through_ipc():
    ctx = mp.get_context("spawn")
    a, b = ctx.Pipe()
    barrier = ctx.Barrier(2)
    q = ctx.Queue()
    env_root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    procs = [ctx.Process(target=ipc_word_worker, args=(r, env_root, c, barrier, q)) for r, c in ((0, a), (1, b))]
    try:
        for p in procs:
            p.start()
        res = [q.get(timeout=600) for _ in range(2)]
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.terminate()
    res.sort()
    for rank, word, kth, exact_ok in res:
        assert word is not None, kth
        assert exact_ok
        assert word >> 32 == 7
        assert (word & 0xFFFFFFFF) <= _f2key(kth + 1e-6)
    assert res[0][1] == res[1][1]  # each scan raised both words
