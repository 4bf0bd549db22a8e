"""Worker processes for the multi-process (gloo, CPU) shard tests."""
import json
import os
import sys


def _paths(root):
    for p in (os.path.join(root, "circuit-rag_b200"), root):
        if p not in sys.path:
            sys.path.insert(0, p)


def search_worker(rank, world, port, root, index_path, queries_path, out_path, k, fail_rank=-1):
    _paths(root)
    import numpy as np
    import torch
    import torch.distributed as dist

    from circuit_rag.shard import ShardedSearcher, load_shard, merge_topk_batch_host, merge_topk_host
    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime

    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=4))
    result = {"rank": rank}
    try:
        idx = load_shard(index_path, rank, world, device="cpu")
        X = idx.leaf_vectors.numpy()
        gid = idx.original_ids.numpy()
        if rank == fail_rank:
            raise SystemExit(3)  # a rank that dies before its first collective

        def local(q, kk, _mh):
            s, rows = oracle.brute_topk(X, q.numpy(), min(kk, len(X)))
            out_s = torch.full((kk,), float("-inf"))
            out_i = torch.full((kk,), -1, dtype=torch.int32)
            out_s[:len(s)] = torch.from_numpy(s).float()
            out_i[:len(s)] = torch.from_numpy(gid[rows]).int()
            return out_s, out_i

        srch = ShardedSearcher(None, local_search=local, merge=merge_topk_host)
        Q = np.load(queries_path)
        res = []
        for q in Q:
            s, i = srch.search(torch.from_numpy(q), k=k)
            res.append({"scores": s.tolist(), "ids": i.tolist()})
        def local_batch(qs, kk):
            pairs = [local(q, kk, 0) for q in qs]
            return torch.stack([a for a, _ in pairs]), torch.stack([b for _, b in pairs])

        bs, bi = srch.search_batch(torch.from_numpy(Q), k=k, local_batch=local_batch, merge_batch=merge_topk_batch_host)

        # threshold exchange: seed = k-th best of this shard's first rows (any k
        # real rows qualify); finish = this shard's rows at or above the
        # exchanged threshold, padded with empty slots
        def seed(q, kk):
            n0 = min(len(X), max(kk, 40))
            s0 = np.sort(X[:n0].astype(np.float64) @ q.numpy().astype(np.float64))[::-1]
            return torch.tensor([s0[kk - 1] if n0 >= kk else float("-inf")], dtype=torch.float32)

        def finish(q, kk, T):
            s, rows = oracle.brute_topk(X, q.numpy(), min(kk, len(X)))
            keep = s >= float(T[0]) - 1e-6
            out_s = torch.full((kk,), float("-inf"))
            out_i = torch.full((kk,), -1, dtype=torch.int32)
            out_s[:int(keep.sum())] = torch.from_numpy(s[keep]).float()
            out_i[:int(keep.sum())] = torch.from_numpy(gid[rows[keep]]).int()
            return out_s, out_i

        ex = []
        for q in Q:
            s, i = srch.search(torch.from_numpy(q), k=k, exchange_threshold=True, local_seed=seed, local_finish=finish)
            ex.append({"scores": s.tolist(), "ids": i.tolist()})
        # no seed all-reduce: each shard finishes from its own seed
        own = []
        for q in Q:
            s, i = srch.search(torch.from_numpy(q), k=k, exchange_threshold=True, local_seed=seed, local_finish=finish,
                               seed_allreduce=False)
            own.append({"scores": s.tolist(), "ids": i.tolist()})
        try:
            srch.search(torch.from_numpy(Q[0]), k=k, exchange_threshold=True, local_seed=seed, seed_allreduce=False)
            needs_shared = False
        except ValueError:
            needs_shared = True
        result.update(ok=True, results=res, shard_rows=int(len(X)), shard_ids=gid.tolist(),
                      batch_results={"scores": bs.tolist(), "ids": bi.tolist()}, exchange_results=ex,
                      own_seed_results=own, own_seed_needs_shared=needs_shared)
    except SystemExit:
        raise
    except Exception as e:  # the survivor of a lost rank lands here
        result.update(ok=False, error=f"{type(e).__name__}: {e}")
    with open(out_path, "w") as f:
        json.dump(result, f)
    try:
        dist.destroy_process_group()
    except Exception:
        pass


def build_worker(rank, world, port, root, n, out_path):
    """Builds this rank's shard of a small clustered corpus with the
    shard-aware streaming builder (gloo collectives: broadcast of the root
    centres, all-gather of the row labels) and saves it."""
    _paths(root)
    import datetime

    import torch.distributed as dist

    from circuit_rag.hierarchy.build import build_circuit_index_streaming
    from circuit_rag.synthetic import WORKLOADS

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    w = WORKLOADS["zipf-10m"]
    idx = build_circuit_index_streaming(lambda s, e: w.corpus(s, e), n, w.dim, 12, 4, 6, device="cpu",
                                        chunk=1500, sample=4000, shard_rank=rank, world=world, block_rows=16)
    idx.save(out_path)
    with open(out_path + ".json", "w") as f:
        json.dump(idx.shard_info, f)
    dist.destroy_process_group()


def ipc_word_worker(rank, root, conn, barrier, result_q):
    """One of two processes on one GPU that open each other's shared threshold
    word through CUDA IPC and search the same query with the same tag."""
    _paths(root)
    import ctypes
    import dataclasses

    import numpy as np

    import torch

    from circuit_rag import _native, build_circuit_index
    from circuit_rag.synthetic import WORKLOADS

    try:
        torch.cuda.set_device(0)
        w = dataclasses.replace(WORKLOADS["clustered-50k"], name="c200k", n=200_000)
        X = w.corpus(device="cuda")
        idx = build_circuit_index(X, num_roots=w.num_roots, children_per_root=w.children_per_root, rank=w.rank,
                                  device="cuda")
        L = _native.lib()
        word = torch.zeros(1, dtype=torch.int64, device="cuda")
        handle = (ctypes.c_ubyte * 64)()
        off = ctypes.c_int64()
        assert L.circuit_ipc_export(word.data_ptr(), handle, ctypes.byref(off)) == 0, _native.last_error()
        conn.send((bytes(handle), off.value))
        peer_handle, peer_off = conn.recv()
        ptr = ctypes.c_void_p()
        assert L.circuit_ipc_import(peer_handle, 0, ctypes.byref(ptr)) == 0, _native.last_error()
        peers = torch.tensor([ptr.value + peer_off], dtype=torch.int64, device="cuda")
        barrier.wait(timeout=120)
        q = w.query_batch(3, device="cuda")[2].contiguous()
        k = w.k
        st = torch.cuda.current_stream().cuda_stream
        T = torch.empty(1, device="cuda")
        s = torch.empty(k, device="cuda")
        i = torch.empty(k, dtype=torch.int32, device="cuda")
        assert L.circuit_search_seed_async(idx.native_handle(), q.data_ptr(), k, T.data_ptr(), st) == 0
        assert L.circuit_search_finish_shared_async(idx.native_handle(), q.data_ptr(), k, T.data_ptr(),
                                                    word.data_ptr(), peers.data_ptr(), 1, 7, s.data_ptr(),
                                                    i.data_ptr(), None, st, None, None) == 0
        torch.cuda.synchronize()
        exact = (X.double() @ q.double()).cpu().numpy()
        oracle_kth = float(np.sort(exact)[-k])
        ok_ids = set(np.argsort(-exact)[:k].tolist())
        barrier.wait(timeout=120)  # both scans are complete: both words are final
        torch.cuda.synchronize()
        result_q.put((rank, int(word.item()), oracle_kth, sorted(i.cpu().tolist()) == sorted(ok_ids)))
        barrier.wait(timeout=120)  # the peer has read its word before the mapping goes
        assert L.circuit_ipc_close(ptr) == 0
        idx.close()
    except Exception as e:  # reported to the parent
        result_q.put((rank, None, repr(e), False))
