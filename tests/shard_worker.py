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
        result.update(ok=True, results=res, shard_rows=int(len(X)), shard_ids=gid.tolist(),
                      batch_results={"scores": bs.tolist(), "ids": bi.tolist()}, exchange_results=ex)
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
