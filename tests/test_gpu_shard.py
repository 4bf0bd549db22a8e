"""GPU side of the sharded search: the device merge kernel and shards loaded
from one .circuit file, searched one by one and merged, against brute force."""
import os

import numpy as np
import pytest
import torch

from circuit_rag import build_circuit_index, circuit_search
from circuit_rag.shard import load_shard, merge_topk, merge_topk_host
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
