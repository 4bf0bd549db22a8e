"""Builder invariants that the search's pruning relies on (CPU)."""
import numpy as np
import pytest
import torch

from circuit_rag import build_circuit_index, circuit_search
from circuit_rag.synthetic import WORKLOADS


def _check_invariants(idx, X):
    lv = idx.leaf_vectors.double()
    assert torch.equal(idx.leaf_vectors, torch.from_numpy(X)[idx.original_ids.long()])
    assert sorted(idx.original_ids.tolist()) == list(range(len(X)))
    covered = 0
    for c in range(idx.num_total_children):
        n = int(idx.leaf_sizes[c])
        if n == 0:
            continue
        o, p = int(idx.leaf_offsets[c]), int(idx.child_parent_ids[c])
        x = lv[o:o + n]
        cP = idx.root_centers[p].double()
        V = idx.bases[p].double()
        d = x - cP
        assert (d.norm(dim=1) <= idx.root_radii[p].double()).all()
        z = d @ V
        assert (z >= idx.child_intervals_l[c].double()).all() and (z <= idx.child_intervals_u[c].double()).all()
        r = d - z @ V.T
        assert (r.norm(dim=1) <= idx.child_radii[c].double()).all()
        covered += n
    assert covered == len(X)
    # root-major, child-contiguous layout
    offs = idx.leaf_offsets[idx.leaf_sizes > 0]
    assert torch.all(offs[1:] > offs[:-1])


@pytest.mark.parametrize("rank", [1, 8, 64])
def test_certificates_hold_exactly(rank):
    X = WORKLOADS["clustered-50k"].corpus(0, 3000).numpy()
    idx = build_circuit_index(X, num_roots=8, children_per_root=4, rank=rank, device="cpu")
    _check_invariants(idx, X)
    V = idx.bases[0].double()
    assert torch.allclose(V.T @ V, torch.eye(rank, dtype=torch.float64), atol=1e-5)


def test_rank_limits():
    X = np.random.default_rng(0).normal(size=(200, 8)).astype(np.float32)
    with pytest.raises(ValueError):
        build_circuit_index(X, num_roots=4, children_per_root=2, rank=65, device="cpu")
    with pytest.raises(ValueError):
        build_circuit_index(X, num_roots=4, children_per_root=2, rank=0, device="cpu")


def test_search_requires_cuda_and_validates_shape():
    X = np.random.default_rng(0).normal(size=(300, 8)).astype(np.float32)
    idx = build_circuit_index(X, num_roots=4, children_per_root=2, rank=2, device="cpu")
    with pytest.raises(ValueError):
        circuit_search(torch.zeros(7), idx)
    with pytest.raises(RuntimeError, match="CUDA"):
        circuit_search(torch.zeros(8), idx)
    # the batched search and the per-stage ops refuse CPU tensors too (no CPU path)
    from circuit_rag import circuit_search_batch
    import circuit_cuda

    with pytest.raises(ValueError):
        circuit_search_batch(torch.zeros(3, 7), idx, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        circuit_search_batch(torch.zeros(3, 8), idx, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        circuit_cuda.flat_exact_score(torch.zeros(8), torch.zeros(300, 8))
    with pytest.raises(RuntimeError, match="CUDA"):
        circuit_cuda.evaluate_root_bounds(torch.zeros(8), torch.zeros(4, 8), torch.zeros(4), 0.0)


def test_append_keeps_certificates_and_layout():
    """CircuitIndex.append: new rows (some far from every centre) join their
    nearest root under new children; every certificate still holds exactly and
    the layout stays root-major and child-contiguous."""
    w = WORKLOADS["clustered-50k"]
    X1 = w.corpus(0, 3000).numpy()
    idx = build_circuit_index(X1, num_roots=8, children_per_root=4, rank=6, device="cpu")
    rng = np.random.default_rng(7)
    X2 = w.corpus(3000, 3400).numpy()
    X3 = (rng.normal(size=(60, X1.shape[1])) * 3.0).astype(np.float32)  # outside every root's old radius
    idx.append(X2)
    idx.append(X3)
    X = np.concatenate([X1, X2, X3])
    assert idx.N == len(X)
    assert idx.num_total_children > 8 * 4
    _check_invariants(idx, X)


def test_append_validates_shapes():
    X = np.random.default_rng(0).normal(size=(300, 8)).astype(np.float32)
    idx = build_circuit_index(X, num_roots=4, children_per_root=2, rank=2, device="cpu")
    with pytest.raises(ValueError):
        idx.append(np.zeros((3, 7), np.float32))
    with pytest.raises(ValueError):
        idx.append(np.zeros((3, 8), np.float32), ids_new=[1, 2])


def test_rag_appends_then_rebuilds():
    from circuit_rag import CircuitRAG

    dim = 16

    def embed(texts):
        out = np.stack([np.random.default_rng(abs(hash(t)) % (2 ** 32)).normal(size=dim) for t in texts])
        return (out / np.linalg.norm(out, axis=1, keepdims=True)).astype(np.float32)

    rag = CircuitRAG(device="cpu", embed_fn=embed)
    ids = rag.add_documents([f"doc {i}" for i in range(600)])
    assert ids == list(range(600)) and rag.index.N == 600 and rag.appended_rows == 0
    rag.add_documents([f"more {i}" for i in range(200)], [{"i": i} for i in range(200)])
    assert rag.index.N == 800 and rag.appended_rows == 200  # appended, not rebuilt
    rag.add_documents([f"late {i}" for i in range(200)])
    assert rag.index.N == 1000 and rag.appended_rows == 0   # beyond half of the last build: rebuilt
    with pytest.raises(ValueError):
        rag.add_documents(["a", "b"], [{}])


def test_appended_index_saves_and_shards(tmp_path):
    from circuit_rag.shard import load_shard

    w = WORKLOADS["clustered-50k"]
    X1 = w.corpus(0, 2000).numpy()
    idx = build_circuit_index(X1, num_roots=6, children_per_root=3, rank=4, device="cpu")
    X2 = w.corpus(2000, 2300).numpy()
    idx.append(X2)
    X = np.concatenate([X1, X2])
    path = str(tmp_path / "a.circuit")
    idx.save(path)
    ids = []
    for r in range(2):
        sh = load_shard(path, r, 2, device="cpu")
        assert torch.equal(sh.leaf_vectors, torch.from_numpy(X)[sh.original_ids.long()])
        offs = sh.leaf_offsets[sh.leaf_sizes > 0]
        assert torch.all(offs[1:] > offs[:-1])
        ids += sh.original_ids.tolist()
    assert sorted(ids) == list(range(len(X)))
