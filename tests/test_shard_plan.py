"""Shard planning and the shard-aware streaming builder (CPU; gloo world 2).

A root too large for one rank's share is cut between children (or between
blocks of rows in the builder); every part keeps a contiguous range, all rows
are covered exactly once, and the busiest rank stays within 1.05 x the mean."""
import json
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

from circuit_rag.hierarchy.build import build_circuit_index_streaming
from circuit_rag.shard import load_shard, plan_shard_parts
from circuit_rag.storage.format import load_circuit_index
from circuit_rag.synthetic import WORKLOADS, zipf_cdf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _zipf_shaped_roots(num_roots=256, children=32, n=10_000_000, centers=4096, seed=0):
    """Root and child sizes shaped like the zipf-10m index: 4,096 Zipf(1.1)
    clusters grouped into 256 roots (the largest cluster alone is ~15 % of the
    rows), each root cut into 32 children of random proportions."""
    rng = np.random.default_rng(seed)
    cdf = zipf_cdf(centers, 1.1).numpy()
    mass = np.diff(np.concatenate([[0.0], cdf])) * n
    owner = rng.integers(0, num_roots, size=centers)
    owner[0] = 0
    root_rows = np.bincount(owner, weights=mass, minlength=num_roots)
    atoms, ptr = [], [0]
    for p in range(num_roots):
        w = rng.dirichlet(np.ones(children))
        sizes = np.floor(w * root_rows[p]).astype(np.int64)
        sizes[0] += int(round(root_rows[p])) - sizes.sum()
        sizes = np.maximum(sizes, 0)
        atoms.extend(sizes.tolist())
        ptr.append(len(atoms))
    return np.array(atoms, np.int64), np.array(ptr, np.int64)


def _check_plan(plan, atoms, ptr, world):
    R = len(ptr) - 1
    covered = np.zeros(len(atoms), np.int64)
    for p, a, b in zip(plan["part_root"], plan["part_atom_begin"], plan["part_atom_end"]):
        assert ptr[p] <= a < b <= ptr[p + 1]  # a contiguous atom range of one root
        covered[a:b] += 1
    assert np.all(covered[atoms > 0] == 1)
    loads = np.zeros(world, np.int64)
    for p, a, b, r in zip(plan["part_root"], plan["part_atom_begin"], plan["part_atom_end"], plan["part_rank"]):
        loads[r] += atoms[a:b].sum()
    assert np.array_equal(loads, plan["rank_rows"])
    assert loads.sum() == atoms.sum()
    return loads


@pytest.mark.parametrize("world", [2, 4, 8])
def test_zipf_shaped_roots_balance_within_5_percent(world):
    atoms, ptr = _zipf_shaped_roots()
    root_rows = np.add.reduceat(atoms, ptr[:-1])
    assert root_rows.max() > atoms.sum() / 8  # a root larger than one of 8 shares
    plan = plan_shard_parts(atoms, ptr, world, 1.05)
    loads = _check_plan(plan, atoms, ptr, world)
    assert loads.max() <= 1.05 * loads.mean(), (loads.max() / loads.mean())
    # whole-root planning could not do this at 8 ranks
    if world == 8:
        assert root_rows.max() > 1.05 * loads.mean()


def test_plan_keeps_whole_roots_when_they_fit():
    atoms = np.array([5, 5, 3, 3, 2, 2, 1, 1], np.int64)
    ptr = np.array([0, 2, 4, 6, 8], np.int64)
    plan = plan_shard_parts(atoms, ptr, 2, 1.5)
    assert len(plan["part_root"]) == 4  # no root is cut
    _check_plan(plan, atoms, ptr, 2)
    one = plan_shard_parts(atoms, ptr, 1, 1.05)
    assert (one["part_rank"] == 0).all() and len(one["part_root"]) == 4


def _check_certificates(idx, X):
    lv = idx.leaf_vectors.double()
    assert torch.equal(idx.leaf_vectors, torch.from_numpy(X)[idx.original_ids.long()])
    for c in range(idx.num_total_children):
        n = int(idx.leaf_sizes[c])
        if n == 0:
            continue
        o, p = int(idx.leaf_offsets[c]), int(idx.child_parent_ids[c])
        d = lv[o:o + n] - idx.root_centers[p].double()
        V = idx.bases[p].double()
        assert (d.norm(dim=1) <= idx.root_radii[p].double()).all()
        z = d @ V
        assert (z >= idx.child_intervals_l[c].double()).all() and (z <= idx.child_intervals_u[c].double()).all()
        assert ((d - z @ V.T).norm(dim=1) <= idx.child_radii[c].double()).all()
    offs = idx.leaf_offsets[idx.leaf_sizes > 0]
    assert torch.all(offs[1:] > offs[:-1])


def test_streaming_builder_certificates_hold_exactly():
    """One process: every row inside its root sphere, its child box and its
    residual radius (float64), root-major child-contiguous layout."""
    w = WORKLOADS["mixed-100m"]
    n = 9000
    X = w.corpus(0, n).numpy()
    idx = build_circuit_index_streaming(lambda s, e: w.corpus(s, e), n, w.dim, 10, 6, 12, device="cpu",
                                        chunk=2000, sample=5000)
    assert sorted(idx.original_ids.tolist()) == list(range(n))
    _check_certificates(idx, X)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_build_over_gloo(tmp_path):
    """Two ranks build their shards with collectives: together they hold every
    row exactly once, each shard's certificates hold, and the shards are
    balanced within 1.05 x the mean (plus one block of rows)."""
    n, world = 6000, 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    from shard_worker import build_worker

    outs = [str(tmp_path / f"s{r}.circuit") for r in range(world)]
    procs = [ctx.Process(target=build_worker, args=(r, world, port, ROOT, n, outs[r])) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("builder did not finish")
    assert all(p.exitcode == 0 for p in procs)
    X = WORKLOADS["zipf-10m"].corpus(0, n).numpy()
    ids = []
    rows = []
    for o in outs:
        sh = load_circuit_index(o, device="cpu")
        _check_certificates(sh, X)
        ids += sh.original_ids.tolist()
        rows.append(sh.N)
        info = json.load(open(o + ".json"))
        assert info["rank_rows"] == json.load(open(outs[0] + ".json"))["rank_rows"]
    assert sorted(ids) == list(range(n))
    assert max(rows) <= 1.05 * n / world + 16


def test_file_shards_cut_oversized_roots(tmp_path):
    """load_shard on an index whose largest root exceeds a rank's share: that
    root is split between children, each part a root of its shard with the
    original centre; shards partition the rows and stay balanced."""
    w = WORKLOADS["zipf-10m"]
    X = w.corpus(0, 8000).numpy()
    from circuit_rag import build_circuit_index

    idx = build_circuit_index(X, num_roots=3, children_per_root=12, rank=4, device="cpu")
    path = str(tmp_path / "z.circuit")
    idx.save(path)
    world = 4
    ids, loads = [], []
    for r in range(world):
        sh = load_shard(path, r, world, device="cpu")
        assert np.array_equal(sh.leaf_vectors.numpy(), X[sh.original_ids.numpy()])
        _check_certificates(sh, X)
        for j, p in enumerate(sh.shard_info["part_root"]):
            assert torch.equal(sh.root_centers[j], idx.root_centers[p])
        ids += sh.original_ids.tolist()
        loads.append(sh.N)
    assert sorted(ids) == list(range(len(X)))
    sizes = idx.leaf_sizes.numpy()
    assert max(loads) <= 1.05 * len(X) / world + sizes.max()


def _random_roots(rng, num_roots, max_atoms, max_rows, zero_frac):
    atoms, ptr = [], [0]
    for _ in range(num_roots):
        n = int(rng.integers(0, max_atoms + 1))
        sizes = rng.integers(0, max_rows + 1, size=n)
        sizes[rng.random(n) < zero_frac] = 0
        atoms.extend(int(x) for x in sizes)
        ptr.append(len(atoms))
    return np.array(atoms, np.int64), np.array(ptr, np.int64)


@pytest.mark.parametrize("seed", range(40))
def test_plan_invariants_on_random_roots(seed):
    """Any roots (empty roots, zero-row atoms, one root holding most rows, more
    ranks than roots): every non-empty atom is planned once, each part is a
    contiguous atom range of one root, the rank loads add up, no rank exceeds
    max_imbalance x the mean by more than one atom, and the plan is the same
    every time (every rank computes it on its own)."""
    rng = np.random.default_rng(seed)
    num_roots = int(rng.integers(1, 40))
    atoms, ptr = _random_roots(rng, num_roots, max_atoms=int(rng.integers(1, 12)),
                               max_rows=int(rng.choice([1, 10, 1000])), zero_frac=float(rng.choice([0.0, 0.3])))
    if seed % 5 == 0 and len(atoms):
        atoms[int(rng.integers(0, len(atoms)))] += int(atoms.sum()) * 3  # one dominant atom's root
    world = int(rng.integers(1, 10))
    imb = float(rng.choice([1.0, 1.05, 1.5]))
    plan = plan_shard_parts(atoms, ptr, world, imb)
    loads = _check_plan(plan, atoms, ptr, world)
    if atoms.sum() > 0:
        assert loads.max() <= imb * atoms.sum() / world + atoms.max(), (loads, imb, atoms.max())
    again = plan_shard_parts(atoms, ptr, world, imb)
    for key in plan:
        assert np.array_equal(plan[key], again[key]), key
    # parts are ordered by rank, root, first atom
    order = list(zip(plan["part_rank"], plan["part_root"], plan["part_atom_begin"]))
    assert order == sorted(order)


def test_plan_rejects_bad_arguments():
    from circuit_rag import _native

    atoms = np.array([3, 4, 5], np.int64)
    with pytest.raises(_native.NativeLibraryError):
        plan_shard_parts(atoms, np.array([0, 2, 3], np.int64), 0, 1.05)  # no ranks
    with pytest.raises(_native.NativeLibraryError):
        plan_shard_parts(atoms, np.array([0, 2, 3], np.int64), 2, 0.9)  # imbalance below 1
    with pytest.raises(_native.NativeLibraryError):
        plan_shard_parts(atoms, np.array([0, 2, 1], np.int64), 2, 1.05)  # decreasing pointers
    with pytest.raises(_native.NativeLibraryError):
        plan_shard_parts(np.array([3, -4, 5], np.int64), np.array([0, 2, 3], np.int64), 2, 1.05)  # negative rows
