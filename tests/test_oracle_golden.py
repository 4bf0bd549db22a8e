"""Pins the oracle against outputs of the reference package itself
(tests/golden/*, produced by tests/golden/make_golden.py)."""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _g(name):
    return os.path.join(GOLDEN, name)


def clustered_like_reference_test(n=40000, dim=128, clusters=64, seed=0):
    """tests/test_exact.py:9-14 of the reference, restated."""
    rng = np.random.default_rng(seed)
    centers = rng.normal(size=(clusters, dim))
    X = centers[rng.integers(0, clusters, n)] + 0.3 * rng.normal(size=(n, dim))
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    return X.astype(np.float32)


def test_manifest_matches_fixtures():
    man = json.load(open(_g("MANIFEST.json")))["sha256"]
    for name, digest in man.items():
        with open(_g(name), "rb") as f:
            assert hashlib.sha256(f.read()).hexdigest() == digest, name


def test_reference_test_data_and_truth():
    """The restated generator reproduces the reference test's corpus, and the
    oracle's brute force reproduces the reference's torch.topk truth."""
    g = np.load(_g("ref_test_exact.npz"))
    X = clustered_like_reference_test()
    assert np.isclose(X.astype(np.float64).sum(), float(g["x_sum"]), rtol=0, atol=1e-6)
    assert np.array_equal(X[0], g["x_row0"]) and np.array_equal(X[-1], g["x_row_last"])
    for qi, tv, ti in zip(g["qids"], g["truth_scores"], g["truth_ids"]):
        exact = oracle.exact_scores(X, X[qi])
        s, rows = oracle.brute_topk(X, X[qi], 10)
        assert set(rows.tolist()) == set(ti.tolist())
        np.testing.assert_allclose(np.sort(s)[::-1], tv, atol=1e-5)
        oracle.check_topk(exact, 10, tv, ti)


@pytest.mark.parametrize("fixture,circuit,ks", [
    ("ref_small_search.npz", "ref_small.circuit", (1, 5, 10)),
    ("ref_d384_search.npz", "ref_d384.circuit", (10,)),
])
def test_oracle_matches_reference_search_and_seed(fixture, circuit, ks):
    g = np.load(_g(fixture))
    ix = oracle.read_circuit(_g(circuit))
    X = oracle.corpus_from_index(ix)
    for k in ks:
        for qi, q in enumerate(g["queries"]):
            exact = oracle.exact_scores(X, q)
            # reference circuit_search (CPU, flat) == exact top-k
            oracle.check_topk(exact, k, g[f"scores_k{k}"][qi], g[f"ids_k{k}"][qi])
            # C brute force agrees with numpy brute force
            s1, r1 = oracle.brute_topk(X, q, k)
            s2, r2 = oracle.brute_topk_c(X, q, k)
            np.testing.assert_allclose(s1, s2, rtol=0, atol=1e-12)
            # reference _seed_threshold (float32 torch) vs the restatement
            T_ref = float(g[f"seed_k{k}"][qi])
            T32, _ = oracle.seed_threshold(ix, q, k, f64=False)
            T64, _ = oracle.seed_threshold(ix, q, k, f64=True)
            if T_ref == -1e9:
                assert T32 == -1e9 and T64 == -1e9
            else:
                assert abs(T32 - T_ref) < 1e-5 and abs(T64 - T_ref) < 1e-5


@pytest.mark.parametrize("circuit", ["ref_small.circuit", "ref_d384.circuit"])
def test_reference_pipeline_restatement_is_exact(circuit):
    """The reference's hierarchical algorithm (bounds + seed), restated in C,
    returns brute-force results on reference-built indexes."""
    ix = oracle.read_circuit(_g(circuit))
    X = oracle.corpus_from_index(ix)
    rng = np.random.default_rng(5)
    for _ in range(12):
        q = X[rng.integers(0, len(X))]
        s, ids, scored, cmask = oracle.hierarchical_search(ix, q, 10)
        oracle.check_topk(oracle.exact_scores(X, q), 10, s, ids)
        assert 0 < scored <= ix["N"]


def test_bound_restatement_is_an_upper_bound():
    """Every leaf's exact score is <= its child's (reference-formula) bound."""
    ix = oracle.read_circuit(_g("ref_small.circuit"))
    X = oracle.corpus_from_index(ix)
    q = X[17]
    qn = float(np.linalg.norm(q.astype(np.float64)))
    mask, dots = oracle.root_bounds(q, ix["root_centers"], ix["root_radii"], qn, -1e30)
    proj, perp = oracle.project(q, ix["bases"], np.arange(ix["num_roots"]), qn * qn)
    cmask, ub = oracle.child_bounds(proj, perp, dots, ix["child_intervals_l"], ix["child_intervals_u"],
                                    ix["child_radii"], ix["child_parent_ids"], mask, -1e30)
    leaf = ix["leaf_vectors"].astype(np.float64)
    for c in range(ix["num_total_children"]):
        o, n = int(ix["leaf_offsets"][c]), int(ix["leaf_sizes"][c])
        if n:
            assert (leaf[o:o + n] @ q.astype(np.float64)).max() <= ub[c] + 1e-5
    for r in range(ix["num_roots"]):
        assert dots[r] + qn * ix["root_radii"][r] >= -1e30


def test_check_topk_rejects_wrong_answers():
    rng = np.random.default_rng(0)
    exact = rng.normal(size=1000)
    s, rows = np.sort(exact)[::-1][:10], np.argsort(-exact)[:10]
    oracle.check_topk(exact, 10, s, rows)
    bad = rows.copy()
    bad[-1] = np.argsort(-exact)[20]
    with pytest.raises(AssertionError):
        oracle.check_topk(exact, 10, s, bad)
    with pytest.raises(AssertionError):
        oracle.check_topk(exact, 10, s + 1e-3, rows)
    with pytest.raises(AssertionError):
        oracle.check_topk(exact, 10, s[::-1], rows[::-1])


def test_reftest_workload_is_the_reference_test_data():
    """The bench's reftest-40k workload generates the reference test's corpus
    and its query rows (tests/test_exact.py:9-19), pinned to the fixture."""
    import torch
    from circuit_rag.synthetic import WORKLOADS

    g = np.load(_g("ref_test_exact.npz"))
    w = WORKLOADS["reftest-40k"]
    X = w.corpus().numpy()
    assert np.isclose(X.astype(np.float64).sum(), float(g["x_sum"]), rtol=0, atol=1e-6)
    assert np.array_equal(X[0], g["x_row0"]) and np.array_equal(X[-1], g["x_row_last"])
    Q = w.query_batch(25).numpy()
    assert np.array_equal(Q, X[g["qids"]])
    assert torch.equal(w.corpus(1000, 1100), torch.from_numpy(X[1000:1100]))
