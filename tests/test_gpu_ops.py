"""GPU parity of the per-stage `circuit_cuda` ops (reference torch extension
semantics) against the oracle's restatement of the reference formulas, and --
when oracle/_ref/libcircuit_ref.so was built from the reference sources --
against the reference's own kernels on the same inputs."""
import ctypes
import os

import numpy as np
import pytest
import torch

import circuit_cuda
from circuit_rag import CircuitIndex, build_circuit_index
from circuit_rag.synthetic import WORKLOADS
from oracle import oracle

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libcircuit_ref.so")
DEV = "cuda"
NEAR = 1e-4  # masks may differ only where a bound is this close to the threshold


@pytest.fixture(scope="module")
def setup():
    w = WORKLOADS["clustered-50k"]
    X = w.corpus(0, 20000, device=DEV)
    idx = build_circuit_index(X, num_roots=32, children_per_root=8, rank=8, device=DEV)
    ix = {k: getattr(idx, k).cpu().numpy() for k in oracle.TENSORS}
    ix.update(dim=idx.dim, rank=idx.rank, num_roots=idx.num_roots, num_total_children=idx.num_total_children,
              N=idx.N)
    qs = w.query_batch(6, device=DEV)
    return idx, ix, qs


def _masks_agree(got, want, margin_vals, thr):
    diff = np.nonzero(got != want)[0]
    assert all(abs(margin_vals[d] - thr) < NEAR for d in diff), diff[:10]


def test_root_project_child_ops(setup):
    idx, ix, qs = setup
    for q in qs:
        qn = q.cpu().numpy()
        qnorm = float(np.linalg.norm(qn.astype(np.float64)))
        T, _ = oracle.seed_threshold(ix, qn, 10, f64=True)
        mask, sidx, cnt, dots = circuit_cuda.evaluate_root_bounds(q, idx.root_centers, idx.root_radii, T, qnorm)
        om, od = oracle.root_bounds(qn, ix["root_centers"], ix["root_radii"], qnorm, T)
        np.testing.assert_allclose(dots.cpu().numpy(), od, atol=1e-5)
        _masks_agree(mask.cpu().numpy(), om, od + qnorm * ix["root_radii"], T)
        n = int(cnt.item())
        assert sorted(sidx[:n].tolist()) == sorted(np.nonzero(mask.cpu().numpy())[0].tolist())
        proj, perp = circuit_cuda.project_parents(q, idx.bases, sidx, n, idx.rank, qnorm * qnorm)
        op, opp = oracle.project(qn, ix["bases"], sidx[:n].cpu().numpy(), qnorm * qnorm)
        np.testing.assert_allclose(proj.cpu().numpy(), op, atol=1e-5)
        np.testing.assert_allclose(perp.cpu().numpy(), opp, atol=2e-3)  # sqrt of a cancellation-prone difference
        cm, cidx, ccnt = circuit_cuda.evaluate_child_bounds(proj, perp, dots, idx.child_intervals_l,
                                                            idx.child_intervals_u, idx.child_radii,
                                                            idx.child_parent_ids, mask, T, idx.rank)
        ocm, oub = oracle.child_bounds(op, opp, od, ix["child_intervals_l"], ix["child_intervals_u"],
                                       ix["child_radii"], ix["child_parent_ids"], mask.cpu().numpy(), T)
        _masks_agree(cm.cpu().numpy(), ocm, oub, T)
        # scoring surviving leaves, then top-k = exact top-k (the reference pipeline is exact)
        nc = int(ccnt.item())
        (vs,) = circuit_cuda.score_surviving_leaves(q, idx.leaf_vectors, idx.leaf_offsets, idx.leaf_sizes, cidx, nc)
        vs = vs.cpu().numpy()
        surv_rows = np.zeros(idx.N, bool)
        for c in cidx[:nc].tolist():
            surv_rows[ix["leaf_offsets"][c]:ix["leaf_offsets"][c] + ix["leaf_sizes"][c]] = True
        assert np.all(vs[~surv_rows] == np.float32(-1e9))
        exact_rows = ix["leaf_vectors"].astype(np.float64) @ qn.astype(np.float64)
        np.testing.assert_allclose(vs[surv_rows], exact_rows[surv_rows], atol=1e-5)
        top = np.argsort(-vs, kind="stable")[:10]
        X = oracle.corpus_from_index(ix)
        oracle.check_topk(oracle.exact_scores(X, qn), 10, vs[top], ix["original_ids"][top])


def test_flat_and_hierarchical_ops(setup):
    idx, ix, qs = setup
    X = oracle.corpus_from_index(ix)
    for q in qs[:3]:
        qn = q.cpu().numpy()
        s = circuit_cuda.flat_exact_score(q, idx.leaf_vectors).cpu().numpy()
        np.testing.assert_allclose(s, ix["leaf_vectors"].astype(np.float64) @ qn.astype(np.float64), atol=1e-5)
        qnorm = float(np.linalg.norm(qn.astype(np.float64)))
        T, _ = oracle.seed_threshold(ix, qn, 10, f64=False)
        vs = circuit_cuda.hierarchical_search(
            q, idx.root_centers, idx.root_radii, idx.bases, idx.child_intervals_l, idx.child_intervals_u,
            idx.child_radii, idx.child_parent_ids, idx.leaf_vectors, idx.leaf_offsets, idx.leaf_sizes,
            idx.ws_survivor_mask, idx.ws_survivor_indices, idx.ws_num_survivors, idx.ws_root_dot_products,
            idx.ws_projected_queries, idx.ws_perp_norms, idx.ws_child_survivor_mask, idx.ws_child_survivor_indices,
            idx.ws_num_child_survivors, idx.ws_vector_scores, T, idx.rank, qnorm)
        top = torch.topk(vs, 10)
        oracle.check_topk(oracle.exact_scores(X, qn), 10, top.values.cpu().numpy(),
                          idx.original_ids[top.indices].cpu().numpy())
        assert int(idx.ws_num_child_survivors.item()) < idx.num_total_children  # it pruned


def test_ops_reject_cpu_tensors(setup):
    idx, _, _ = setup
    with pytest.raises(RuntimeError, match="CUDA"):
        circuit_cuda.flat_exact_score(torch.zeros(128), idx.leaf_vectors)


def test_rank_above_32_projection(setup):
    """The reference cannot launch rank > 32 (README.md:114); ours handles up to 64."""
    X = WORKLOADS["spread-5k"].corpus(0, 3000, device=DEV)
    idx = build_circuit_index(X, num_roots=4, children_per_root=2, rank=48, device=DEV)
    q = X[11]
    qn = q.cpu().numpy()
    allr = torch.arange(4, dtype=torch.int32, device=DEV)
    proj, perp = circuit_cuda.project_parents(q, idx.bases, allr, 4, 48, 1.0)
    op, opp = oracle.project(qn, idx.bases.cpu().numpy(), np.arange(4), 1.0)
    np.testing.assert_allclose(proj.cpu().numpy(), op, atol=1e-5)


# ------------------------------------------------------------------ reference kernels, same inputs
@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libcircuit_ref.so not built (no reference checkout at build time)")
    L = ctypes.CDLL(REF_LIB)
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    L.ref_root_bounds.argtypes = [P, P, P, F, F, I, I, P, P, P, P]
    L.ref_project.argtypes = [P, F, P, P, I, I, I, P, P]
    L.ref_child_bounds.argtypes = [P, P, P, P, P, P, P, P, F, I, I, P, P, P]
    L.ref_flat_score.argtypes = [P, P, I, I, P]
    L.ref_select_topk.argtypes = [P, P, I, I, P, P]
    return L


def test_ops_match_reference_kernels(setup, ref):
    idx, ix, qs = setup
    torch.cuda.synchronize()
    R, C, D, r = idx.num_roots, idx.num_total_children, idx.dim, idx.rank
    for q in qs[:3]:
        qn = q.cpu().numpy()
        qnorm = float(np.linalg.norm(qn.astype(np.float64)))
        T, _ = oracle.seed_threshold(ix, qn, 10, f64=False)
        mask, sidx, cnt, dots = circuit_cuda.evaluate_root_bounds(q, idx.root_centers, idx.root_radii, T, qnorm)
        torch.cuda.synchronize()
        rm = torch.zeros(R, dtype=torch.int32, device=DEV)
        ri = torch.zeros(R, dtype=torch.int32, device=DEV)
        rc = torch.zeros(1, dtype=torch.int32, device=DEV)
        rd = torch.zeros(R, device=DEV)
        assert ref.ref_root_bounds(q.data_ptr(), idx.root_centers.data_ptr(), idx.root_radii.data_ptr(), qnorm, T,
                                   R, D, rm.data_ptr(), ri.data_ptr(), rc.data_ptr(), rd.data_ptr()) == 0
        np.testing.assert_allclose(dots.cpu().numpy(), rd.cpu().numpy(), atol=1e-5)
        _masks_agree(mask.cpu().numpy(), rm.cpu().numpy(), rd.cpu().numpy() + qnorm * ix["root_radii"], T)
        n = int(rc.item())
        proj, perp = circuit_cuda.project_parents(q, idx.bases, ri, n, r, qnorm * qnorm)
        torch.cuda.synchronize()
        rp = torch.zeros(R, r, device=DEV)
        rpp = torch.zeros(R, device=DEV)
        assert ref.ref_project(q.data_ptr(), qnorm * qnorm, idx.bases.data_ptr(), ri.data_ptr(), n, D, r,
                               rp.data_ptr(), rpp.data_ptr()) == 0
        np.testing.assert_allclose(proj.cpu().numpy(), rp.cpu().numpy(), atol=1e-5)
        np.testing.assert_allclose(perp.cpu().numpy(), rpp.cpu().numpy(), atol=2e-3)
        cm, _, _ = circuit_cuda.evaluate_child_bounds(proj, perp, dots, idx.child_intervals_l, idx.child_intervals_u,
                                                      idx.child_radii, idx.child_parent_ids, mask, T, r)
        torch.cuda.synchronize()
        rcm = torch.zeros(C, dtype=torch.int32, device=DEV)
        rci = torch.zeros(C, dtype=torch.int32, device=DEV)
        rcc = torch.zeros(1, dtype=torch.int32, device=DEV)
        assert ref.ref_child_bounds(rp.data_ptr(), rpp.data_ptr(), rd.data_ptr(), idx.child_intervals_l.data_ptr(),
                                    idx.child_intervals_u.data_ptr(), idx.child_radii.data_ptr(),
                                    idx.child_parent_ids.data_ptr(), rm.data_ptr(), T, C, r, rcm.data_ptr(),
                                    rci.data_ptr(), rcc.data_ptr()) == 0
        _, oub = oracle.child_bounds(rp.cpu().numpy().astype(np.float64), rpp.cpu().numpy().astype(np.float64),
                                     rd.cpu().numpy().astype(np.float64), ix["child_intervals_l"],
                                     ix["child_intervals_u"], ix["child_radii"], ix["child_parent_ids"],
                                     rm.cpu().numpy(), T)
        _masks_agree(cm.cpu().numpy(), rcm.cpu().numpy(), oub, T)
        fs = torch.zeros(idx.N, device=DEV)
        assert ref.ref_flat_score(q.data_ptr(), idx.leaf_vectors.data_ptr(), idx.N, D, fs.data_ptr()) == 0
        ours = circuit_cuda.flat_exact_score(q, idx.leaf_vectors)
        np.testing.assert_allclose(ours.cpu().numpy(), fs.cpu().numpy(), atol=1e-5)
