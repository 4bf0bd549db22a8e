"""Generate the golden fixtures under tests/golden/ by running the REFERENCE package.

Run from the repository root, in a container where the reference checkout is
mounted, with that checkout on PYTHONPATH (this script is the only committed
file that imports it):

    PYTHONPATH=$CIRCUIT_REF_DIR python tests/golden/make_golden.py

What it pins (all produced by the reference's own code, on CPU):

* ``ref_small.circuit``      -- an index built by the reference CPU builder
  (``circuit_rag/hierarchy/build.py:256-387``) and written by the reference
  writer (``circuit_rag/storage/format.py:13-80``).  Pins the byte layout of the
  ``.circuit`` format: our loader must read it and our writer must reproduce it
  byte for byte.
* ``ref_small_search.npz``   -- the reference ``circuit_search`` results
  (``circuit_rag/search.py:45-84``; flat path on CPU) and the reference
  ``_seed_threshold`` values (``search.py:26-41``) for seeded queries against
  that index, for k = 1, 5, 10.
* ``ref_test_exact.npz``     -- the data generator of ``tests/test_exact.py:9-14``
  (checksums of X) and the brute-force truth of ``tests/test_exact.py:17-28``
  (25 queries, k = 10).
* ``ref_d384.circuit`` / ``ref_d384_search.npz`` -- a D=384 spread-corpus index
  (the shape regime of the SciFact stand-in) built and searched by the reference.

The corpus X of each index is recoverable from the index itself
(``leaf_vectors[argsort(original_ids)]``).  The fixtures are small (about 2.5 MB) and are committed together with this script.
"""
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _require_reference():
    import circuit_rag  # noqa: F401  (must be the reference package)
    src = os.path.abspath(circuit_rag.__file__)
    if "reference" not in src:
        sys.exit(f"make_golden.py must import the reference package, got {src}")
    return circuit_rag


def clustered_like_reference_test(n=40000, dim=128, clusters=64, seed=0):
    """Restates tests/test_exact.py:9-14 (Gaussian centres, noise 0.3, renormalised)."""
    rng = np.random.default_rng(seed)
    centers = rng.normal(size=(clusters, dim))
    X = centers[rng.integers(0, clusters, n)] + 0.3 * rng.normal(size=(n, dim))
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    return X.astype(np.float32)


def spread_unit(n, dim, seed):
    """Anisotropic spread corpus with a shared mean direction (per-dim std ~ i^-0.5)."""
    rng = np.random.default_rng(seed)
    std = 1.0 / np.sqrt(np.arange(1, dim + 1))
    noise = rng.normal(size=(n, dim)) * std
    noise *= 0.6 / np.linalg.norm(noise, axis=1, keepdims=True)
    mean = rng.normal(size=dim)
    mean *= 0.6 / np.linalg.norm(mean)
    X = noise + mean
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    return X.astype(np.float32)


def search_fixture(circuit_rag, index, X, query_rows, extra_queries, ks):
    from circuit_rag.search import _seed_threshold

    Q = np.concatenate([X[query_rows], extra_queries]).astype(np.float32)
    out = {"queries": Q, "ks": np.array(ks, dtype=np.int32)}
    for k in ks:
        S, I, T = [], [], []
        for q in Q:
            qt = torch.from_numpy(q.copy())
            scores, ids, trace = circuit_rag.circuit_search(qt, index, k=k)
            assert trace.path == "flat"
            S.append(scores.numpy())
            I.append(ids.numpy().astype(np.int32))
            T.append(_seed_threshold(qt, index, k))
        out[f"scores_k{k}"] = np.stack(S).astype(np.float32)
        out[f"ids_k{k}"] = np.stack(I).astype(np.int32)
        out[f"seed_k{k}"] = np.array(T, dtype=np.float64)
    return out


def main():
    circuit_rag = _require_reference()
    torch.manual_seed(0)
    manifest = {}

    # 1. small clustered index built + saved by the reference (format + seed + search pins)
    X = clustered_like_reference_test(n=3000, dim=32, clusters=16, seed=0)
    idx = circuit_rag.build_circuit_index(X, num_roots=8, children_per_root=4, rank=4, device="cpu")
    path = os.path.join(HERE, "ref_small.circuit")
    idx.save(path)
    rng = np.random.default_rng(7)
    rows = rng.integers(0, len(X), 12)
    extra = rng.normal(size=(4, X.shape[1]))
    extra /= np.linalg.norm(extra, axis=1, keepdims=True)
    fx = search_fixture(circuit_rag, idx, X, rows, extra, ks=[1, 5, 10])
    np.savez_compressed(os.path.join(HERE, "ref_small_search.npz"), **fx)

    # 2. the reference test's own data + brute-force truth (tests/test_exact.py)
    Xt = clustered_like_reference_test()
    corpus = torch.from_numpy(Xt)
    rng = np.random.default_rng(1)
    qids = rng.integers(0, len(Xt), 25)
    tv, ti = [], []
    for qi in qids:
        truth = torch.topk(corpus @ corpus[qi], 10)
        tv.append(truth.values.numpy())
        ti.append(truth.indices.numpy().astype(np.int32))
    np.savez_compressed(
        os.path.join(HERE, "ref_test_exact.npz"),
        qids=qids.astype(np.int64),
        truth_scores=np.stack(tv).astype(np.float32),
        truth_ids=np.stack(ti).astype(np.int32),
        x_sum=np.float64(Xt.astype(np.float64).sum()),
        x_row0=Xt[0],
        x_row_last=Xt[-1],
    )

    # 3. D=384 spread index (SciFact-shape regime), reference-built and searched
    X3 = spread_unit(1200, 384, seed=3)
    idx3 = circuit_rag.build_circuit_index(X3, num_roots=8, children_per_root=4, rank=8, device="cpu")
    path3 = os.path.join(HERE, "ref_d384.circuit")
    idx3.save(path3)
    rng = np.random.default_rng(11)
    rows3 = rng.integers(0, len(X3), 6)
    extra3 = spread_unit(2, 384, seed=12)
    fx3 = search_fixture(circuit_rag, idx3, X3, rows3, extra3, ks=[10])
    np.savez_compressed(os.path.join(HERE, "ref_d384_search.npz"), **fx3)

    for name in sorted(os.listdir(HERE)):
        if name.endswith((".circuit", ".npz")):
            with open(os.path.join(HERE, name), "rb") as f:
                manifest[name] = hashlib.sha256(f.read()).hexdigest()
    with open(os.path.join(HERE, "MANIFEST.json"), "w") as f:
        json.dump({"generated_by": "tests/golden/make_golden.py", "sha256": manifest}, f, indent=1)
    print(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    main()
