"""The reference's own native search library, compiled unchanged for sm_100a
(oracle/_ref/libcircuit_ref.so from reference native/src/gpu_index.cpp,
api.cpp and its kernels), against this repository's libcircuit.so: same
.circuit files, same queries, one process, one GPU (oracle/native_compare.cpp).

Both libraries' results must pass the float64 oracle and agree with each other
(ids identical except among scores tied within 1e-6).  The timings (host
buffers and device buffers, circuit_bench's method) are printed as one table
row per workload; run with -s to see them.  Skipped when the reference build is
absent (it is built from a reference checkout by `make -C oracle ref`)."""
import json
import os
import subprocess

import numpy as np
import pytest
import torch

from circuit_rag import _native, build_circuit_index
from circuit_rag.synthetic import WORKLOADS
from oracle import oracle

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libcircuit_ref.so")
HARNESS = os.path.join(ROOT, "oracle", "_ref", "native_compare")
DEV = "cuda"


@pytest.mark.skipif(not (os.path.exists(REF_SO) and os.path.exists(HARNESS)), reason="reference build absent")
@pytest.mark.parametrize("name", ["spread-5k", "clustered-50k", "spread-200k"])
def test_native_library_against_the_reference_library(tmp_path, name):
    w = WORKLOADS[name]
    X = w.corpus(0, w.n, device=DEV)
    idx = build_circuit_index(X, num_roots=w.num_roots, children_per_root=w.children_per_root, rank=w.rank,
                              device=DEV)
    path = str(tmp_path / f"{name}.circuit")
    idx.save(path)
    idx.close()
    nq, k = 1000, w.k  # the reference clamps k to 32 (gpu_index.cpp:243)
    Q = w.query_batch(nq).numpy().astype(np.float32)
    qpath = str(tmp_path / "q.f32")
    Q.tofile(qpath)
    out = str(tmp_path / "res")
    p = subprocess.run([HARNESS, _native.LIB_PATH, REF_SO, path, qpath, str(nq), str(w.dim), str(k), out],
                       capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr
    # the reference library prints its own progress lines to stdout as well
    rows = {json.loads(line)["lib"]: json.loads(line) for line in p.stdout.splitlines() if line.startswith('{"lib"')}
    res = {}
    for lib in ("ours", "reference"):
        s = np.fromfile(f"{out}.{lib}.scores", np.float32).reshape(nq, k)
        i = np.fromfile(f"{out}.{lib}.ids", np.int32).reshape(nq, k)
        res[lib] = (s, i)
    Xc = X.double()
    Qd = torch.from_numpy(Q).to(DEV).double()
    bad = {"ours": 0, "reference": 0}
    disagree = 0
    for a in range(0, nq, 100):
        exact = (Qd[a:a + 100] @ Xc.T).cpu().numpy()
        for b in range(exact.shape[0]):
            for lib in ("ours", "reference"):
                s, i = res[lib]
                try:
                    oracle.check_topk(exact[b], k, s[a + b], i[a + b])
                except AssertionError:
                    bad[lib] += 1
            si, ii = res["ours"][1][a + b], res["reference"][1][a + b]
            if set(si.tolist()) != set(ii.tolist()):
                kth = np.sort(exact[b])[-k]
                diff = set(si.tolist()) ^ set(ii.tolist())
                if any(abs(exact[b][j] - kth) > oracle.TIE_ABS for j in diff):
                    disagree += 1
    o, r = rows["ours"], rows["reference"]
    print(f"\n[native] {name} N={w.n} D={w.dim} k={k} | host p50/p99 us: ours {o['host_p50_us']:.1f}/"
          f"{o['host_p99_us']:.1f}, reference {r['host_p50_us']:.1f}/{r['host_p99_us']:.1f} | device-buffer "
          f"p50 us: ours {o['dev_p50_us']:.1f}, reference {r['dev_p50_us']:.1f} | q/s host: ours "
          f"{o['host_qps']:.0f}, reference {r['host_qps']:.0f} | load ms: ours {o['load_ms']:.1f}, reference "
          f"{r['load_ms']:.1f} | oracle misses: ours {bad['ours']}, reference {bad['reference']} of {nq}")
    assert bad["ours"] == 0
    assert disagree <= bad["reference"]  # any disagreement is the reference missing the oracle, never ours
