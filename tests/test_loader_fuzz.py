"""The native .circuit loaders against corrupted files (CPU): child tables with
out-of-range parent ids, offsets and sizes, header integers and tensor_meta
entries with hostile values, random header bytes, truncations and bad header
lengths.  Each corrupted file goes to circuit_load_index and to
circuit_load_shard; every call must return (a handle or NULL with an error
message) and none may crash.  The loaders run in a child process, so a crash
fails this test instead of ending the session."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


@pytest.mark.parametrize("fixture,seed", [("ref_small.circuit", 1), ("ref_d384.circuit", 2)])
def test_loaders_survive_corrupted_files(tmp_path, fixture, seed):
    worker = os.path.join(ROOT, "tests", "loader_fuzz_worker.py")
    out = subprocess.run([sys.executable, worker, ROOT, os.path.join(GOLDEN, fixture), str(tmp_path), "240",
                          str(seed)], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, (out.returncode, out.stderr[-2000:])
    res = json.loads(out.stdout.strip().splitlines()[-1])
    assert res["tried"] >= 400, res
    assert res["tried"] == res["rejected"] + res["loaded"], res
    assert not res["unexplained"], res  # every rejection says why


@pytest.mark.parametrize("fixture,seed", [("ref_small.circuit", 3), ("ref_d384.circuit", 4)])
def test_python_loaders_agree_with_the_native_checks(tmp_path, fixture, seed):
    """The Python loaders (load_circuit_index, load_shard) reject exactly the
    corrupted files that the native loader rejects before any CUDA call, with
    CircuitFormatError and never another exception; the others load."""
    import ctypes

    import numpy as np

    from circuit_rag import _native
    from circuit_rag.shard import load_shard
    from circuit_rag.storage.format import CircuitFormatError, load_circuit_index

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import loader_fuzz_worker as W

    data = open(os.path.join(GOLDEN, fixture), "rb").read()
    L = _native.lib()
    path = str(tmp_path / "f.circuit")
    n_valid = n_bad = 0
    for kind, blob in W.mutants(data, np.random.default_rng(seed), 120):
        with open(path, "wb") as f:
            f.write(blob)
        h = L.circuit_load_index(path.encode(), 0)
        if h:  # a GPU is present and the file is valid
            L.circuit_destroy_index(h)
            native_ok = True
        else:
            native_ok = "cudaSetDevice" in _native.last_error() or "CUDA" in _native.last_error()
        for load in (lambda: load_circuit_index(path, device="cpu"),
                     lambda: load_circuit_index(path, device="cpu", use_mmap=False),
                     lambda: load_shard(path, 0, 2, device="cpu")):
            try:
                load()
                ok = True
            except CircuitFormatError:
                ok = False
            except ValueError as e:  # load_shard: a rank with no rows is a valid refusal of a valid file
                assert "owns no rows" in str(e), (kind, e)
                ok = True
            assert ok == native_ok, (kind, native_ok, _native.last_error())
        n_valid += native_ok
        n_bad += not native_ok
    assert n_valid > 0 and n_bad > 0, (n_valid, n_bad)
