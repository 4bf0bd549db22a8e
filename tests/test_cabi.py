"""The C ABI library loads, exports every symbol the public headers declare,
and rejects bad input without touching a GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

from circuit_rag import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


def _declared_functions():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if not h.endswith(".h"):
            continue
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w ]*?[\s\*]+(circuit_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    declared = _declared_functions()
    assert len(declared) >= 18
    L = ctypes.CDLL(_native.LIB_PATH)
    missing = [n for n in sorted(declared) if not hasattr(L, n)]
    assert not missing, missing
    assert set(_native.EXPORTED_SYMBOLS) == declared


def test_abi_version_and_null_handles():
    L = _native.lib()
    assert L.circuit_abi_version() == 2
    # reference convention: -1 for a null index (api.cpp:28-29, :41-42)
    q = np.zeros(8, np.float32)
    s = np.zeros(4, np.float32)
    i = np.zeros(4, np.int32)
    assert L.circuit_search(None, q.ctypes.data, 4, s.ctypes.data, i.ctypes.data, None) == -1
    assert L.circuit_search_device(None, q.ctypes.data, 4, s.ctypes.data, i.ctypes.data, None) == -1
    L.circuit_destroy_index(None)  # no-op


def test_extension_entry_points_reject_null_handles():
    """Every entry point that takes an index handle returns CIRCUIT_ERR_NULL (-1)
    for a null one before any CUDA call (the reference's convention, extended)."""
    L = _native.lib()
    q = np.zeros(8, np.float32)
    s = np.zeros(8, np.float32)
    i = np.zeros(8, np.int32)
    n = ctypes.c_int(0)
    info = (ctypes.c_int64 * 8)()
    tx = _native.TraceEx()
    P = lambda a: a.ctypes.data  # noqa: E731
    assert L.circuit_search_batch(None, P(q), 2, 4, P(s), P(i)) == -1
    assert L.circuit_search_batch_device(None, P(q), 2, 4, P(s), P(i)) == -1
    assert L.circuit_search_batch_async(None, P(q), 2, 4, P(s), P(i), None, None, None) == -1
    assert L.circuit_batch_overflow(None, ctypes.byref(n)) == -1
    assert L.circuit_search_async(None, P(q), 4, 10001, P(s), P(i), None, None, None, None) == -1
    assert L.circuit_search_seed_async(None, P(q), 4, P(s), None) == -1
    assert L.circuit_search_finish_async(None, P(q), 4, P(s), P(s), P(i), None, None, None, None) == -1
    assert L.circuit_index_info(None, info) == -1
    assert L.circuit_last_trace(None, ctypes.byref(tx)) == -1


@pytest.mark.parametrize("mutate,msg", [
    (lambda d: b"XXXXXXXX" + d[8:], "magic"),
    (lambda d: d[:9], "too small"),
    (lambda d: d[:-4096], "outside the file"),
])
def test_loader_rejects_malformed_files_before_any_cuda_call(tmp_path, mutate, msg):
    data = open(os.path.join(GOLDEN, "ref_small.circuit"), "rb").read()
    p = tmp_path / "bad.circuit"
    p.write_bytes(mutate(data))
    L = _native.lib()
    assert not L.circuit_load_index(str(p).encode(), 0)
    assert msg in _native.last_error()


def test_loader_rejects_missing_file():
    L = _native.lib()
    assert not L.circuit_load_index(b"/nonexistent/file.circuit", 0)
    assert "cannot open" in _native.last_error()


def test_loader_rejects_overlapping_children(tmp_path):
    from circuit_rag.storage.format import load_circuit_index

    idx = load_circuit_index(os.path.join(GOLDEN, "ref_small.circuit"), device="cpu")
    idx.leaf_offsets[1] = idx.leaf_offsets[0]  # two children claim the same rows
    p = tmp_path / "overlap.circuit"
    idx.save(str(p))
    assert not _native.lib().circuit_load_index(str(p).encode(), 0)
    err = _native.last_error()
    assert "overlap" in err or "cover" in err


def test_shard_loader_rejects_bad_arguments_before_any_cuda_call(tmp_path):
    """circuit_load_shard validates rank / world and the file before touching a device."""
    import ctypes

    from circuit_rag import _native

    L = _native.lib()
    assert not L.circuit_load_shard(b"/nonexistent.circuit", 0, 2, 0, 1.05)
    assert "cannot open" in _native.last_error()
    assert not L.circuit_load_shard(b"/nonexistent.circuit", 2, 2, 0, 1.05)
    assert "rank" in _native.last_error()
    p = tmp_path / "bad.circuit"
    p.write_bytes(b"NOTCIRC1" + b"\0" * 64)
    assert not L.circuit_load_shard(str(p).encode(), 0, 2, 0, 1.05)
    assert "magic" in _native.last_error()
