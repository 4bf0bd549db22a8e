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
