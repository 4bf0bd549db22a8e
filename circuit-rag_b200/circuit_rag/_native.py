"""ctypes binding of libcircuit.so (include/circuit.h, circuit_ops.h, circuit_shard.h).

The library is built in-tree next to this file (``make -C circuit-rag_b200/csrc``
or ``__graft_entry__.build()``).  There is no fallback: if the shared library is
missing or fails to load, every search raises :class:`NativeLibraryError`.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcircuit.so")

CIRCUIT_OK = 0
CIRCUIT_MAX_K = 256
CIRCUIT_BATCH_MAX_K = 256
CIRCUIT_BATCH_MAX_DIM = 2048
CIRCUIT_MAX_RANK = 64
CIRCUIT_MAX_DIM = 2048
TRACE_SNAPSHOT_BYTES = 96

# every symbol declared in include/circuit.h and include/circuit_ops.h
EXPORTED_SYMBOLS = (
    "circuit_load_index",
    "circuit_search",
    "circuit_search_device",
    "circuit_destroy_index",
    "circuit_last_error",
    "circuit_abi_version",
    "circuit_index_from_device",
    "circuit_index_info",
    "circuit_search_async",
    "circuit_last_trace",
    "circuit_trace_snapshot_async",
    "circuit_trace_decode",
    "circuit_op_evaluate_root_bounds",
    "circuit_op_project_parents",
    "circuit_op_evaluate_child_bounds",
    "circuit_op_score_surviving_leaves",
    "circuit_op_flat_exact_score",
    "circuit_op_hierarchical_search",
    "circuit_merge_topk",
    "circuit_merge_topk_batch",
    "circuit_plan_shards",
    "circuit_plan_shard_parts",
    "circuit_load_shard",
    "circuit_flat_search_noalloc",
    "circuit_selftest_wait_timeout",
    "circuit_selftest_batch_wait_timeout",
    "circuit_search_seed_async",
    "circuit_search_finish_async",
    "circuit_search_batch_async",
    "circuit_batch_overflow",
    "circuit_search_batch",
    "circuit_search_batch_device",
    "circuit_search_finish_shared_async",
    "circuit_ipc_export",
    "circuit_ipc_import",
    "circuit_ipc_close",
)


class NativeLibraryError(RuntimeError):
    """libcircuit.so is missing, failed to load, or a call returned an error."""


class TraceEx(ctypes.Structure):
    """circuit_trace_ex_t"""

    _fields_ = [
        ("latency_us", ctypes.c_float),
        ("path", ctypes.c_int32),
        ("vectors_scored", ctypes.c_int64),
        ("vectors_total", ctypes.c_int64),
        ("surviving_roots", ctypes.c_int32),
        ("surviving_children", ctypes.c_int32),
        ("total_children", ctypes.c_int32),
        ("best_root", ctypes.c_int32),
        ("seed_threshold", ctypes.c_float),
        ("device_error", ctypes.c_int32),
        ("seed_sample_rows", ctypes.c_int32),
        ("rows_streamed", ctypes.c_int32),
    ]


class Trace(ctypes.Structure):
    """circuit_trace_t (reference native/include/circuit/circuit.h:16-19)"""

    _fields_ = [("latency_us", ctypes.c_float), ("vectors_scored", ctypes.c_int)]


_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float


def _declare(lib):
    sig = {
        "circuit_load_index": (_P, [ctypes.c_char_p, _I]),
        "circuit_search": (_I, [_P, _P, _I, _P, _P, _P]),
        "circuit_search_device": (_I, [_P, _P, _I, _P, _P, _P]),
        "circuit_destroy_index": (None, [_P]),
        "circuit_last_error": (ctypes.c_char_p, []),
        "circuit_abi_version": (_I, []),
        "circuit_index_from_device": (_P, [_I, _I, _I, _I, _I, _I64] + [_P] * 11),
        "circuit_index_info": (_I, [_P, _P]),
        "circuit_search_async": (_I, [_P, _P, _I, _I64, _P, _P, _P, _P, _P, _P]),
        "circuit_last_trace": (_I, [_P, _P]),
        "circuit_trace_snapshot_async": (_I, [_P, _P, _P]),
        "circuit_trace_decode": (_I, [_P, _P, _I, _P]),
        "circuit_op_evaluate_root_bounds": (_I, [_P, _P, _P, _F, _F, _I, _I, _P, _P, _P, _P, _P]),
        "circuit_op_project_parents": (_I, [_P, _P, _P, _I, _I, _I, _I, _F, _P, _P, _P]),
        "circuit_op_evaluate_child_bounds": (_I, [_P] * 8 + [_F, _I, _I, _P, _P, _P, _P]),
        "circuit_op_score_surviving_leaves": (_I, [_P, _P, _P, _P, _P, _I, _I64, _I, _P, _P]),
        "circuit_op_flat_exact_score": (_I, [_P, _P, _I64, _I, _P, _P]),
        "circuit_op_hierarchical_search": (_I, [_P] * 21 + [_I, _I, _I64, _I, _F, _I, _F, _P]),
        "circuit_merge_topk": (_I, [_P, _P, _I, _I, _P, _P, _P]),
        "circuit_merge_topk_batch": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P]),
        "circuit_plan_shards": (_I, [_P, _I, _I, _P, _P]),
        "circuit_plan_shard_parts": (_I, [_P, _P, _I, _I, ctypes.c_double, _P, _P, _P, _P, _I, _P, _P]),
        "circuit_load_shard": (_P, [ctypes.c_char_p, _I, _I, _I, ctypes.c_double]),
        "circuit_flat_search_noalloc": (_I, [_P, _I64, _I, _P, _I, _P, _P, _P]),
        "circuit_search_batch_async": (_I, [_P, _P, _I, _I, _P, _P, _P, _P, _P]),
        "circuit_search_seed_async": (_I, [_P, _P, _I, _P, _P]),
        "circuit_selftest_wait_timeout": (_I, [_I, _P]),
        "circuit_selftest_batch_wait_timeout": (_I, [_P, _P]),
        "circuit_search_finish_async": (_I, [_P, _P, _I, _P, _P, _P, _P, _P, _P, _P]),
        "circuit_batch_overflow": (_I, [_P, _P]),
        "circuit_search_batch": (_I, [_P, _P, _I, _I, _P, _P]),
        "circuit_search_batch_device": (_I, [_P, _P, _I, _I, _P, _P]),
        "circuit_search_finish_shared_async": (_I, [_P, _P, _I, _P, _P, _P, _I, ctypes.c_uint32, _P, _P, _P, _P, _P,
                                                    _P]),
        "circuit_ipc_export": (_I, [_P, _P, _P]),
        "circuit_ipc_import": (_I, [_P, _I, _P]),
        "circuit_ipc_close": (_I, [_P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def lib():
    """The loaded library (loads it on first use; raises NativeLibraryError)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryError(
                f"{LIB_PATH} is missing: build it with `make -C circuit-rag_b200/csrc` "
                "(or __graft_entry__.build()); circuit-b200 has no CPU fallback"
            )
        try:
            handle = ctypes.CDLL(LIB_PATH)
        except OSError as e:  # pragma: no cover - depends on the host
            raise NativeLibraryError(f"cannot load {LIB_PATH}: {e}") from e
        _declare(handle)
        _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().circuit_last_error()
    return msg.decode("utf-8", "replace") if msg else ""


def check(rc: int, what: str) -> None:
    if rc != CIRCUIT_OK:
        raise NativeLibraryError(f"{what} failed ({rc}): {last_error()}")
