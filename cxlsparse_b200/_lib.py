"""ctypes binding of the C ABI in ``include/cxlsparse.h``.

The shared library is built in-tree by ``cxlsparse_b200/build.py``. There is
no fallback: if the library is missing or cannot be loaded, every entry point
raises. Raw device pointers come from torch tensors (``data_ptr()``) and the
stream from ``torch.cuda.current_stream().cuda_stream``.
"""

import ctypes
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libcxlsparse_b200.so"

# Status codes (enum cxs_status).
OK, ERR_INVALID, ERR_CUDA, ERR_CAPACITY, ERR_REGISTRATION, ERR_UNSUPPORTED = range(6)
# Device error word bits.
DEVICE_ERR_READY_TIMEOUT, DEVICE_ERR_COPY_TIMEOUT, DEVICE_ERR_BAD_BLOCK = 1, 2, 4
ORDER_PHYSICAL, ORDER_DEPTH, ORDER_DEPTH_SHARED = 0, 1, 2
READ_ORDERS = {
    "physical": ORDER_PHYSICAL,
    "consumption_depth": ORDER_DEPTH,
    "consumption_depth_shared": ORDER_DEPTH_SHARED,
}

c_i32, c_i64, c_vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p
ABI_VERSION = 4  # CXS_ABI_VERSION
# CXS_NOALLOC_MAX_PHYSICAL: most physical blocks cxs_fetch_attend_noalloc
# takes; its static scratch is 16 bytes per block + 256 (checked against the
# header by tests/test_abi.py and at compile time in attend.cu).
NOALLOC_MAX_PHYSICAL = 16384
NOALLOC_SCRATCH_BYTES = 16 * NOALLOC_MAX_PHYSICAL + 256


class CxsError(RuntimeError):
    """A C-ABI call returned a failure status."""

    def __init__(self, status, message):
        super().__init__(f"cxlsparse_b200 status {status}: {message}")
        self.status = status


class CapacityError(CxsError):
    """Capacity refusal raised before any device work was enqueued."""


class PlanGeometry(ctypes.Structure):
    _fields_ = [(name, c_i32) for name in (
        "queries", "heads", "width", "block_size", "map_blocks", "per_head",
        "sort_extent", "hot", "max_history", "regions", "page_size",
        "consumer_ctas", "read_order", "private_plan", "launch_mode")] + [("pool_tokens", c_i64)]


PLAN_BUFFER_FIELDS = (
    "blocks", "positions", "desc", "bases", "tags", "locs", "host_locs", "hot_data",
    "mapping", "insert_keys", "active_keys", "active_counts", "required", "frequencies",
    "stats", "address", "hbm", "valid", "starts", "flags", "slots", "ioids", "ranks",
    "missing", "all_ids", "all_counts", "row_positions", "region_counts", "row_depth",
    "first_depth", "near_consumers", "chosen", "private_required",
    "private_occurrences", "canonical", "hbm_locs",
)


class PlanBuffers(ctypes.Structure):
    _fields_ = [(name, c_vp) for name in PLAN_BUFFER_FIELDS]


class AttendGeometry(ctypes.Structure):
    _fields_ = [(name, c_i32) for name in (
        "queries", "heads", "width", "block_size", "physical", "window", "window_len",
        "gate")] + [(name, c_i64) for name in (
            "window_start", "spin_limit", "segment_start", "segment_tokens")] + [
        ("out_heads", c_i32), ("out_head0", c_i32), ("ctas", c_i32)]


class SelectGeometry(ctypes.Structure):
    _fields_ = [(name, c_i32) for name in (
        "queries", "heads", "block_size", "count", "summaries", "window", "stride",
        "forced")] + [(name, c_i64) for name in ("total", "segment_start", "segment_tokens")]


ATTEND_BUFFER_FIELDS = (
    "query", "kv", "all_ids", "all_counts", "row_positions", "starts", "valid", "flags",
    "ioids", "missing", "address", "sources", "kinds", "ready", "control", "error",
    "window_kv", "compressed", "gates", "out", "out_peer", "first_depth",
    "near_consumers",
)


class AttendBuffers(ctypes.Structure):
    _fields_ = [(name, c_vp) for name in ATTEND_BUFFER_FIELDS]


_lib = None


def lib():
    """Load the in-tree library once; raise if it is absent (no CPU fallback)."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise ImportError(
                f"{LIBRARY.name} is not built; run `python -m cxlsparse_b200.build` "
                "(the NSA transport has no CPU fallback)")
        handle = ctypes.CDLL(str(LIBRARY))
        sigs = {
            "cxs_abi_version": (c_i32, []),
            "cxs_last_error": (ctypes.c_char_p, []),
            "cxs_launch_count": (c_i64, []),
            "cxs_pool_create": (c_i32, [ctypes.c_size_t, c_i32, c_i32,
                                        ctypes.POINTER(c_vp), ctypes.POINTER(c_i32)]),
            "cxs_pool_destroy": (c_i32, [c_vp, ctypes.c_size_t]),
            "cxs_pool_register": (c_i32, [c_vp, ctypes.c_size_t]),
            "cxs_pool_unregister": (c_i32, [c_vp]),
            "cxs_device_numa_node": (c_i32, [c_i32]),
            "cxs_pool_write": (c_i32, [c_vp, c_vp, c_i64, c_vp, c_i32, c_i32, c_vp]),
            "cxs_plan_check": (c_i32, [ctypes.POINTER(PlanGeometry)]),
            "cxs_plan": (c_i32, [ctypes.POINTER(PlanGeometry), ctypes.POINTER(PlanBuffers),
                                 c_vp]),
            "cxs_plan_core": (c_i32, [ctypes.POINTER(PlanGeometry), ctypes.POINTER(PlanBuffers),
                                      c_vp]),
            "cxs_plan_select_commit_hot": (c_i32, [ctypes.POINTER(PlanGeometry),
                                                   ctypes.POINTER(PlanBuffers), c_vp, c_vp,
                                                   c_vp, c_vp]),
            "cxs_plan_commit_hot": (c_i32, [ctypes.POINTER(PlanGeometry),
                                            ctypes.POINTER(PlanBuffers), c_vp, c_vp, c_vp,
                                            c_vp]),
            "cxs_fetch_attend": (c_i32, [ctypes.POINTER(AttendGeometry),
                                         ctypes.POINTER(AttendBuffers), c_vp]),
            "cxs_attend_capacity": (c_i32, [c_i32, ctypes.POINTER(c_i32)]),
            "cxs_fetch_attend_noalloc": (c_i32, [ctypes.POINTER(AttendGeometry),
                                                 ctypes.POINTER(AttendBuffers), c_vp]),
            "cxs_compressed_select": (c_i32, [c_vp, c_vp, c_i32, c_vp, c_i32, c_i32, c_i32,
                                              c_i32, c_i64, c_vp, c_vp, c_vp, c_vp]),
            "cxs_compressed_select_segments": (c_i32, [c_vp, c_vp, c_i32, c_vp, c_i32, c_i32,
                                                       c_i32, c_i32, c_i64, c_i64, c_i64, c_vp,
                                                       c_vp, c_vp, c_vp]),
            "cxs_compressed_select_nsa": (c_i32, [ctypes.POINTER(SelectGeometry), c_vp, c_vp,
                                                  c_vp, c_vp, c_vp, c_vp, c_vp]),
            "cxs_select_score_columns": (c_i32, [ctypes.POINTER(SelectGeometry),
                                                 ctypes.POINTER(c_i32)]),
            "cxs_block_summaries": (c_i32, [c_vp, c_i64, c_i32, c_i32, c_vp, c_vp]),
            "cxs_block_summaries_segments": (c_i32, [c_vp, c_i64, c_i32, c_i32, c_vp, c_i32,
                                                     c_i64, c_i64, c_vp]),
            "cxs_rms_norm": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_i32, ctypes.c_float, c_vp]),
            "cxs_residual_rms_norm": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, ctypes.c_float,
                                              c_vp]),
            "cxs_qkv_rope": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_i32, c_i32, c_i32, c_vp, c_vp,
                                     c_i32, c_vp, c_i32, c_vp, c_vp]),
            "cxs_qkv_rope_segments": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_i32, c_i32, c_i32,
                                              c_vp, c_vp, c_i32, c_vp, c_i32, c_vp, c_i32,
                                              c_i32, c_vp]),
            "cxs_silu_mul": (c_i32, [c_vp, c_i32, c_i32, c_vp, c_vp]),
            "cxs_compress_windows": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp,
                                             c_vp, c_vp, c_vp, c_vp, c_vp]),
            "cxs_device_alloc": (c_i32, [ctypes.c_size_t, ctypes.POINTER(c_vp)]),
            "cxs_device_free": (c_i32, [c_vp]),
            "cxs_ipc_get_handle": (c_i32, [c_vp, c_vp]),
            "cxs_ipc_open_handle": (c_i32, [c_vp, ctypes.POINTER(c_vp)]),
            "cxs_ipc_close": (c_i32, [c_vp]),
            "cxs_exchange_barrier": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_i32, c_i64, c_vp,
                                             c_vp]),
        }
        for name, (restype, argtypes) in sigs.items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = restype, argtypes
        if handle.cxs_abi_version() != ABI_VERSION:
            raise ImportError("cxlsparse_b200 ABI version mismatch")
        _lib = handle
    return _lib


def check(status):
    """Raise the matching exception for a non-zero status."""
    if status == OK:
        return
    message = lib().cxs_last_error().decode(errors="replace")
    if status == ERR_CAPACITY:
        raise CapacityError(status, message)
    if status == ERR_INVALID:
        raise ValueError(f"cxlsparse_b200: {message}")
    raise CxsError(status, message)


def ptr(tensor):
    """Device address of a tensor, or None for a missing optional buffer."""
    return None if tensor is None else tensor.data_ptr()


def exported_symbols():
    """Names the header declares (used by the CPU symbol test)."""
    return ("cxs_abi_version", "cxs_last_error", "cxs_launch_count", "cxs_pool_create", "cxs_pool_destroy",
            "cxs_pool_register", "cxs_pool_unregister", "cxs_device_numa_node",
            "cxs_pool_write", "cxs_plan_check", "cxs_plan", "cxs_plan_core",
            "cxs_plan_select_commit_hot", "cxs_plan_commit_hot",
            "cxs_fetch_attend", "cxs_attend_capacity", "cxs_fetch_attend_noalloc",
            "cxs_compressed_select", "cxs_compressed_select_segments",
            "cxs_compressed_select_nsa", "cxs_select_score_columns",
            "cxs_block_summaries", "cxs_block_summaries_segments", "cxs_rms_norm",
            "cxs_residual_rms_norm",
            "cxs_qkv_rope", "cxs_qkv_rope_segments", "cxs_silu_mul", "cxs_compress_windows",
            "cxs_device_alloc",
            "cxs_device_free", "cxs_ipc_get_handle", "cxs_ipc_open_handle", "cxs_ipc_close",
            "cxs_exchange_barrier")
