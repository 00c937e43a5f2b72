"""ctypes binding of ``libpaged_decode_b200.so`` (the C ABI in include/paged_decode.h).

The library is built in-tree by ``paged-decode-lab_b200/build.py``.  Loading
fails loudly when it is missing: there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_NAME = "libpaged_decode_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

PD_OK, PD_ERR_VALUE, PD_ERR_TYPE, PD_ERR_CUDA, PD_ERR_DEVICE, PD_ERR_UNBOUND = range(6)
PD_FLOAT16, PD_FLOAT32 = 0, 1
PD_DEVERR_TIMEOUT, PD_DEVERR_BAD_PAGE = 1, 2
PD_BARRIER_PLAIN, PD_BARRIER_COOPERATIVE, PD_BARRIER_LEAVE_AT_ONCE = 0, 1, 2
PD_ENGINE_WARP, PD_ENGINE_TCGEN05 = 0, 1

# Every function the header declares, with its ctypes signature.
_c_int32, _c_int64, _c_size, _vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p


class Layout(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("query_heads", ctypes.c_int32),
                ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("page_size", ctypes.c_int32), ("physical_pages", ctypes.c_int64)]


class PlanInfo(ctypes.Structure):
    _fields_ = [("splits", ctypes.c_int32), ("max_context", ctypes.c_int32),
                ("num_ctas", ctypes.c_int32), ("num_segments", ctypes.c_int32),
                ("num_groups", ctypes.c_int32), ("num_pieces", ctypes.c_int32),
                ("slot_stride", ctypes.c_int32),
                ("group_tile", ctypes.c_int32), ("heads_per_tile", ctypes.c_int32),
                ("total_pages", ctypes.c_int32),
                ("merge_rows", ctypes.c_int32), ("merge_in_kernel", ctypes.c_int32),
                ("dynamic", ctypes.c_int32), ("max_span", ctypes.c_int32),
                ("workspace_bytes", ctypes.c_int64), ("device_bytes", ctypes.c_int64),
                ("engine", ctypes.c_int32), ("cluster_ctas", ctypes.c_int32)]


SIGNATURES = {
    "pd_plan_create": (_c_int32, [ctypes.POINTER(Layout), _vp, _c_int64, _vp, _c_int32, _c_int32,
                                  _c_int32, _c_int32, _c_int32, ctypes.POINTER(_vp)]),
    "pd_plan_create_dynamic": (_c_int32, [ctypes.POINTER(Layout), _vp, _c_int64, _vp, _vp, _c_int32,
                                          _c_int32, _c_int32, _c_int32, _c_int32, ctypes.POINTER(_vp)]),
    "pd_plan_destroy": (None, [_vp]),
    "pd_plan_get_info": (_c_int32, [_vp, ctypes.POINTER(PlanInfo)]),
    "pd_plan_copy_worklist": (_c_int32, [_vp, _vp, _vp, _vp]),
    "pd_plan_device_bytes": (_c_size, [_vp]),
    "pd_plan_bind": (_c_int32, [_vp, _vp, _c_size, _vp]),
    "pd_plan_metadata_bytes": (_c_size, [_vp]),
    "pd_plan_workspace_bytes": (_c_size, [_vp]),
    "pd_plan_bind_split": (_c_int32, [_vp, _vp, _c_size, _vp, _c_size, _vp]),
    "pd_decode": (_c_int32, [_vp, _vp, _vp, _vp, _c_int32, _vp, _vp]),
    "pd_decode_dynamic": (_c_int32, [_vp, _vp, _vp, _vp, _c_int32, _vp, _vp, _vp, _vp, _vp]),
    "pd_exchange_bytes": (_c_size, [_vp, _c_int32]),
    "pd_exchange_alloc": (_c_int32, [_c_int32, _c_size, ctypes.POINTER(_vp), _vp]),
    "pd_exchange_open": (_c_int32, [_c_int32, _vp, ctypes.POINTER(_vp)]),
    "pd_exchange_close": (_c_int32, [_c_int32, _vp]),
    "pd_exchange_free": (_c_int32, [_c_int32, _vp]),
    "pd_decode_exchange": (_c_int32, [_vp, _vp, _vp, _vp, _c_int32, _vp, _c_int32, _c_int32, _vp, _vp, _vp]),
    "pd_decode_with_stats": (_c_int32, [_vp, _vp, _vp, _vp, _c_int32, _vp, _vp, _vp]),
    "pd_merge_shards": (_c_int32, [_vp, _vp, _c_int32, _c_int64, _c_int64, _c_int32, _vp, _vp]),
    "pd_gather_debug": (_c_int32, [_vp, _vp, _vp, _c_int32, _vp, _vp, _vp]),
    "pd_plan_read_errors": (_c_int32, [_vp, ctypes.POINTER(ctypes.c_uint32), _vp]),
    "pd_plan_set_barrier": (_c_int32, [_vp, _c_int32]),
    "pd_plan_read_barrier_fallbacks": (_c_int32, [_vp, ctypes.POINTER(ctypes.c_uint32), _vp]),
    "pd_decode_static": (_c_int32, [_vp, _vp, _vp, _vp, _c_int32, _vp, _vp]),
    "pd_static_scratch_capacity": (_c_size, []),
    "pd_static_read_errors": (_c_int32, [_c_int32, ctypes.POINTER(ctypes.c_uint32), _vp]),
    "pd_status_string": (ctypes.c_char_p, [_c_int32]),
    "pd_last_error": (ctypes.c_char_p, []),
    "pd_abi_version": (_c_int32, []),
    "pd_selftest_wait_timeouts": (_c_int32, [_c_int32, ctypes.c_uint32, _vp]),
    "pd_selftest_barrier_leave": (_c_int32, [_c_int32, ctypes.c_uint32, _vp]),
}

_lib = None


def load():
    """Load the native library (once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_NAME} is not built; run `python paged-decode-lab_b200/build.py` "
                "(nvcc, sm_100a). There is no CPU fallback.")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if lib.pd_abi_version() != 8:
            raise RuntimeError("paged_decode native ABI version mismatch")
        _lib = lib
    return _lib


def check(status: int, what: str = "") -> None:
    """Map a pd_status to the reference's Python exception types."""
    if status == PD_OK:
        return
    msg = (load().pd_last_error() or b"").decode(errors="replace")
    if what:
        msg = f"{what}: {msg}"
    if status == PD_ERR_VALUE:
        raise ValueError(msg)
    if status == PD_ERR_TYPE:
        raise TypeError(msg)
    raise RuntimeError(msg)
