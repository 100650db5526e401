"""ctypes binding of libproxima_b200.so (the C ABI in include/px.h).

Loading never falls back to anything else: if the library is missing or was
built for another architecture, the import error says so and the caller
fails. ctypes drops the GIL for the duration of every foreign call, which is
what the reference's PyO3 layer does with ``py.allow_threads``.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libproxima_b200.so")

PX_OK = 0
PX_EINVAL = 1
PX_ECUDA = 2
PX_ENOMEM = 3
PX_ESTATE = 4
PX_ENCCL = 5
PX_ETIMEOUT = 6
PX_EUNSUPPORTED = 7
PX_MAX_K = 768

_STATUS_NAMES = {
    PX_EINVAL: "EINVAL", PX_ECUDA: "ECUDA", PX_ENOMEM: "ENOMEM", PX_ESTATE: "ESTATE",
    PX_ENCCL: "ENCCL", PX_ETIMEOUT: "ETIMEOUT", PX_EUNSUPPORTED: "EUNSUPPORTED",
}

# Every exported symbol of include/px.h with its (restype, argtypes).
_c = ctypes
_vp = _c.c_void_p
_i32 = _c.c_int32
_i64 = _c.c_int64
_u64 = _c.c_uint64
_f32p = _c.POINTER(_c.c_float)
_i64p = _c.POINTER(_c.c_int64)
_i32p = _c.POINTER(_c.c_int32)
_u8p = _c.POINTER(_c.c_uint8)
_llp = _c.POINTER(_c.c_longlong)

class ProfileTotals(ctypes.Structure):
    """px_profile_totals (include/px.h)."""
    _fields_ = [("main_kernel_ms", ctypes.c_double), ("profiled_searches", ctypes.c_int64),
                ("searches", ctypes.c_int64), ("fallback_queries", ctypes.c_int64),
                ("refined_queries", ctypes.c_int64)]


class SearchProfile(ctypes.Structure):
    """px_search_profile (include/px.h)."""
    _fields_ = [("path", ctypes.c_int32), ("launches", ctypes.c_int32),
                ("fallback_queries", ctypes.c_int32), ("profiled", ctypes.c_int32),
                ("main_kernel_ms", ctypes.c_float), ("refined_queries", ctypes.c_int32),
                ("first_pass", ctypes.c_int32), ("sample_tiles", ctypes.c_int32)]


SIGNATURES = {
    "px_last_error": (_c.c_char_p, []),
    "px_version": (_c.c_char_p, []),
    "px_device_count": (_i32, []),
    "knn_gpu_create": (_vp, [_f32p, _c.c_int, _c.c_int]),
    "knn_gpu_search": (_c.c_int, [_vp, _f32p, _c.c_int, _c.c_int, _c.c_int, _llp, _f32p]),
    "knn_gpu_free": (None, [_vp]),
    "px_flat_create": (_i32, [_i32, _i32, _i32p, _i32, _c.POINTER(_vp)]),
    "px_flat_destroy": (_i32, [_vp]),
    "px_flat_add": (_i32, [_vp, _f32p, _i64]),
    "px_flat_add_device": (_i32, [_vp, _vp, _i64]),
    "px_flat_reserve": (_i32, [_vp, _i64]),
    "px_flat_read_rows": (_i32, [_vp, _i64, _i64, _f32p]),
    "px_pq_read_codes": (_i32, [_vp, _i64, _i64, _u8p]),
    "px_flat_size": (_i64, [_vp]),
    "px_flat_dim": (_i32, [_vp]),
    "px_flat_metric": (_i32, [_vp]),
    "px_flat_set_id_offset": (_i32, [_vp, _i64]),
    "px_flat_set_path": (_i32, [_vp, _i32]),
    "px_flat_set_sample_pass": (_i32, [_vp, _i32]),
    "px_set_profiling": (None, [_i32]),
    "px_flat_last_profile": (_i32, [_vp, _vp]),
    "px_flat_profile_totals": (_i32, [_vp, _i32, _vp]),
    "px_launch_count": (_i64, []),
    "px_flat_search": (_i32, [_vp, _f32p, _i64, _i32, _i64p, _f32p]),
    "px_flat_search_filtered": (_i32, [_vp, _f32p, _i64, _i32, _u8p, _i64p, _f32p]),
    "px_flat_search_device": (_i32, [_vp, _vp, _i64, _i32, _i32, _vp, _vp, _vp]),
    "px_flat_search_noalloc": (_i32, [_vp, _i64, _i32, _i32, _vp, _i64, _i32, _vp, _vp, _vp]),
    "px_flat_debug_candidates": (_i32, [_vp, _f32p, _i64, _i32, _i32, _i64p, _f32p, _i32p, _i32p]),
    "px_merge_shards_device": (_i32, [_i32, _vp, _vp, _i32, _i64, _i32, _i32, _i32, _vp, _vp, _vp]),
    "px_shard_record_bytes": (_i64, [_i64, _i32]),
    "px_merge_shard_records_device": (_i32, [_i32, _vp, _i32, _i64, _i32, _i32, _i32, _vp, _vp, _vp]),
    "px_pq_train": (_i32, [_f32p, _i64, _i32, _i32, _i32, _i32, _i64, _u64, _i32, _f32p]),
    "px_pq_create": (_i32, [_i32, _i32, _i32, _i32, _f32p, _i32p, _i32, _c.POINTER(_vp)]),
    "px_pq_destroy": (_i32, [_vp]),
    "px_pq_add": (_i32, [_vp, _f32p, _i64]),
    "px_pq_add_codes": (_i32, [_vp, _u8p, _i64]),
    "px_pq_encode": (_i32, [_vp, _f32p, _i64, _u8p]),
    "px_pq_size": (_i64, [_vp]),
    "px_pq_last_profile": (_i32, [_vp, _vp]),
    "px_pq_search": (_i32, [_vp, _f32p, _i64, _i32, _i64p, _f32p]),
    "px_pq_search_device": (_i32, [_vp, _vp, _i64, _i32, _i32, _vp, _vp, _vp]),
    "px_pq_search_filtered": (_i32, [_vp, _f32p, _i64, _i32, _u8p, _i64p, _f32p]),
}

_lib = None


class PxError(RuntimeError):
    """A px_* call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} [{_STATUS_NAMES.get(status, status)}]")
        self.status = status


def load():
    """Returns the loaded library; raises ImportError if it cannot be loaded."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing; build it with `python -m proxima_b200.build` "
                "(there is no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error() -> str:
    msg = load().px_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    if status != PX_OK:
        raise PxError(status, last_error())


def device_count() -> int:
    return int(load().px_device_count())


def set_profiling(enable: bool) -> None:
    """Brackets each search's dominant kernel with CUDA events (see px.h)."""
    load().px_set_profiling(1 if enable else 0)


def launch_count() -> int:
    """Kernels launched by libproxima_b200 in this process so far."""
    return int(load().px_launch_count())
