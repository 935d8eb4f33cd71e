"""ctypes binding of ``librefinekv_b200.so`` (the C ABI in ``include/refinekv_b200.h``).

The library is loaded on first use.  A missing or unloadable library raises
``RuntimeError``: this package has no CPU or library fallback.
"""

from __future__ import annotations

import ctypes
import pathlib
import threading

LIB_PATH = pathlib.Path(__file__).resolve().parent / "_lib" / "librefinekv_b200.so"
ABI_VERSION = 2

RKV_OK = 0
RKV_ERR_INVALID_ARGUMENT = 1
RKV_ERR_UNSUPPORTED = 2
RKV_ERR_ALIGNMENT = 3
RKV_ERR_WORKSPACE = 4
RKV_ERR_CUDA = 5

DEVICE_TIMEOUT = 1
DEVICE_BAD_INPUT = 2

GQA_CODES = {"mean": 0, "max": 1, "any": 2}
DTYPE_BF16 = 0
DTYPE_F32 = 1

PHASE_STATS = 1
PHASE_FINAL = 2
PHASE_ATTEND = 4
PHASE_COMBINE = 8
PHASE_ALL = 15

SPLIT_STATS = 1
SPLIT_ATTEND = 2
SPLIT_MERGE = 4
SPLIT_FINAL = 2

#: Every symbol the header declares.
EXPORTS = (
    "rkv_summarize",
    "rkv_summarize_f32",
    "rkv_summarize_into",
    "rkv_select_workspace_size",
    "rkv_select",
    "rkv_decode_workspace_size",
    "rkv_decode",
    "rkv_decode_static",
    "rkv_decode_static_status",
    "rkv_decode_dense_workspace_size",
    "rkv_decode_dense",
    "rkv_decode_launch_count",
    "rkv_decode_kernel_count",
    "rkv_set_fused_selector",
    "rkv_select_split_slab",
    "rkv_select_split",
    "rkv_split_exchange_slabs",
    "rkv_decode_split",
    "rkv_selftest_wait_timeout",
    "rkv_last_error",
    "rkv_status_string",
    "rkv_abi_version",
)

c_i64 = ctypes.c_int64
c_ptr = ctypes.c_void_p


class Summary(ctypes.Structure):
    """``struct rkv_summary``."""

    _fields_ = [
        ("key_pages", c_ptr),
        ("value_pages", c_ptr),
        ("key_page_head_stride", c_i64),
        ("value_page_head_stride", c_i64),
        ("counts", c_ptr),
        ("key_mean", c_ptr),
        ("value_mean", c_ptr),
        ("ellipsoid", c_ptr),
        ("value_norm", c_ptr),
        ("max_value_norm", c_ptr),
        ("heads", c_i64),
        ("blocks", c_i64),
        ("block_size", c_i64),
        ("head_dim", c_i64),
        ("prompt_length", c_i64),
        ("sequences", c_i64),
        ("prompt_lengths", c_ptr),
        ("page_table", c_ptr),
        ("page_table_stride", c_i64),
        ("pool_pages", c_i64),
        ("key_page_stride", c_i64),
        ("value_page_stride", c_i64),
        ("key_token_stride", c_i64),
        ("value_token_stride", c_i64),
    ]


_SIGNATURES = {
    "rkv_summarize": (ctypes.c_int, [c_ptr, c_ptr, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                     c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr,
                                     c_ptr, c_ptr, c_ptr]),
    "rkv_summarize_f32": (ctypes.c_int, [c_ptr, c_ptr, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                     c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr,
                                     c_ptr, c_ptr, c_ptr]),
    "rkv_summarize_into": (ctypes.c_int, [c_ptr, c_ptr, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                          c_i64, c_i64, c_ptr, c_i64, c_ptr, c_i64, c_ptr, c_ptr,
                                          c_ptr, c_ptr, c_ptr, c_ptr, c_ptr]),
    "rkv_select_workspace_size": (ctypes.c_size_t, [c_i64, c_i64, c_i64, c_i64, c_i64]),
    "rkv_select": (ctypes.c_int, [ctypes.POINTER(Summary), c_ptr, ctypes.c_int, c_i64, c_i64,
                                  ctypes.c_float, ctypes.c_int, c_ptr, ctypes.c_int, c_ptr,
                                  ctypes.c_size_t, c_ptr]),
    "rkv_decode_workspace_size": (ctypes.c_size_t, [c_i64, c_i64, c_i64, c_i64, c_i64]),
    "rkv_decode": (ctypes.c_int, [ctypes.POINTER(Summary), c_ptr, ctypes.c_int, c_i64, c_ptr,
                                  c_ptr, c_i64, c_i64, c_i64, c_i64, c_i64, c_ptr, c_i64, c_ptr,
                                  ctypes.c_float, ctypes.c_int, c_ptr, c_ptr, c_ptr,
                                  ctypes.c_size_t, ctypes.c_uint, c_ptr]),
    "rkv_decode_static": (ctypes.c_int, [ctypes.POINTER(Summary), c_ptr, ctypes.c_int, c_i64,
                                         c_ptr, c_ptr, c_i64, c_i64, c_i64, c_i64, c_i64, c_ptr,
                                         c_i64, c_ptr, ctypes.c_float, ctypes.c_int, c_ptr, c_ptr,
                                         c_ptr]),
    "rkv_decode_static_status": (ctypes.c_int, [c_ptr, c_ptr]),
    "rkv_decode_dense_workspace_size": (ctypes.c_size_t, [c_i64, c_i64, c_i64, c_i64, c_i64]),
    "rkv_decode_dense": (ctypes.c_int, [ctypes.POINTER(Summary), c_ptr, ctypes.c_int, c_i64,
                                        c_ptr, c_ptr, c_i64, c_i64, c_i64, c_i64, c_i64, c_ptr,
                                        c_i64, c_ptr, c_ptr, ctypes.c_size_t, c_ptr]),
    "rkv_decode_launch_count": (ctypes.c_int, [ctypes.c_uint]),
    "rkv_decode_kernel_count": (ctypes.c_int, [c_i64, c_i64, c_i64, c_i64, c_i64]),
    "rkv_set_fused_selector": (None, [ctypes.c_int]),
    "rkv_select_split_slab": (ctypes.c_size_t, [c_i64, c_i64, c_i64, c_i64]),
    "rkv_select_split": (ctypes.c_int, [ctypes.POINTER(Summary), c_ptr, ctypes.c_int, c_i64, c_i64,
                                        ctypes.c_float, ctypes.c_int, c_ptr, ctypes.c_int, c_ptr,
                                        ctypes.c_size_t, c_i64, c_i64, c_i64, c_ptr,
                                        ctypes.c_size_t, ctypes.c_uint, c_ptr]),
    "rkv_split_exchange_slabs": (ctypes.c_int, [c_i64, c_i64, c_i64, c_i64,
                                                ctypes.POINTER(ctypes.c_size_t),
                                                ctypes.POINTER(ctypes.c_size_t)]),
    "rkv_decode_split": (ctypes.c_int, [ctypes.POINTER(Summary), c_ptr, ctypes.c_int, c_i64,
                                        c_ptr, c_ptr, c_i64, c_i64, c_i64, c_i64, c_i64, c_ptr,
                                        c_i64, c_ptr, ctypes.c_float, ctypes.c_int, c_ptr, c_ptr,
                                        c_ptr, ctypes.c_size_t, c_i64, c_i64, c_i64, c_ptr,
                                        ctypes.c_size_t, ctypes.c_uint, c_ptr]),
    "rkv_selftest_wait_timeout": (ctypes.c_int, [c_ptr, c_i64, c_ptr]),
    "rkv_last_error": (ctypes.c_char_p, []),
    "rkv_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "rkv_abi_version": (ctypes.c_int, []),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the library once, declare every signature and check the ABI version."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python refinekv-release_b200/build.py` "
                "(refinekv_b200 has no CPU fallback)")
        try:
            lib = ctypes.CDLL(str(LIB_PATH))
        except OSError as error:
            raise RuntimeError(f"cannot load {LIB_PATH}: {error}") from error
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if lib.rkv_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{LIB_PATH} has ABI {lib.rkv_abi_version()}, expected {ABI_VERSION}")
        _lib = lib
        return lib


def check(rc: int) -> None:
    """Turn an rkv_status into the exception the reference raises for that kind of error."""
    if rc == RKV_OK:
        return
    lib = load()
    message = f"{lib.rkv_status_string(rc).decode()}: {lib.rkv_last_error().decode()}"
    if rc in (RKV_ERR_INVALID_ARGUMENT, RKV_ERR_UNSUPPORTED, RKV_ERR_ALIGNMENT):
        raise ValueError(message)
    raise RuntimeError(message)
