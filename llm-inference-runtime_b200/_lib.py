"""ctypes binding of the C ABI in ``include/paged_attn.h``.

The shared library ``libpaged_attn.so`` is built in-tree (see ``build.py``)
next to this file. There is no fallback: if the library is missing or fails
to load, every entry point raises. Status codes other than ``PA_OK`` become
``RuntimeError`` — the same failure surface the reference sees from
FlashInfer, caught by its batch-failure path
(src/engine/runtime/process_loop.py:129-132).
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int32, c_int64, c_size_t, c_void_p

LIB_NAME = "libpaged_attn.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

PA_OK = 0
PA_ERR_INVALID_ARGUMENT = 1
PA_ERR_UNSUPPORTED = 2
PA_ERR_WORKSPACE_TOO_SMALL = 3
PA_ERR_CUDA = 4
PA_ERR_DEVICE_CHECK = 5
PA_ERR_TIMEOUT = 6
PA_ERR_NOT_PLANNED = 7

PA_DTYPE_F16 = 0
PA_DTYPE_BF16 = 1

PA_NOALLOC_SCRATCH_BYTES = 24 * 1024 * 1024

# PA_ABI_VERSION of include/paged_attn.h that SIGNATURES mirrors; a library
# reporting another version is refused (argument lists would not line up).
ABI_VERSION = 101


class PagedKVCache(ctypes.Structure):
    """Mirror of ``pa_kv_cache``."""

    _fields_ = [
        ("k_base", c_void_p),
        ("v_base", c_void_p),
        ("page_stride", c_int64),
        ("head_stride", c_int64),
        ("token_stride", c_int64),
        ("num_pages", c_int64),
        ("num_kv_heads", c_int32),
        ("page_size", c_int32),
        ("head_dim", c_int32),
        ("dtype", c_int32),
    ]


# name -> (restype, argtypes); exactly the functions include/paged_attn.h declares.
SIGNATURES = {
    "pa_status_string": (ctypes.c_char_p, [c_int32]),
    "pa_abi_version": (c_int32, []),
    "pa_device_status": (c_int32, []),
    "pa_batch_indices_positions": (
        c_int32,
        [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p],
    ),
    "pa_append_paged_kv_cache": (
        c_int32,
        [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int32,
         POINTER(PagedKVCache), c_void_p, c_int64, c_void_p, c_int32, c_void_p],
    ),
    "pa_apply_rope_pos_ids_inplace": (
        c_int32,
        [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_int32, c_int32,
         c_int32, c_int32, c_int32, c_int32, c_float, c_float, c_int32, c_void_p],
    ),
    "pa_apply_rope_append": (
        c_int32,
        [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64,
         c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_float, c_float,
         POINTER(PagedKVCache), c_void_p, c_int64, c_void_p, c_int32, c_void_p],
    ),
    "pa_build_decode_tables": (
        c_int32,
        [c_void_p, c_int64, c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_int64,
         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "pa_build_prefill_tables": (
        c_int32,
        [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_void_p,
         c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
         c_void_p, c_void_p],
    ),
    "pa_fork_pages": (
        c_int32,
        [c_void_p, c_int64, c_int32, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int32,
         c_void_p],
    ),
    "pa_qkv_rope_append": (
        c_int32,
        [c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32, c_int32, c_void_p, c_int64,
         c_void_p, c_void_p, c_int32, c_int32, c_float, c_float, POINTER(PagedKVCache), c_void_p,
         c_int64, c_void_p, c_int32, c_void_p],
    ),
    "pa_selftest_wait_timeout": (c_int32, [c_int64, c_void_p]),
    "pa_decode_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32]),
    "pa_decode_plan": (
        c_int32,
        [c_void_p, c_void_p, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32, c_void_p,
         c_size_t, c_void_p],
    ),
    "pa_decode_run": (
        c_int32,
        [c_void_p, c_int64, c_int64, POINTER(PagedKVCache), c_void_p, c_void_p, c_void_p, c_int32,
         c_int32, c_float, c_void_p, c_size_t, c_void_p, c_void_p, c_void_p],
    ),
    "pa_decode_append_run": (
        c_int32,
        [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64,
         c_void_p, POINTER(PagedKVCache), c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_float,
         c_void_p, c_size_t, c_void_p, c_void_p, c_void_p],
    ),
    "pa_cascade_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32]),
    "pa_cascade_plan": (
        c_int32,
        [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int32, c_int64, c_int32, c_int32,
         c_int32, c_int32, c_void_p, c_size_t, c_void_p],
    ),
    "pa_cascade_run": (
        c_int32,
        [c_void_p, c_int64, c_int64, POINTER(PagedKVCache), c_void_p, c_void_p, c_void_p,
         c_void_p, c_int32, c_int32, c_float, c_void_p, c_size_t, c_void_p, c_void_p, c_void_p],
    ),
    "pa_cascade_append_run": (
        c_int32,
        [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64,
         c_void_p, POINTER(PagedKVCache), c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
         c_float, c_void_p, c_size_t, c_void_p, c_void_p, c_void_p],
    ),
    "pa_prefill_workspace_bytes": (c_size_t, [c_int32, c_int64, c_int32, c_int32, c_int32]),
    "pa_prefill_plan": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_int32, c_int64, c_int64, c_int32, c_int32, c_int32,
         c_int32, c_void_p, c_size_t, c_void_p],
    ),
    "pa_prefill_run": (
        c_int32,
        [c_void_p, c_int64, c_int64, POINTER(PagedKVCache), c_void_p, c_void_p, c_void_p,
         c_void_p, c_int32, c_int64, c_int32, c_int32, c_float, c_void_p, c_size_t, c_void_p,
         c_void_p, c_void_p],
    ),
    "pa_decode_noalloc": (
        c_int32,
        [c_void_p, c_int64, c_int64, POINTER(PagedKVCache), c_void_p, c_void_p, c_void_p, c_int32,
         c_int64, c_int32, c_float, c_void_p, c_void_p, c_void_p],
    ),
    "pa_merge_states": (
        c_int32,
        [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p,
         c_void_p],
    ),
}

_lib = None


def load() -> ctypes.CDLL:
    """Loads the in-tree library once; raises if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_NAME} not found at {LIB_PATH}; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` (needs nvcc)"
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        got = lib.pa_abi_version()
        if got != ABI_VERSION:
            raise RuntimeError(
                f"{LIB_NAME} reports ABI version {got}, this binding needs {ABI_VERSION}; "
                "rebuild the library from this checkout")
        _lib = lib
    return _lib


def status_string(code: int) -> str:
    return load().pa_status_string(code).decode()


def check(code: int, what: str) -> None:
    """Raises RuntimeError for a non-zero pa_status."""
    if code != PA_OK:
        raise RuntimeError(f"{what} failed: {status_string(code)} (status {code})")


def device_status() -> int:
    """Reads and clears the device-side status word (synchronises)."""
    return load().pa_device_status()


def check_device(what: str = "paged attention") -> None:
    code = device_status()
    if code != PA_OK:
        raise RuntimeError(f"{what}: device reported {status_string(code)} (status {code})")
