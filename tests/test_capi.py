"""The C-ABI library builds, loads and exports what include/paged_attn.h declares.

CPU only: these calls return on host-side argument checks before any launch.
"""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import REPO


def _declared_functions():
    with open(os.path.join(REPO, "include", "paged_attn.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pa_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree(lir):
    declared = _declared_functions()
    assert declared == sorted(lir._lib.SIGNATURES), "ctypes binding out of sync with the header"


def test_library_exports_every_declared_symbol(lir):
    lir.build.build()
    lib = ctypes.CDLL(lir._lib.LIB_PATH)
    missing = [name for name in _declared_functions() if not hasattr(lib, name)]
    assert not missing


def test_status_strings(lir):
    lir.build.build()
    assert lir._lib.status_string(0) == "ok"
    assert "unsupported" in lir._lib.status_string(lir._lib.PA_ERR_UNSUPPORTED)
    assert lir._lib.load().pa_abi_version() == lir._lib.ABI_VERSION


def test_header_and_binding_name_the_same_abi_version(lir):
    import re
    with open(os.path.join(REPO, "include", "paged_attn.h")) as f:
        m = re.search(r"#define PA_ABI_VERSION (\d+)", f.read())
    assert m and int(m.group(1)) == lir._lib.ABI_VERSION


def test_library_of_another_abi_version_is_refused(lir, monkeypatch):
    lir.build.build()
    monkeypatch.setattr(lir._lib, "_lib", None)
    monkeypatch.setattr(lir._lib, "ABI_VERSION", lir._lib.ABI_VERSION + 1)
    with pytest.raises(RuntimeError, match="ABI version"):
        lir._lib.load()


def test_host_side_validation_without_launch(lir):
    lib = lir._lib.load()
    dummy = ctypes.c_void_p(0x1000)
    # unsupported head_dim / page size / group size are rejected before any device query
    assert lib.pa_decode_plan(dummy, dummy, 4, 10, 32, 4, 96, 16, dummy, 1 << 20, None) == \
        lir._lib.PA_ERR_UNSUPPORTED
    assert lib.pa_decode_plan(dummy, dummy, 4, 10, 32, 4, 64, 8, dummy, 1 << 20, None) == \
        lir._lib.PA_ERR_UNSUPPORTED
    assert lib.pa_decode_plan(dummy, dummy, 4, 10, 64, 2, 64, 16, dummy, 1 << 20, None) == \
        lir._lib.PA_ERR_UNSUPPORTED
    # null pointers / bad sizes
    assert lib.pa_decode_plan(None, dummy, 4, 10, 32, 4, 64, 16, dummy, 1 << 20, None) == \
        lir._lib.PA_ERR_INVALID_ARGUMENT
    assert lib.pa_decode_plan(dummy, dummy, 0, 10, 32, 4, 64, 16, dummy, 1 << 20, None) == \
        lir._lib.PA_ERR_INVALID_ARGUMENT
    assert lib.pa_decode_plan(dummy, dummy, 4, 10, 30, 4, 64, 16, dummy, 1 << 20, None) == \
        lir._lib.PA_ERR_INVALID_ARGUMENT
    # empty work is a no-op success
    assert lib.pa_batch_indices_positions(dummy, dummy, 3, 0, None, None, None) == 0
    assert lib.pa_merge_states(None, None, 0, 2, 4, 64, 1, None, None, None) == 0
    assert lib.pa_merge_states(dummy, dummy, 4, 2, 4, 64, 7, dummy, None, None) == \
        lir._lib.PA_ERR_UNSUPPORTED


def test_cache_descriptor_validation(lir):
    lib = lir._lib.load()
    desc = lir._lib.PagedKVCache()
    desc.k_base = 0x1000
    desc.v_base = 0x1008  # not 16-byte aligned
    desc.page_stride, desc.head_stride, desc.token_stride = 2 * 4 * 16 * 64, 16 * 64, 64
    desc.num_pages, desc.num_kv_heads, desc.page_size, desc.head_dim = 8, 4, 16, 64
    desc.dtype = lir._lib.PA_DTYPE_BF16
    d = ctypes.c_void_p(0x1000)
    rc = lib.pa_decode_run(d, 2048, 64, ctypes.byref(desc), d, d, d, 4, 32, 0.0, d, 1 << 20, d,
                           None, None)
    assert rc == lir._lib.PA_ERR_INVALID_ARGUMENT
    desc.v_base = 0x2000
    desc.dtype = 9
    rc = lib.pa_decode_run(d, 2048, 64, ctypes.byref(desc), d, d, d, 4, 32, 0.0, d, 1 << 20, d,
                           None, None)
    assert rc == lir._lib.PA_ERR_UNSUPPORTED


def test_missing_library_raises(lir, monkeypatch, tmp_path):
    monkeypatch.setattr(lir._lib, "_lib", None)
    monkeypatch.setattr(lir._lib, "LIB_PATH", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError, match="not found"):
        lir._lib.load()
