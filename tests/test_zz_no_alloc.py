"""pa_decode_noalloc: decode attention that allocates nothing.

Some callers cannot allocate device memory: C / FFI hosts that only hold
buffers another runtime allocated, and serving loops that must not call
cudaMalloc once the KV pool has taken most of HBM. pa_decode_noalloc keeps
its scratch in a static device array of the library instead of a workspace.
This test calls it through the C ABI twice in a row (different geometries,
so the second call starts from the first call's leftover scratch) and checks
each output against the workspace-based entry points (pa_decode_plan +
pa_decode_run) within the decode tolerance, max-abs 2e-2 / mean-abs 2e-3.
It is collected last so a failure here cannot hide the other tests.
"""

from __future__ import annotations

import ctypes
import importlib

import numpy as np
import pytest
import torch

from oracle import attention

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _desc(lir, pool_layer):
    fa = importlib.import_module("llm-inference-runtime_b200.flashinfer_api")
    return fa.kv_cache_desc(pool_layer, "HND")


def _run_both(lir, prob):
    lib = lir._lib.load()
    pool = prob.pool[0].to(DEV)
    q = prob.q.to(DEV)
    indptr, indices, last = prob.device_tables(DEV)
    desc = _desc(lir, pool)
    B, hq, d = q.shape
    stream = torch.cuda.current_stream().cuda_stream
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    out_ref = torch.empty_like(q)
    ws = torch.empty(128 << 20, dtype=torch.uint8, device=DEV)
    rc = lib.pa_decode_plan(p(indptr), p(last), B, indices.numel(), hq, desc.num_kv_heads, d,
                            16, p(ws), ws.numel(), stream)
    assert rc == 0, lir._lib.status_string(rc)
    rc = lib.pa_decode_run(p(q), q.stride(0), q.stride(1), ctypes.byref(desc), p(indices),
                           p(indptr), p(last), B, hq, 0.0, p(ws), ws.numel(), p(out_ref), None,
                           stream)
    assert rc == 0, lir._lib.status_string(rc)

    out = torch.full_like(q, float("nan"))
    rc = lib.pa_decode_noalloc(p(q), q.stride(0), q.stride(1), ctypes.byref(desc), p(indices),
                               p(indptr), p(last), B, indices.numel(), hq, 0.0, p(out), None,
                               stream)
    assert rc == 0, lir._lib.status_string(rc)
    assert lir._lib.device_status() == 0
    return out.cpu(), out_ref.cpu()


def test_noalloc_matches_workspace_entry_points_twice(lir, fi, workloads):
    # call 1: few long Llama-3 requests, every segment split and LSE-merged
    a = workloads.make_decode_problem(workloads.LLAMA3_8B, 5, 3000, 9000, seed=21, num_layers=1)
    # call 2: TinyLlama configuration 1 geometry, reusing the same scratch
    b = workloads.make_decode_problem(workloads.TINYLLAMA, 8, 16, 512, seed=22, num_layers=1,
                                      pool_pages=1024)
    for prob in (a, b):
        got, ref = _run_both(lir, prob)
        mx, mean, ok = attention.compare(got, ref)
        assert ok, f"no-alloc vs workspace entry point: max-abs {mx:.3e} mean-abs {mean:.3e}"
        want, _ = attention.decode(prob.q, prob.pool[0].float(), prob.kv_indptr,
                                   prob.kv_indices, prob.kv_last_page_len)
        assert attention.compare(got, want)[2]


def test_noalloc_rejects_batches_beyond_its_scratch(lir):
    lib = lir._lib.load()
    d = ctypes.c_void_p(256)
    desc = lir._lib.PagedKVCache()
    desc.k_base, desc.v_base = 0x10000, 0x20000
    desc.page_stride, desc.head_stride, desc.token_stride = 2 * 8 * 16 * 128, 16 * 128, 128
    desc.num_pages, desc.num_kv_heads, desc.page_size, desc.head_dim = 1 << 20, 8, 16, 128
    desc.dtype = lir._lib.PA_DTYPE_BF16
    # 400k requests need more than PA_NOALLOC_SCRATCH_BYTES of plan + counters
    rc = lib.pa_decode_noalloc(d, 4096, 128, ctypes.byref(desc), d, d, d, 400_000, 1 << 22, 32,
                               0.0, d, None, None)
    assert rc == lir._lib.PA_ERR_WORKSPACE_TOO_SMALL
