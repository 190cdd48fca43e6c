"""The engine-level swap, run through the reference's own modules (CPU).

The reference's unmodified step executor (src/engine/runtime/
step_executor.py:82-259) drives a small random-init LLaMA through four
serving steps (``tests/engine_scenario.py``), with its attention module
bound two ways:

* the reference's own ``src/models/llama.py``, its ``import flashinfer``
  resolved to a CPU stand-in that binds every call, positional and keyword
  arguments as written at llama.py:55-67, 79, 106, 138, 175, 188, 218 and
  236, to this package's ``flashinfer_api`` signatures;
* this package's ``llama`` module as ``models.llama`` (the swap of the
  integration guide), its own calls bound the same way.

Both runs must reproduce transformers' eager logits (float32 on the CPU; the
attention math is the CPU oracle, the point here is the call surface). The
committed trace that the GPU replay uses is regenerated from the live
reference and must match. These tests need the reference checkout
($PA_REFERENCE_ROOT or a ``reference`` directory beside this repository).
"""

from __future__ import annotations

import copy
import importlib
import json
import os

import pytest
import torch

import cpu_flashinfer
import engine_scenario as sc
from conftest import GOLDEN

REF_SRC = sc.reference_src()
pytestmark = pytest.mark.skipif(REF_SRC is None, reason="reference checkout not present")


def _check_logits(recorded, streams, eager):
    maps = sc.row_maps()
    assert len(recorded) == len(maps)
    for logits, (mode, rows) in zip(recorded, maps):
        flat = logits.reshape(-1, logits.shape[-1])
        assert flat.shape[0] == len(rows), mode
        for k, (i, pos) in enumerate(rows):
            want = eager[i][pos]
            err = (flat[k] - want).abs().max() / want.abs().max()
            assert err < 1e-3, (mode, i, pos, float(err))


def _scenario(llama_module, se, patch):
    ref = sc.tiny_llama("cpu", torch.float32)
    model = copy.deepcopy(ref)
    patch(model)
    pool = torch.zeros((sc.LAYERS, sc.NUM_PAGES, 2, sc.KV_HEADS, sc.P, sc.HEAD_DIM),
                       dtype=torch.float32)
    llama_module.init_flashinfer_state(kv_pool=pool, page_size=sc.P, device="cpu")
    rec = sc.LogitsRecorder(model)
    res = sc.run(se, rec, "cpu")
    _check_logits(rec.logits, res["streams"], sc.eager_logits(ref, res["streams"]))
    return pool


def test_reference_llama_call_sites_bind_to_flashinfer_api():
    shim = cpu_flashinfer.CpuFlashInfer()
    ref_llama = sc.load_reference_llama(REF_SRC, shim)
    se = sc.import_step_executor(REF_SRC, ref_llama)
    _scenario(ref_llama, se, ref_llama.patch_llama_model)
    # every FlashInfer entry point the reference uses was reached
    for name in ("BatchPrefillWithPagedKVCacheWrapper", "BatchDecodeWithPagedKVCacheWrapper",
                 "get_batch_indices_positions", "apply_rope_pos_ids_inplace",
                 "append_paged_kv_cache", "BatchPrefillWithPagedKVCacheWrapper.plan",
                 "BatchPrefillWithPagedKVCacheWrapper.forward",
                 "BatchDecodeWithPagedKVCacheWrapper.plan",
                 "BatchDecodeWithPagedKVCacheWrapper.forward"):
        assert name in shim.calls, name


def test_engine_runs_with_this_package_as_models_llama(monkeypatch):
    shim = cpu_flashinfer.CpuFlashInfer()
    llama = importlib.import_module("llm-inference-runtime_b200.llama")
    monkeypatch.setattr(llama, "flashinfer", shim)
    monkeypatch.setattr(llama, "_FUSED_QKV", False)
    # the engine's prefill call passes no row count: the build must wait for
    # the first layer (which knows it) rather than read it back from the device
    resolved = []
    orig = llama.PagedAttnState._resolve_pending.__func__

    def spy(cls, nnz):
        if cls._pending is not None:
            assert nnz is not None, "positions built with a device read-back"
            resolved.append(nnz)
        return orig(cls, nnz)

    monkeypatch.setattr(llama.PagedAttnState, "_resolve_pending", classmethod(spy))
    se = sc.import_step_executor(REF_SRC, llama)
    _scenario(llama, se, llama.patch_llama_model)
    assert resolved == [73, 34]  # the two prefill steps' rows
    assert "apply_rope_append" in shim.calls
    assert "BatchPrefillWithPagedKVCacheWrapper.forward" in shim.calls
    assert "BatchDecodeWithPagedKVCacheWrapper.forward" in shim.calls


def test_committed_engine_trace_matches_the_reference():
    import golden.make_engine_trace as mk
    with open(os.path.join(GOLDEN, "engine_trace.json")) as f:
        committed = json.load(f)
    assert json.loads(json.dumps(mk.trace(REF_SRC))) == committed
