"""A CPU stand-in for this package's ``flashinfer_api`` — test infrastructure.

Every call is first bound, with ``inspect.signature(...).bind``, to the
signature of the ``flashinfer_api`` function or wrapper method of the same
name, so a call the real module would reject (unknown keyword, missing or
surplus positional argument) fails here as well. The results come from the
CPU oracle (``oracle.paged_kv`` / ``oracle.attention``), so a model driven
through it produces real logits on a machine without a GPU.

Used by the engine-swap tests to run the reference's own step executor and
``models/llama.py`` (src/engine/runtime/step_executor.py:82-259,
src/models/llama.py:39-249) on the CPU against this package's call surface.
"""

from __future__ import annotations

import importlib
import inspect

import numpy as np
import torch

from oracle import attention, paged_kv

API = importlib.import_module("llm-inference-runtime_b200.flashinfer_api")


def _bind(fn, *args, **kwargs) -> dict:
    ba = inspect.signature(fn).bind(*args, **kwargs)
    ba.apply_defaults()
    return dict(ba.arguments)


def _np(t) -> np.ndarray:
    return t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


def _rope_inplace(x: torch.Tensor, pos, rotary_dim, interleave, rope_scale, rope_theta) -> None:
    y = paged_kv.rope_reference(x.detach().float().cpu().numpy(), _np(pos), rotary_dim,
                                bool(interleave), float(rope_scale), float(rope_theta))
    x.copy_(torch.from_numpy(y).to(x.dtype))


class CpuFlashInfer:
    """Module-like object with flashinfer_api's names; records what was called."""

    def __init__(self):
        self.calls: list[str] = []
        outer = self

        class BatchDecodeWithPagedKVCacheWrapper:
            def __init__(self, *args, **kwargs):
                a = _bind(API.BatchDecodeWithPagedKVCacheWrapper.__init__, self, *args, **kwargs)
                outer.calls.append("BatchDecodeWithPagedKVCacheWrapper")
                self.layout = a["kv_layout"]

            def plan(self, *args, **kwargs):
                a = _bind(API.BatchDecodeWithPagedKVCacheWrapper.plan, self, *args, **kwargs)
                outer.calls.append("BatchDecodeWithPagedKVCacheWrapper.plan")
                self.t = a

            begin_forward = plan

            def run(self, *args, **kwargs):
                a = _bind(API.BatchDecodeWithPagedKVCacheWrapper.run, self, *args, **kwargs)
                outer.calls.append("BatchDecodeWithPagedKVCacheWrapper.run")
                return self._attend(a["q"], a["paged_kv_cache"])

            def forward(self, *args, **kwargs):
                a = _bind(API.BatchDecodeWithPagedKVCacheWrapper.forward, self, *args, **kwargs)
                outer.calls.append("BatchDecodeWithPagedKVCacheWrapper.forward")
                return self._attend(a["q"], a["paged_kv_cache"])

            def _attend(self, q, cache):
                o, _ = attention.decode(q, cache.float(), _np(self.t["indptr"]),
                                        _np(self.t["indices"]), _np(self.t["last_page_len"]),
                                        layout=self.layout, sm_scale=self.t["sm_scale"])
                return o.to(q.dtype)

        class BatchPrefillWithPagedKVCacheWrapper:
            def __init__(self, *args, **kwargs):
                a = _bind(API.BatchPrefillWithPagedKVCacheWrapper.__init__, self, *args, **kwargs)
                outer.calls.append("BatchPrefillWithPagedKVCacheWrapper")
                self.layout = a["kv_layout"]

            def plan(self, *args, **kwargs):
                a = _bind(API.BatchPrefillWithPagedKVCacheWrapper.plan, self, *args, **kwargs)
                outer.calls.append("BatchPrefillWithPagedKVCacheWrapper.plan")
                self.t = a
                self.causal = bool(a["causal"])

            begin_forward = plan

            def run(self, *args, **kwargs):
                a = _bind(API.BatchPrefillWithPagedKVCacheWrapper.run, self, *args, **kwargs)
                outer.calls.append("BatchPrefillWithPagedKVCacheWrapper.run")
                return self._attend(a["q"], a["paged_kv_cache"])

            def forward(self, *args, **kwargs):
                a = _bind(API.BatchPrefillWithPagedKVCacheWrapper.forward, self, *args, **kwargs)
                outer.calls.append("BatchPrefillWithPagedKVCacheWrapper.forward")
                self.causal = bool(a["causal"])
                return self._attend(a["q"], a["paged_kv_cache"])

            def _attend(self, q, cache):
                o, _ = attention.prefill(q, _np(self.t["qo_indptr"]), cache.float(),
                                         _np(self.t["paged_kv_indptr"]),
                                         _np(self.t["paged_kv_indices"]),
                                         _np(self.t["paged_kv_last_page_len"]),
                                         causal=self.causal, layout=self.layout,
                                         sm_scale=self.t["sm_scale"])
                return o.to(q.dtype)

        self.BatchDecodeWithPagedKVCacheWrapper = BatchDecodeWithPagedKVCacheWrapper
        self.BatchPrefillWithPagedKVCacheWrapper = BatchPrefillWithPagedKVCacheWrapper

    def get_batch_indices_positions(self, *args, **kwargs):
        a = _bind(API.get_batch_indices_positions, *args, **kwargs)
        self.calls.append("get_batch_indices_positions")
        bi, pos = paged_kv.batch_indices_positions(_np(a["append_indptr"]), _np(a["seq_lens"]),
                                                   int(a["nnz"]))
        dev = a["append_indptr"].device
        return torch.from_numpy(bi).to(dev), torch.from_numpy(pos).to(dev)

    def apply_rope_pos_ids_inplace(self, *args, **kwargs):
        a = _bind(API.apply_rope_pos_ids_inplace, *args, **kwargs)
        self.calls.append("apply_rope_pos_ids_inplace")
        for x in (a["q"], a["k"]):
            _rope_inplace(x, a["pos_ids"], a["rotary_dim"], a["interleave"], a["rope_scale"],
                          a["rope_theta"])

    def append_paged_kv_cache(self, *args, **kwargs):
        a = _bind(API.append_paged_kv_cache, *args, **kwargs)
        self.calls.append("append_paged_kv_cache")
        paged_kv.append_paged_kv_cache(a["append_key"], a["append_value"],
                                       _np(a["batch_indices"]), _np(a["positions"]),
                                       a["paged_kv_cache"], _np(a["kv_indices"]),
                                       _np(a["kv_indptr"]), layout=a["kv_layout"])

    def apply_rope_append(self, *args, **kwargs):
        a = _bind(API.apply_rope_append, *args, **kwargs)
        self.calls.append("apply_rope_append")
        for x in (a["q"], a["k"]):
            _rope_inplace(x, a["positions"], a["rotary_dim"], a["interleave"], a["rope_scale"],
                          a["rope_theta"])
        paged_kv.append_paged_kv_cache(a["k"], a["v"], _np(a["batch_indices"]),
                                       _np(a["positions"]), a["paged_kv_cache"],
                                       _np(a["kv_indices"]), _np(a["kv_indptr"]),
                                       layout=a["kv_layout"])

    def __getattr__(self, name):
        raise AttributeError(f"flashinfer_api has no CPU stand-in for {name!r} in this test")
