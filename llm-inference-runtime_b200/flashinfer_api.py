"""FlashInfer-compatible operator surface backed by the sm_100a kernels.

The reference engine reaches its GPU work only through these FlashInfer
0.6.11 names (src/models/llama.py:3, 55-67, 79, 106, 138, 175, 188, 218,
236). This module provides the same names, arguments and error behaviour,
so ``models/llama.py`` works with ``import flashinfer`` pointed here:

* ``get_batch_indices_positions``   (llama.py:79)
* ``append_paged_kv_cache``         (llama.py:188, kv_layout "HND" or "NHD")
* ``apply_rope_pos_ids_inplace``    (llama.py:175)
* ``BatchPrefillWithPagedKVCacheWrapper`` plan/begin_forward/run/forward
  (llama.py:55-60, 106, 218)
* ``BatchDecodeWithPagedKVCacheWrapper`` plan/begin_forward/run/forward
  (llama.py:62-67, 138, 236)
* ``merge_state`` / ``merge_states`` / ``get_seq_lens`` (split-KV helpers)
* ``MultiLevelCascadeAttentionWrapper`` (two levels: a prefix every request
  shares, then each request's own pages) for radix-shared decode batches

Every call goes through the C ABI (``_lib``) on the current torch CUDA
stream. There is no CPU or PyTorch fallback: a missing library, an
unsupported option or a failing status raises. Setting ``PA_CHECK=1`` makes
each call synchronise and raise on device-side validation errors.
"""

from __future__ import annotations

import ctypes
import math
import os
from typing import Optional, Tuple, Union

import torch

from . import _lib

_CHECK = os.environ.get("PA_CHECK", "0") not in ("", "0")

_DTYPE_CODES = {torch.float16: _lib.PA_DTYPE_F16, torch.bfloat16: _lib.PA_DTYPE_BF16}
_STR_DTYPES = {"float16": torch.float16, "half": torch.float16, "bfloat16": torch.bfloat16}


def _dtype_code(dt: torch.dtype) -> int:
    if dt not in _DTYPE_CODES:
        raise NotImplementedError(f"dtype {dt} is not supported (float16 / bfloat16 only)")
    return _DTYPE_CODES[dt]


def _as_dtype(dt) -> Optional[torch.dtype]:
    if dt is None or isinstance(dt, torch.dtype):
        return dt
    return _STR_DTYPES[str(dt).replace("torch.", "")]


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _p(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _i32_on(t: torch.Tensor, device: torch.device, name: str) -> torch.Tensor:
    if t.dtype != torch.int32:
        raise ValueError(f"{name} must be int32, got {t.dtype}")
    if t.device != device:
        t = t.to(device, non_blocking=True)
    return t.contiguous()


def _after(what: str) -> None:
    if _CHECK:
        _lib.check_device(what)


def kv_cache_desc(paged_kv_cache, kv_layout: str = "NHD") -> _lib.PagedKVCache:
    """Describes one layer of a FlashInfer-layout paged KV cache.

    Accepts the single 5-D tensor ``[N, 2, H, P, D]`` ("HND") /
    ``[N, 2, P, H, D]`` ("NHD") or a ``(k_cache, v_cache)`` tuple of 4-D
    tensors, exactly as ``append_paged_kv_cache`` and the wrappers do.
    """
    if kv_layout not in ("NHD", "HND"):
        raise KeyError(f"Invalid kv_layout {kv_layout}")
    if isinstance(paged_kv_cache, torch.Tensor):
        if paged_kv_cache.dim() != 5 or paged_kv_cache.size(1) != 2:
            raise ValueError("paged_kv_cache tensor must be 5-D [num_pages, 2, ...]")
        k = paged_kv_cache.select(1, 0)
        v = paged_kv_cache.select(1, 1)
    else:
        k, v = paged_kv_cache
        if k.dim() != 4 or v.shape != k.shape:
            raise ValueError("k_cache / v_cache must be 4-D tensors of equal shape")
        if k.stride() != v.stride():
            raise ValueError("k_cache and v_cache must have the same strides")
    if k.stride(-1) != 1:
        raise ValueError("the head_dim dimension of the KV cache must be contiguous")
    if kv_layout == "HND":
        n, h, p, d = k.shape
        head_stride, token_stride = k.stride(1), k.stride(2)
    else:
        n, p, h, d = k.shape
        token_stride, head_stride = k.stride(1), k.stride(2)
    desc = _lib.PagedKVCache()
    desc.k_base = k.data_ptr()
    desc.v_base = v.data_ptr()
    desc.page_stride = k.stride(0)
    desc.head_stride = head_stride
    desc.token_stride = token_stride
    desc.num_pages = n
    desc.num_kv_heads = h
    desc.page_size = p
    desc.head_dim = d
    desc.dtype = _dtype_code(k.dtype)
    return desc


def _row_strides(x: torch.Tensor, name: str) -> Tuple[int, int]:
    if x.dim() != 3:
        raise ValueError(f"{name} must be 3-D [tokens, heads, head_dim]")
    if x.stride(-1) != 1:
        raise ValueError(f"{name}: head_dim must be contiguous")
    return x.stride(0), x.stride(1)


# ----------------------------------------------------------------- indexing
def get_seq_lens(kv_indptr: torch.Tensor, kv_last_page_len: torch.Tensor,
                 page_size: int) -> torch.Tensor:
    """KV length per request: (pages - 1) * page_size + last_page_len, 0 if no pages."""
    pages = kv_indptr[1:] - kv_indptr[:-1]
    return (torch.clamp(pages - 1, min=0) * page_size
            + torch.where(pages > 0, kv_last_page_len, torch.zeros_like(kv_last_page_len)))


def get_batch_indices_positions(append_indptr: torch.Tensor, seq_lens: torch.Tensor, nnz: int,
                                batch_indices: Optional[torch.Tensor] = None,
                                positions: Optional[torch.Tensor] = None,
                                ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Ragged append rows -> (owning request, absolute position) per row.

    positions[t] = seq_lens[b] - append_len[b] + (t - append_indptr[b]).
    """
    device = append_indptr.device
    batch = append_indptr.numel() - 1
    append_indptr = _i32_on(append_indptr, device, "append_indptr")
    seq_lens = _i32_on(seq_lens, device, "seq_lens")
    if batch_indices is None:
        batch_indices = torch.empty((nnz,), dtype=torch.int32, device=device)
    if positions is None:
        positions = torch.empty((nnz,), dtype=torch.int32, device=device)
    _lib.check(_lib.load().pa_batch_indices_positions(
        _p(append_indptr), _p(seq_lens), batch, nnz, _p(batch_indices), _p(positions), _stream()),
        "get_batch_indices_positions")
    _after("get_batch_indices_positions")
    return batch_indices, positions


def append_paged_kv_cache(append_key: torch.Tensor, append_value: torch.Tensor,
                          batch_indices: torch.Tensor, positions: torch.Tensor,
                          paged_kv_cache, kv_indices: torch.Tensor, kv_indptr: torch.Tensor,
                          kv_last_page_len: torch.Tensor, kv_layout: str = "NHD") -> None:
    """Scatters new K/V rows into their pages (in place, bit-exact copy)."""
    desc = kv_cache_desc(paged_kv_cache, kv_layout)
    if append_key.dtype != append_value.dtype or _dtype_code(append_key.dtype) != desc.dtype:
        raise ValueError("append_key / append_value must have the KV cache's dtype")
    ksn, ksh = _row_strides(append_key, "append_key")
    vsn, vsh = _row_strides(append_value, "append_value")
    nnz = append_key.size(0)
    if append_key.size(1) != desc.num_kv_heads or append_key.size(2) != desc.head_dim:
        raise ValueError("append_key shape does not match the KV cache")
    device = append_key.device
    batch_indices = _i32_on(batch_indices, device, "batch_indices")
    positions = _i32_on(positions, device, "positions")
    kv_indices = _i32_on(kv_indices, device, "kv_indices")
    kv_indptr = _i32_on(kv_indptr, device, "kv_indptr")
    _lib.check(_lib.load().pa_append_paged_kv_cache(
        _p(append_key), ksn, ksh, _p(append_value), vsn, vsh, _p(batch_indices), _p(positions),
        nnz, ctypes.byref(desc), _p(kv_indices), kv_indices.numel(), _p(kv_indptr),
        kv_indptr.numel() - 1, _stream()), "append_paged_kv_cache")
    _after("append_paged_kv_cache")


def apply_rope_pos_ids_inplace(q: torch.Tensor, k: torch.Tensor, pos_ids: torch.Tensor,
                               rotary_dim: Optional[int] = None, interleave: bool = False,
                               rope_scale: float = 1, rope_theta: float = 1e4) -> None:
    """Rotary embedding on q [nnz, Hq, D] and k [nnz, Hkv, D] in place."""
    qsn, qsh = _row_strides(q, "q")
    ksn, ksh = _row_strides(k, "k")
    if q.dtype != k.dtype:
        raise ValueError("q and k must share a dtype")
    d = q.size(-1)
    if rotary_dim is None:
        rotary_dim = d
    pos_ids = _i32_on(pos_ids, q.device, "pos_ids")
    _lib.check(_lib.load().pa_apply_rope_pos_ids_inplace(
        _p(q), qsn, qsh, _p(k), ksn, ksh, _p(pos_ids), q.size(0), q.size(1), k.size(1), d,
        rotary_dim, int(bool(interleave)), float(rope_scale), float(rope_theta),
        _dtype_code(q.dtype), _stream()), "apply_rope_pos_ids_inplace")
    _after("apply_rope_pos_ids_inplace")


def apply_rope_append(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      batch_indices: torch.Tensor, positions: torch.Tensor, paged_kv_cache,
                      kv_indices: torch.Tensor, kv_indptr: torch.Tensor,
                      kv_last_page_len: torch.Tensor, kv_layout: str = "NHD",
                      rotary_dim: Optional[int] = None, interleave: bool = False,
                      rope_scale: float = 1, rope_theta: float = 1e4) -> None:
    """apply_rope_pos_ids_inplace(q, k, positions, ...) followed by
    append_paged_kv_cache(k, v, batch_indices, positions, ...), in one launch
    (the pair the reference runs per layer at src/models/llama.py:175-210).
    Same results as the two calls: q and k rotated in place, the rotated k and
    v written into their page slots."""
    desc = kv_cache_desc(paged_kv_cache, kv_layout)
    if not (q.dtype == k.dtype == v.dtype) or _dtype_code(q.dtype) != desc.dtype:
        raise ValueError("q / k / v must have the KV cache's dtype")
    qsn, qsh = _row_strides(q, "q")
    ksn, ksh = _row_strides(k, "k")
    vsn, vsh = _row_strides(v, "v")
    if k.shape != v.shape or k.size(1) != desc.num_kv_heads or k.size(2) != desc.head_dim:
        raise ValueError("k / v shape does not match the KV cache")
    if q.size(0) != k.size(0) or q.size(2) != k.size(2):
        raise ValueError("q and k must have the same rows and head_dim")
    d = q.size(-1)
    if rotary_dim is None:
        rotary_dim = d
    device = q.device
    batch_indices = _i32_on(batch_indices, device, "batch_indices")
    positions = _i32_on(positions, device, "positions")
    kv_indices = _i32_on(kv_indices, device, "kv_indices")
    kv_indptr = _i32_on(kv_indptr, device, "kv_indptr")
    _lib.check(_lib.load().pa_apply_rope_append(
        _p(q), qsn, qsh, _p(k), ksn, ksh, _p(v), vsn, vsh, _p(batch_indices), _p(positions),
        q.size(0), q.size(1), rotary_dim, int(bool(interleave)), float(rope_scale),
        float(rope_theta), ctypes.byref(desc), _p(kv_indices), kv_indices.numel(),
        _p(kv_indptr), kv_indptr.numel() - 1, _stream()), "apply_rope_append")
    _after("apply_rope_append")


# -------------------------------------------------------------------- merge
def merge_states(v: torch.Tensor, s: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """v [n, S, H, D], s [n, S, H] (float32, base-2 LSE) -> merged (v, s)."""
    n, ns, h, d = v.shape
    if s.shape != (n, ns, h) or s.dtype != torch.float32:
        raise ValueError("s must be float32 [seq_len, num_states, num_heads]")
    v = v.contiguous()
    s = s.contiguous()
    vm = torch.empty((n, h, d), dtype=v.dtype, device=v.device)
    sm = torch.empty((n, h), dtype=torch.float32, device=v.device)
    _lib.check(_lib.load().pa_merge_states(_p(v), _p(s), n, ns, h, d, _dtype_code(v.dtype),
                                           _p(vm), _p(sm), _stream()), "merge_states")
    _after("merge_states")
    return vm, sm


def merge_state(v_a: torch.Tensor, s_a: torch.Tensor, v_b: torch.Tensor,
                s_b: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Merges two attention states over disjoint KV segments."""
    return merge_states(torch.stack([v_a, v_b], dim=1), torch.stack([s_a, s_b], dim=1))


# ----------------------------------------------------------------- wrappers
def _check_plan_options(pos_encoding_mode: str, window_left: int,
                        logits_soft_cap: Optional[float]) -> None:
    if pos_encoding_mode not in ("NONE", None):
        raise NotImplementedError("pos_encoding_mode other than 'NONE' is not supported")
    if window_left is not None and window_left >= 0:
        raise NotImplementedError("sliding-window attention (window_left >= 0) is not supported")
    if logits_soft_cap not in (None, 0, 0.0):
        raise NotImplementedError("logits_soft_cap is not supported")


def _check_scales(q_scale, k_scale, v_scale) -> float:
    if v_scale not in (None, 1, 1.0):
        raise NotImplementedError("v_scale is not supported")
    return float(q_scale or 1.0) * float(k_scale or 1.0)


class BatchDecodeWithPagedKVCacheWrapper:
    """Batched decode over a paged KV cache (one query row per request).

    Same constructor / plan / run surface as FlashInfer's wrapper of this
    name as the reference builds it (src/models/llama.py:62-67, 138-147,
    236-239). The workspace buffer holds the device-side plan and the
    split-KV partial states.
    """

    def __init__(self, float_workspace_buffer: torch.Tensor, kv_layout: str = "NHD",
                 use_cuda_graph: bool = False, use_tensor_cores: bool = False, **kwargs) -> None:
        if kv_layout not in ("NHD", "HND"):
            raise KeyError(f"Invalid kv_layout {kv_layout}")
        self._ws = float_workspace_buffer
        self._kv_layout = kv_layout
        self._planned = False

    @property
    def is_cuda_graph_enabled(self) -> bool:
        return False

    def reset_workspace_buffer(self, float_workspace_buffer: torch.Tensor, *args) -> None:
        self._ws = float_workspace_buffer

    def plan(self, indptr: torch.Tensor, indices: torch.Tensor, last_page_len: torch.Tensor,
             num_qo_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
             pos_encoding_mode: str = "NONE", window_left: int = -1,
             logits_soft_cap: Optional[float] = None, q_data_type="float16",
             kv_data_type=None, data_type=None, sm_scale: Optional[float] = None,
             rope_scale: Optional[float] = None, rope_theta: Optional[float] = None,
             non_blocking: bool = True, **kwargs) -> None:
        _check_plan_options(pos_encoding_mode, window_left, logits_soft_cap)
        device = self._ws.device
        self._indptr = _i32_on(indptr, device, "indptr")
        self._indices = _i32_on(indices, device, "indices")
        self._last = _i32_on(last_page_len, device, "last_page_len")
        self._batch = self._indptr.numel() - 1
        self._hq, self._hkv, self._d, self._p = num_qo_heads, num_kv_heads, head_dim, page_size
        self._q_dtype = _as_dtype(data_type) or _as_dtype(q_data_type)
        self._kv_dtype = _as_dtype(kv_data_type) or self._q_dtype
        self._sm_scale = sm_scale
        _lib.check(_lib.load().pa_decode_plan(
            _p(self._indptr), _p(self._last), self._batch, self._indices.numel(), num_qo_heads,
            num_kv_heads, head_dim, page_size, _p(self._ws), self._ws.numel() *
            self._ws.element_size(), _stream()), "BatchDecodeWithPagedKVCacheWrapper.plan")
        _after("BatchDecodeWithPagedKVCacheWrapper.plan")
        self._planned = True

    begin_forward = plan

    def end_forward(self) -> None:
        pass

    def run(self, q: torch.Tensor, paged_kv_cache, *args, q_scale=None, k_scale=None,
            v_scale=None, out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
            return_lse: bool = False, **kwargs):
        return self._run(q, paged_kv_cache, None, q_scale, k_scale, v_scale, out, lse,
                         return_lse)

    def run_with_append(self, q: torch.Tensor, paged_kv_cache, append_key: torch.Tensor,
                        append_value: torch.Tensor, positions: torch.Tensor, *,
                        out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
                        return_lse: bool = False):
        """This package's extension: the decode step's
        ``append_paged_kv_cache(append_key, append_value, arange(B), positions, ...)``
        followed by :meth:`run`, as one launch (row b of append_key /
        append_value is request b's new token). The pool afterwards is
        bit-identical to the two-call sequence and so is the output."""
        desc = kv_cache_desc(paged_kv_cache, self._kv_layout)
        if append_key.dtype != append_value.dtype or _dtype_code(append_key.dtype) != desc.dtype:
            raise ValueError("append_key / append_value must have the KV cache's dtype")
        for name, x in (("append_key", append_key), ("append_value", append_value)):
            _row_strides(x, name)
            if tuple(x.shape) != (self._batch, desc.num_kv_heads, desc.head_dim):
                raise ValueError(f"{name} must be [{self._batch}, {desc.num_kv_heads}, "
                                 f"{desc.head_dim}]")
        positions = _i32_on(positions, q.device, "positions")
        if positions.numel() != self._batch:
            raise ValueError("positions must hold one entry per request")
        return self._run(q, paged_kv_cache, (append_key, append_value, positions), None, None,
                         None, out, lse, return_lse)

    def _run(self, q, paged_kv_cache, append, q_scale, k_scale, v_scale, out, lse, return_lse):
        if not self._planned:
            raise RuntimeError("plan() must be called before run()")
        desc = kv_cache_desc(paged_kv_cache, self._kv_layout)
        if (desc.num_kv_heads, desc.head_dim, desc.page_size) != (self._hkv, self._d, self._p):
            raise ValueError("paged_kv_cache geometry differs from the plan")
        if _dtype_code(q.dtype) != desc.dtype:
            raise NotImplementedError("q and the KV cache must have the same dtype")
        qsn, qsh = _row_strides(q, "q")
        if q.size(0) != self._batch or q.size(1) != self._hq or q.size(2) != self._d:
            raise ValueError(f"q must be [{self._batch}, {self._hq}, {self._d}]")
        if out is None:
            out = torch.empty((self._batch, self._hq, self._d), dtype=q.dtype, device=q.device)
        elif not out.is_contiguous() or out.shape != (self._batch, self._hq, self._d):
            raise ValueError("out must be a contiguous [batch, num_qo_heads, head_dim] tensor")
        if return_lse and lse is None:
            lse = torch.empty((self._batch, self._hq), dtype=torch.float32, device=q.device)
        scale = self._sm_scale if self._sm_scale is not None else 1.0 / math.sqrt(self._d)
        scale *= _check_scales(q_scale, k_scale, v_scale)
        ws_bytes = self._ws.numel() * self._ws.element_size()
        if append is None:
            _lib.check(_lib.load().pa_decode_run(
                _p(q), qsn, qsh, ctypes.byref(desc), _p(self._indices), _p(self._indptr),
                _p(self._last), self._batch, self._hq, float(scale), _p(self._ws), ws_bytes,
                _p(out), _p(lse), _stream()), "BatchDecodeWithPagedKVCacheWrapper.run")
            _after("BatchDecodeWithPagedKVCacheWrapper.run")
        else:
            k, v, pos = append
            ksn, ksh = k.stride(0), k.stride(1)
            vsn, vsh = v.stride(0), v.stride(1)
            _lib.check(_lib.load().pa_decode_append_run(
                _p(q), qsn, qsh, _p(k), ksn, ksh, _p(v), vsn, vsh, _p(pos), ctypes.byref(desc),
                _p(self._indices), _p(self._indptr), _p(self._last), self._batch, self._hq,
                float(scale), _p(self._ws), ws_bytes, _p(out), _p(lse), _stream()),
                "BatchDecodeWithPagedKVCacheWrapper.run_with_append")
            _after("BatchDecodeWithPagedKVCacheWrapper.run_with_append")
        return (out, lse) if return_lse else out

    def forward(self, q: torch.Tensor, paged_kv_cache, pos_encoding_mode: str = "NONE",
                q_scale=None, k_scale=None, v_scale=None, window_left: int = -1,
                logits_soft_cap: Optional[float] = None, sm_scale: Optional[float] = None,
                rope_scale=None, rope_theta=None) -> torch.Tensor:
        """Deprecated FlashInfer alias of run() that the reference calls (llama.py:236)."""
        _check_plan_options(pos_encoding_mode, window_left, logits_soft_cap)
        if sm_scale is not None:
            self._sm_scale = sm_scale
        return self.run(q, paged_kv_cache, q_scale=q_scale, k_scale=k_scale, v_scale=v_scale)

    def forward_return_lse(self, q: torch.Tensor, paged_kv_cache, pos_encoding_mode="NONE",
                           q_scale=None, k_scale=None, v_scale=None, window_left=-1,
                           logits_soft_cap=None, sm_scale=None, rope_scale=None,
                           rope_theta=None):
        _check_plan_options(pos_encoding_mode, window_left, logits_soft_cap)
        if sm_scale is not None:
            self._sm_scale = sm_scale
        return self.run(q, paged_kv_cache, q_scale=q_scale, k_scale=k_scale, v_scale=v_scale,
                        return_lse=True)


class BatchPrefillWithPagedKVCacheWrapper:
    """Ragged (chunked) prefill over a paged KV cache.

    Mirrors FlashInfer's wrapper as the reference builds and calls it
    (src/models/llama.py:55-60, 106-116, 218-222): planned once per step,
    run per layer with ``causal=True`` (bottom-right aligned mask).
    """

    def __init__(self, float_workspace_buffer: torch.Tensor, kv_layout: str = "NHD",
                 use_cuda_graph: bool = False, backend: str = "auto", **kwargs) -> None:
        if kv_layout not in ("NHD", "HND"):
            raise KeyError(f"Invalid kv_layout {kv_layout}")
        self._ws = float_workspace_buffer
        self._kv_layout = kv_layout
        self._planned = False
        self._causal = False

    @property
    def is_cuda_graph_enabled(self) -> bool:
        return False

    def reset_workspace_buffer(self, float_workspace_buffer: torch.Tensor, *args) -> None:
        self._ws = float_workspace_buffer

    def plan(self, qo_indptr: torch.Tensor, paged_kv_indptr: torch.Tensor,
             paged_kv_indices: torch.Tensor, paged_kv_last_page_len: torch.Tensor,
             num_qo_heads: int, num_kv_heads: int, head_dim_qk: int, page_size: int,
             head_dim_vo: Optional[int] = None, custom_mask=None, packed_custom_mask=None,
             causal: bool = False, pos_encoding_mode: str = "NONE",
             use_fp16_qk_reduction: bool = False, sm_scale: Optional[float] = None,
             window_left: int = -1, logits_soft_cap: Optional[float] = None,
             rope_scale=None, rope_theta=None, q_data_type="float16", kv_data_type=None,
             non_blocking: bool = True, **kwargs) -> None:
        _check_plan_options(pos_encoding_mode, window_left, logits_soft_cap)
        if custom_mask is not None or packed_custom_mask is not None:
            raise NotImplementedError("custom masks are not supported")
        if head_dim_vo not in (None, head_dim_qk):
            raise NotImplementedError("head_dim_vo must equal head_dim_qk")
        device = self._ws.device
        self._qo_indptr = _i32_on(qo_indptr, device, "qo_indptr")
        self._indptr = _i32_on(paged_kv_indptr, device, "paged_kv_indptr")
        self._indices = _i32_on(paged_kv_indices, device, "paged_kv_indices")
        self._last = _i32_on(paged_kv_last_page_len, device, "paged_kv_last_page_len")
        self._batch = self._indptr.numel() - 1
        self._hq, self._hkv, self._d, self._p = num_qo_heads, num_kv_heads, head_dim_qk, page_size
        self._causal = bool(causal)
        self._sm_scale = sm_scale
        self._plan_total = None
        self._planned = True
        self._needs_device_plan = True
        # The device plan needs the number of query rows (it sizes the work
        # list). It is known here when qo_indptr lives on the host or the
        # caller passes total_qo; otherwise the first run() plans, from
        # q.size(0), without any device-to-host copy.
        total = kwargs.get("total_qo")
        if total is None and qo_indptr.device.type == "cpu":
            total = int(qo_indptr[-1])
        if total is not None:
            self._device_plan(int(total))

    begin_forward = plan

    def end_forward(self) -> None:
        pass

    def _device_plan(self, total_qo: int) -> None:
        _lib.check(_lib.load().pa_prefill_plan(
            _p(self._qo_indptr), _p(self._indptr), _p(self._last), self._batch, total_qo,
            self._indices.numel(), self._hq, self._hkv, self._d, self._p, _p(self._ws),
            self._ws.numel() * self._ws.element_size(), _stream()),
            "BatchPrefillWithPagedKVCacheWrapper.plan")
        _after("BatchPrefillWithPagedKVCacheWrapper.plan")
        self._plan_total = total_qo
        self._needs_device_plan = False

    def run(self, q: torch.Tensor, paged_kv_cache, *args, q_scale=None, k_scale=None,
            v_scale=None, out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
            return_lse: bool = False, **kwargs):
        if not self._planned:
            raise RuntimeError("plan() must be called before run()")
        desc = kv_cache_desc(paged_kv_cache, self._kv_layout)
        if (desc.num_kv_heads, desc.head_dim, desc.page_size) != (self._hkv, self._d, self._p):
            raise ValueError("paged_kv_cache geometry differs from the plan")
        if _dtype_code(q.dtype) != desc.dtype:
            raise NotImplementedError("q and the KV cache must have the same dtype")
        qsn, qsh = _row_strides(q, "q")
        total_qo = q.size(0)
        if q.size(1) != self._hq or q.size(2) != self._d:
            raise ValueError(f"q must be [total_qo, {self._hq}, {self._d}]")
        if self._needs_device_plan or self._plan_total != total_qo:
            self._device_plan(total_qo)
        if out is None:
            out = torch.empty((total_qo, self._hq, self._d), dtype=q.dtype, device=q.device)
        elif not out.is_contiguous() or out.shape != (total_qo, self._hq, self._d):
            raise ValueError("out must be a contiguous [total_qo, num_qo_heads, head_dim] tensor")
        if return_lse and lse is None:
            lse = torch.empty((total_qo, self._hq), dtype=torch.float32, device=q.device)
        scale = self._sm_scale if self._sm_scale is not None else 1.0 / math.sqrt(self._d)
        scale *= _check_scales(q_scale, k_scale, v_scale)
        _lib.check(_lib.load().pa_prefill_run(
            _p(q), qsn, qsh, ctypes.byref(desc), _p(self._qo_indptr), _p(self._indices),
            _p(self._indptr), _p(self._last), self._batch, total_qo, self._hq,
            int(self._causal), float(scale), _p(self._ws),
            self._ws.numel() * self._ws.element_size(), _p(out), _p(lse), _stream()),
            "BatchPrefillWithPagedKVCacheWrapper.run")
        _after("BatchPrefillWithPagedKVCacheWrapper.run")
        return (out, lse) if return_lse else out

    def forward(self, q: torch.Tensor, paged_kv_cache, causal: bool = False,
                pos_encoding_mode: str = "NONE", use_fp16_qk_reduction: bool = False,
                k_scale=None, v_scale=None, window_left: int = -1,
                logits_soft_cap: Optional[float] = None, sm_scale: Optional[float] = None,
                rope_scale=None, rope_theta=None) -> torch.Tensor:
        """Deprecated FlashInfer alias of run(); sets causal like FlashInfer does (llama.py:218)."""
        _check_plan_options(pos_encoding_mode, window_left, logits_soft_cap)
        self._causal = bool(causal)
        if sm_scale is not None:
            self._sm_scale = sm_scale
        return self.run(q, paged_kv_cache, k_scale=k_scale, v_scale=v_scale)

    def forward_return_lse(self, q: torch.Tensor, paged_kv_cache, causal: bool = False,
                           pos_encoding_mode: str = "NONE", use_fp16_qk_reduction=False,
                           k_scale=None, v_scale=None, window_left=-1, logits_soft_cap=None,
                           sm_scale=None, rope_scale=None, rope_theta=None):
        _check_plan_options(pos_encoding_mode, window_left, logits_soft_cap)
        self._causal = bool(causal)
        if sm_scale is not None:
            self._sm_scale = sm_scale
        return self.run(q, paged_kv_cache, k_scale=k_scale, v_scale=v_scale, return_lse=True)


class MultiLevelCascadeAttentionWrapper:
    """This package's two-level cascade decode (FlashInfer's wrapper of this
    name, the subset a radix-shared batch needs): level 0 holds the prefix
    pages every request shares (one group: ``qo_indptr_arr[0] = [0, B]``),
    level 1 each request's pages after it (``qo_indptr_arr[1] = arange(B+1)``,
    one decode query per request). The prefix is attended once for all
    requests instead of once per request, as the reference's per-request
    decode (src/models/llama.py:230-245) does. Tables live on the device; the
    plan never synchronises with the host."""

    def __init__(self, num_levels: int, float_workspace_buffer: torch.Tensor,
                 kv_layout: str = "NHD", use_cuda_graph: bool = False, **kwargs) -> None:
        if num_levels != 2:
            raise NotImplementedError("only two levels (shared prefix + unique pages)")
        if kv_layout not in ("NHD", "HND"):
            raise KeyError(f"Invalid kv_layout {kv_layout}")
        self._ws = float_workspace_buffer
        self._kv_layout = kv_layout
        self._planned = False

    def reset_workspace_buffer(self, float_workspace_buffer: torch.Tensor, *args) -> None:
        self._ws = float_workspace_buffer

    def plan(self, qo_indptr_arr, paged_kv_indptr_arr, paged_kv_indices_arr,
             paged_kv_last_page_len_arr, num_qo_heads: int, num_kv_heads: int, head_dim: int,
             page_size: int, causal: bool = False, pos_encoding_mode: str = "NONE",
             window_left: int = -1, logits_soft_cap: Optional[float] = None,
             sm_scale: Optional[float] = None, q_data_type="float16", kv_data_type=None,
             **kwargs) -> None:
        _check_plan_options(pos_encoding_mode, window_left, logits_soft_cap)
        if len(qo_indptr_arr) != 2:
            raise NotImplementedError("only two levels (shared prefix + unique pages)")
        qo0, qo1 = qo_indptr_arr
        batch = qo1.numel() - 1
        if qo0.numel() != 2 or batch <= 0 or paged_kv_indptr_arr[0].numel() != 2:
            raise NotImplementedError("level 0 must be one prefix shared by every request")
        for name, t in (("qo_indptr_arr[0]", qo0), ("qo_indptr_arr[1]", qo1)):
            if t.device.type == "cpu":  # values are checked only where that costs no sync
                want = [0, batch] if name.endswith("[0]") else list(range(batch + 1))
                if t.tolist() != want:
                    raise NotImplementedError(f"{name} must be {want[:4]}...: one decode "
                                              "query per request, all sharing level 0")
        device = self._ws.device
        self._shared_indptr = _i32_on(paged_kv_indptr_arr[0], device, "paged_kv_indptr_arr[0]")
        self._shared_indices = _i32_on(paged_kv_indices_arr[0], device,
                                       "paged_kv_indices_arr[0]")
        self._shared_last = _i32_on(paged_kv_last_page_len_arr[0], device,
                                    "paged_kv_last_page_len_arr[0]")
        self._indptr = _i32_on(paged_kv_indptr_arr[1], device, "paged_kv_indptr_arr[1]")
        self._indices = _i32_on(paged_kv_indices_arr[1], device, "paged_kv_indices_arr[1]")
        self._last = _i32_on(paged_kv_last_page_len_arr[1], device,
                             "paged_kv_last_page_len_arr[1]")
        # an empty level (no shared prefix, or no request with pages of its
        # own) still passes a valid pointer; the kernels read no entry of it
        if self._shared_indices.numel() == 0:
            self._shared_indices = torch.zeros(1, dtype=torch.int32, device=device)
        if self._indices.numel() == 0:
            self._indices = torch.zeros(1, dtype=torch.int32, device=device)
        self._batch, self._hq, self._hkv, self._d, self._p = (batch, num_qo_heads, num_kv_heads,
                                                             head_dim, page_size)
        self._sm_scale = sm_scale
        _lib.check(_lib.load().pa_cascade_plan(
            _p(self._shared_indptr), _p(self._shared_last), self._shared_indices.numel(),
            _p(self._indptr), _p(self._last), batch, self._indices.numel(), num_qo_heads,
            num_kv_heads, head_dim, page_size,
            _p(self._ws), self._ws.numel() * self._ws.element_size(), _stream()),
            "MultiLevelCascadeAttentionWrapper.plan")
        _after("MultiLevelCascadeAttentionWrapper.plan")
        self._planned = True

    def run(self, q: torch.Tensor, paged_kv_cache, out: Optional[torch.Tensor] = None,
            lse: Optional[torch.Tensor] = None, return_lse: bool = False):
        return self._run(q, paged_kv_cache, None, out, lse, return_lse)

    def run_with_append(self, q: torch.Tensor, paged_kv_cache, append_key: torch.Tensor,
                        append_value: torch.Tensor, positions: torch.Tensor, *,
                        out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
                        return_lse: bool = False):
        """This package's extension: the decode step's
        ``append_paged_kv_cache(append_key, append_value, arange(B), positions, ...)``
        (positions global, as get_batch_indices_positions gives them) fused
        into the level-1 decode, then :meth:`run`'s levels and merge. Each
        appended position must fall inside its request's own (level-1) pages;
        the shared prefix pages are never written."""
        desc = kv_cache_desc(paged_kv_cache, self._kv_layout)
        if append_key.dtype != append_value.dtype or _dtype_code(append_key.dtype) != desc.dtype:
            raise ValueError("append_key / append_value must have the KV cache's dtype")
        for name, x in (("append_key", append_key), ("append_value", append_value)):
            _row_strides(x, name)
            if tuple(x.shape) != (self._batch, desc.num_kv_heads, desc.head_dim):
                raise ValueError(f"{name} must be [{self._batch}, {desc.num_kv_heads}, "
                                 f"{desc.head_dim}]")
        positions = _i32_on(positions, q.device, "positions")
        if positions.numel() != self._batch:
            raise ValueError("positions must hold one entry per request")
        return self._run(q, paged_kv_cache, (append_key, append_value, positions), out, lse,
                         return_lse)

    def _run(self, q, paged_kv_cache, append, out, lse, return_lse):
        if not self._planned:
            raise RuntimeError("plan() must be called before run()")
        desc = kv_cache_desc(paged_kv_cache, self._kv_layout)
        if (desc.num_kv_heads, desc.head_dim, desc.page_size) != (self._hkv, self._d, self._p):
            raise ValueError("paged_kv_cache geometry differs from the plan")
        if _dtype_code(q.dtype) != desc.dtype:
            raise NotImplementedError("q and the KV cache must have the same dtype")
        qsn, qsh = _row_strides(q, "q")
        if tuple(q.shape) != (self._batch, self._hq, self._d):
            raise ValueError(f"q must be [{self._batch}, {self._hq}, {self._d}]")
        if out is None:
            out = torch.empty_like(q, memory_format=torch.contiguous_format)
        elif not out.is_contiguous() or tuple(out.shape) != tuple(q.shape):
            raise ValueError("out must be a contiguous [batch, num_qo_heads, head_dim] tensor")
        if return_lse and lse is None:
            lse = torch.empty((self._batch, self._hq), dtype=torch.float32, device=q.device)
        scale = self._sm_scale if self._sm_scale is not None else 1.0 / math.sqrt(self._d)
        ws_bytes = self._ws.numel() * self._ws.element_size()
        if append is None:
            _lib.check(_lib.load().pa_cascade_run(
                _p(q), qsn, qsh, ctypes.byref(desc), _p(self._shared_indices), _p(self._indices),
                _p(self._indptr), _p(self._last), self._batch, self._hq, float(scale),
                _p(self._ws), ws_bytes, _p(out), _p(lse), _stream()),
                "MultiLevelCascadeAttentionWrapper.run")
            _after("MultiLevelCascadeAttentionWrapper.run")
        else:
            k, v, pos = append
            _lib.check(_lib.load().pa_cascade_append_run(
                _p(q), qsn, qsh, _p(k), k.stride(0), k.stride(1), _p(v), v.stride(0), v.stride(1),
                _p(pos), ctypes.byref(desc), _p(self._shared_indices), _p(self._indices),
                _p(self._indptr), _p(self._last), self._batch, self._hq, float(scale),
                _p(self._ws), ws_bytes, _p(out), _p(lse), _stream()),
                "MultiLevelCascadeAttentionWrapper.run_with_append")
            _after("MultiLevelCascadeAttentionWrapper.run_with_append")
        return (out, lse) if return_lse else out

    forward = run


def cascade_workspace_bytes(batch_size: int, num_qo_heads: int, num_kv_heads: int,
                            head_dim: int) -> int:
    """Workspace bytes MultiLevelCascadeAttentionWrapper needs (this package)."""
    return int(_lib.load().pa_cascade_workspace_bytes(batch_size, num_qo_heads, num_kv_heads,
                                                      head_dim))
