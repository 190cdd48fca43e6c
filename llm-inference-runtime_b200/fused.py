"""Fused QKV projection -> RoPE -> KV append (one tcgen05 GEMM launch).

Replaces the reference's per-layer sequence (src/models/llama.py:163-210):
`qkv = self.qkv_proj(hidden_states)` with the fused [q; k; v] weight
(_fuse_qkv_proj_plain, llama.py:256-280), the split into q / k / v,
`apply_rope_pos_ids_inplace(q, k, positions)` and
`append_paged_kv_cache(k, v, batch_indices, positions, ...)`.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from .flashinfer_api import _after, _dtype_code, _i32_on, _stream, kv_cache_desc


def supported(weight: torch.Tensor, num_qo_heads: int, num_kv_heads: int, head_dim: int,
              dtype: torch.dtype) -> bool:
    """Whether the fused kernel covers this projection geometry."""
    hidden = weight.size(1)
    return (head_dim in (64, 128) and hidden % 64 == 0
            and (num_qo_heads * head_dim) % 128 == 0 and (num_kv_heads * head_dim) % 128 == 0
            and weight.dtype == dtype and dtype in (torch.bfloat16, torch.float16)
            and weight.stride(1) == 1
            and weight.size(0) == (num_qo_heads + 2 * num_kv_heads) * head_dim)


def qkv_rope_append(x: torch.Tensor, weight: torch.Tensor, num_qo_heads: int,
                    batch_indices: torch.Tensor, positions: torch.Tensor, paged_kv_cache,
                    kv_indices: torch.Tensor, kv_indptr: torch.Tensor, kv_layout: str = "HND",
                    rotary_dim: Optional[int] = None, interleave: bool = False,
                    rope_scale: float = 1, rope_theta: float = 1e4,
                    q_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x [tokens, hidden], weight [(Hq + 2 Hkv) * D, hidden] -> rotated q
    [tokens, Hq, D]; the rotated k and v rows are written into the cache."""
    desc = kv_cache_desc(paged_kv_cache, kv_layout)
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be [tokens, hidden] with contiguous rows")
    if x.dtype != weight.dtype or _dtype_code(x.dtype) != desc.dtype:
        raise ValueError("x / weight must have the KV cache's dtype")
    d = desc.head_dim
    if not supported(weight, num_qo_heads, desc.num_kv_heads, d, x.dtype):
        raise NotImplementedError("projection geometry not covered by the fused kernel")
    if weight.size(1) != x.size(1):
        raise ValueError("weight and x disagree on hidden size")
    m = x.size(0)
    if q_out is None:
        q_out = torch.empty((m, num_qo_heads, d), dtype=x.dtype, device=x.device)
    if q_out.stride(2) != 1 or q_out.stride(1) != d:
        raise ValueError("q_out must be [tokens, Hq, D] with contiguous heads")
    if rotary_dim is None:
        rotary_dim = d
    device = x.device
    batch_indices = _i32_on(batch_indices, device, "batch_indices")
    positions = _i32_on(positions, device, "positions")
    kv_indices = _i32_on(kv_indices, device, "kv_indices")
    kv_indptr = _i32_on(kv_indptr, device, "kv_indptr")
    _lib.check(_lib.load().pa_qkv_rope_append(
        x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0), m, x.size(1),
        num_qo_heads, q_out.data_ptr(), q_out.stride(0), batch_indices.data_ptr(),
        positions.data_ptr(), rotary_dim, int(bool(interleave)), float(rope_scale),
        float(rope_theta), ctypes.byref(desc), kv_indices.data_ptr(), kv_indices.numel(),
        kv_indptr.data_ptr(), kv_indptr.numel() - 1, _stream()), "qkv_rope_append")
    _after("qkv_rope_append")
    return q_out
