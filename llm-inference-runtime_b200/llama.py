"""Drop-in replacement for the reference's ``src/models/llama.py``.

Same public names, arguments and global-state contract as the reference
module (src/models/llama.py:16-382), with every FlashInfer call routed to
the sm_100a kernels of this package (``flashinfer_api``):

* ``FlashInferState`` / ``PagedAttnState``   — llama.py:16-36
* ``init_flashinfer_state``                  — llama.py:39-67
* ``build_batch_indices_positions``          — llama.py:70-83
* ``plan_prefill`` / ``plan_decode``         — llama.py:86-147
* ``patched_llama_attention_forward``        — llama.py:150-249
* ``patch_llama_model``                      — llama.py:345-382

The engine swaps it in by importing these names from this module instead of
``models.llama`` (``step_executor.py:8-13``, ``async_engine.py:21``).
State is process-global and per device, like the reference's class
attributes: one engine per process, one device per process.
"""

from __future__ import annotations

import os
from typing import Optional, cast

import torch
from torch import nn

from . import flashinfer_api as flashinfer
from . import fused

# The fused QKV projection kernel (one launch: GEMM + RoPE + KV append) is
# opt-in: on a B200 it loses to cuBLAS + the fused RoPE/append kernel in GPU
# time at decode sizes (15-25 vs 10-13 us) and is on par at 8192 tokens
# (374-387 vs 372-397 us) while saving one launch. PA_FUSED_QKV=1 turns it on.
_FUSED_QKV = os.environ.get("PA_FUSED_QKV", "0") == "1"


class _StateMeta(type):
    """Class-level ``batch_indices`` / ``positions`` whose build can wait.

    ``build_batch_indices_positions`` called without ``nnz`` (the engine's
    own call, step_executor.py:155) records its inputs instead of reading
    ``nnz`` back from the device; the first patched layer of the step builds
    the tensors with ``nnz`` = its number of q rows. Assigning either
    attribute directly (the engine's decode path, step_executor.py:216-221)
    drops a pending build. Reading one while a build is pending builds it
    with ``nnz`` read from the device, the reference's behaviour.
    """

    def _get_batch_indices(cls):
        cls._resolve_pending(None)
        return cls._batch_indices

    def _set_batch_indices(cls, value):
        cls._pending = None
        cls._batch_indices = value

    def _get_positions(cls):
        cls._resolve_pending(None)
        return cls._positions

    def _set_positions(cls, value):
        cls._pending = None
        cls._positions = value

    batch_indices = property(_get_batch_indices, _set_batch_indices)
    positions = property(_get_positions, _set_positions)


class PagedAttnState(metaclass=_StateMeta):
    """Per-process attention state (the reference's FlashInferState)."""

    kv_pool: Optional[torch.Tensor] = None

    kv_indices: Optional[torch.Tensor] = None
    kv_indptr: Optional[torch.Tensor] = None
    kv_last_page_len: Optional[torch.Tensor] = None

    # batch_indices / positions: properties of the metaclass (above)
    _batch_indices: Optional[torch.Tensor] = None
    _positions: Optional[torch.Tensor] = None
    _pending: Optional[tuple] = None  # (append_indptr, seq_lens) awaiting nnz

    @classmethod
    def _resolve_pending(cls, nnz: Optional[int]) -> None:
        if cls._pending is None:
            return
        append_indptr, seq_lens = cls._pending
        if nnz is None:
            nnz = int(append_indptr[-1].item())
        cls._pending = None
        cls._batch_indices, cls._positions = flashinfer.get_batch_indices_positions(
            append_indptr, seq_lens, nnz)

    workspace_buffer: Optional[torch.Tensor] = None

    prefill_wrapper: Optional[flashinfer.BatchPrefillWithPagedKVCacheWrapper] = None
    decode_wrapper: Optional[flashinfer.BatchDecodeWithPagedKVCacheWrapper] = None

    page_size: int = 16
    dtype: Optional[torch.dtype] = None

    mode: str = "prefill"


FlashInferState = PagedAttnState

WORKSPACE_BYTES = 128 * 1024 * 1024  # the reference's workspace size (llama.py:49-53)


def init_flashinfer_state(*, kv_pool: torch.Tensor, page_size: int, device) -> None:
    """Borrows the allocator's pool and builds the two wrappers ("HND")."""
    PagedAttnState.kv_pool = kv_pool
    PagedAttnState.page_size = page_size
    PagedAttnState.dtype = kv_pool.dtype
    PagedAttnState.workspace_buffer = torch.empty(WORKSPACE_BYTES, dtype=torch.uint8,
                                                  device=device)
    PagedAttnState.prefill_wrapper = flashinfer.BatchPrefillWithPagedKVCacheWrapper(
        PagedAttnState.workspace_buffer, "HND")
    PagedAttnState.decode_wrapper = flashinfer.BatchDecodeWithPagedKVCacheWrapper(
        PagedAttnState.workspace_buffer, "HND")


init_paged_attn_state = init_flashinfer_state


def build_batch_indices_positions(append_indptr: torch.Tensor, seq_lens: torch.Tensor,
                                  nnz: Optional[int] = None) -> None:
    """Sets the per-row request ids and positions for RoPE and the KV append.

    The reference reads ``nnz`` back from the device (``.item()``,
    llama.py:74), which synchronises the host with the GPU every prefill
    step. Here, without ``nnz``, the build waits for the step's first
    patched layer, whose q rows number ``nnz`` (the step's input ids), so
    the call never synchronises and can be captured in a CUDA graph.
    Callers that know ``nnz`` may pass it; the build then runs at once.
    """
    if nnz is None:
        PagedAttnState._pending = (append_indptr, seq_lens)
        return
    (PagedAttnState.batch_indices,
     PagedAttnState.positions) = flashinfer.get_batch_indices_positions(
        append_indptr, seq_lens, nnz)


def plan_prefill(*, qo_indptr: torch.Tensor, kv_indptr: torch.Tensor, kv_indices: torch.Tensor,
                 kv_last_page_len: torch.Tensor, num_qo_heads: int, num_kv_heads: int,
                 head_dim: int) -> None:
    PagedAttnState.mode = "prefill"
    PagedAttnState.kv_indptr = kv_indptr
    PagedAttnState.kv_indices = kv_indices
    PagedAttnState.kv_last_page_len = kv_last_page_len
    pw = cast(flashinfer.BatchPrefillWithPagedKVCacheWrapper, PagedAttnState.prefill_wrapper)
    pw.begin_forward(qo_indptr, kv_indptr, kv_indices, kv_last_page_len, num_qo_heads,
                     num_kv_heads, head_dim, PagedAttnState.page_size,
                     q_data_type=PagedAttnState.dtype)


def plan_decode(*, kv_indptr: torch.Tensor, kv_indices: torch.Tensor,
                kv_last_page_len: torch.Tensor, num_qo_heads: int, num_kv_heads: int,
                head_dim: int) -> None:
    PagedAttnState.mode = "decode"
    PagedAttnState.kv_indptr = kv_indptr
    PagedAttnState.kv_indices = kv_indices
    PagedAttnState.kv_last_page_len = kv_last_page_len
    dw = cast(flashinfer.BatchDecodeWithPagedKVCacheWrapper, PagedAttnState.decode_wrapper)
    dw.begin_forward(kv_indptr, kv_indices, kv_last_page_len, num_qo_heads, num_kv_heads,
                     head_dim, PagedAttnState.page_size, q_data_type=PagedAttnState.dtype)


def paged_attention(attn, q_flat: torch.Tensor, k_flat: torch.Tensor,
                    v_flat: torch.Tensor) -> torch.Tensor:
    """RoPE -> KV append -> prefill or decode attention for one layer.

    The body of the reference's patched forward between the QKV and output
    projections (llama.py:173-245). Returns [rows, H_q, D].
    """
    PagedAttnState._resolve_pending(q_flat.shape[0])
    positions = cast(torch.Tensor, PagedAttnState.positions)
    kv_pool = cast(torch.Tensor, PagedAttnState.kv_pool)
    layer_kv_cache = kv_pool[attn.layer_idx]
    # RoPE on q / k and the KV append in one launch; same results as the
    # reference's apply_rope_pos_ids_inplace + append_paged_kv_cache pair.
    flashinfer.apply_rope_append(
        q_flat, k_flat, v_flat,
        batch_indices=cast(torch.Tensor, PagedAttnState.batch_indices),
        positions=positions, paged_kv_cache=layer_kv_cache,
        kv_indices=cast(torch.Tensor, PagedAttnState.kv_indices),
        kv_indptr=cast(torch.Tensor, PagedAttnState.kv_indptr),
        kv_last_page_len=cast(torch.Tensor, PagedAttnState.kv_last_page_len),
        kv_layout="HND", rope_theta=attn.rope_theta, rope_scale=attn.rope_scale,
        interleave=False)
    if PagedAttnState.mode == "prefill":
        pw = cast(flashinfer.BatchPrefillWithPagedKVCacheWrapper, PagedAttnState.prefill_wrapper)
        return pw.forward(q=q_flat, paged_kv_cache=layer_kv_cache, causal=True)
    dw = cast(flashinfer.BatchDecodeWithPagedKVCacheWrapper, PagedAttnState.decode_wrapper)
    return dw.forward(q=q_flat, paged_kv_cache=layer_kv_cache)


def paged_attention_fused(attn, x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """As paged_attention, starting from the layer input: the fused QKV
    projection kernel produces the rotated q and appends k / v, then the
    prefill or decode attention runs. Returns [rows, H_q, D]."""
    PagedAttnState._resolve_pending(x.shape[0])
    kv_pool = cast(torch.Tensor, PagedAttnState.kv_pool)
    layer_kv_cache = kv_pool[attn.layer_idx]
    q_flat = fused.qkv_rope_append(
        x, weight, attn.num_heads,
        batch_indices=cast(torch.Tensor, PagedAttnState.batch_indices),
        positions=cast(torch.Tensor, PagedAttnState.positions),
        paged_kv_cache=layer_kv_cache,
        kv_indices=cast(torch.Tensor, PagedAttnState.kv_indices),
        kv_indptr=cast(torch.Tensor, PagedAttnState.kv_indptr),
        kv_layout="HND", rope_theta=attn.rope_theta, rope_scale=attn.rope_scale,
        interleave=False)
    if PagedAttnState.mode == "prefill":
        pw = cast(flashinfer.BatchPrefillWithPagedKVCacheWrapper, PagedAttnState.prefill_wrapper)
        return pw.forward(q=q_flat, paged_kv_cache=layer_kv_cache, causal=True)
    dw = cast(flashinfer.BatchDecodeWithPagedKVCacheWrapper, PagedAttnState.decode_wrapper)
    return dw.forward(q=q_flat, paged_kv_cache=layer_kv_cache)


def patched_llama_attention_forward(self, hidden_states: torch.Tensor,
                                    position_embeddings=None, attention_mask=None,
                                    past_key_value=None, output_attentions=False,
                                    use_cache=False, cache_position=None, **kwargs):
    """Replacement LlamaAttention.forward (reference: llama.py:150-249)."""
    bsz, q_len, _ = hidden_states.shape
    proj = self.qkv_proj
    x = hidden_states.reshape(-1, hidden_states.size(-1))
    if (_FUSED_QKV and isinstance(proj, torch.nn.Linear) and proj.bias is None
            and x.stride(-1) == 1
            and fused.supported(proj.weight, self.num_heads, self.num_key_value_heads,
                                self.head_dim, x.dtype)):
        # projection, RoPE and KV append in one kernel (qkv never stored)
        out = paged_attention_fused(self, x, proj.weight)
    else:
        qkv = proj(hidden_states)
        q, k, v = qkv.split([self.q_size, self.kv_size, self.kv_size], dim=-1)
        q_flat = q.view(-1, self.num_heads, self.head_dim)
        k_flat = k.view(-1, self.num_key_value_heads, self.head_dim)
        v_flat = v.view(-1, self.num_key_value_heads, self.head_dim)
        out = paged_attention(self, q_flat, k_flat, v_flat)
    if PagedAttnState.mode == "prefill":
        out = out.reshape(bsz, q_len, self.num_heads * self.head_dim)
    else:
        out = out.reshape(bsz, 1, self.num_heads * self.head_dim)
    out = self.o_proj(out)
    return out, None


def _fuse_qkv_proj_plain(attn) -> nn.Linear:
    """One Linear holding [q; k; v] weights (reference: llama.py:256-280)."""
    q_proj, k_proj, v_proj = attn.q_proj, attn.k_proj, attn.v_proj
    fused = nn.Linear(q_proj.in_features,
                      q_proj.out_features + k_proj.out_features + v_proj.out_features,
                      bias=False, device=q_proj.weight.device, dtype=q_proj.weight.dtype)
    with torch.no_grad():
        fused.weight.copy_(torch.cat([q_proj.weight, k_proj.weight, v_proj.weight], dim=0))
    return fused


def patch_llama_model(model) -> None:
    """Fuses QKV and rebinds every layer's attention forward (llama.py:345-382).

    The 4-bit (bitsandbytes) fuse path of the reference is not provided;
    quantised projections raise.
    """
    from transformers.models.llama.modeling_llama import LlamaAttention

    rope_theta = getattr(model.config, "rope_theta", 10000.0)
    rope_scaling = getattr(model.config, "rope_scaling", None)
    if rope_scaling is not None:
        rope_type = rope_scaling.get("rope_type", rope_scaling.get("type"))
        if rope_type not in (None, "default", "linear"):
            raise NotImplementedError(
                f"model.config.rope_scaling type '{rope_type}' is not representable by a "
                "linear rope_scale factor")
        rope_scale = rope_scaling.get("factor", 1.0)
    else:
        rope_scale = 1.0

    for idx, layer in enumerate(model.model.layers):
        attn = layer.self_attn
        if not isinstance(attn.q_proj, nn.Linear):
            raise NotImplementedError("only plain nn.Linear q/k/v projections are supported")
        attn.layer_idx = idx
        attn.num_heads = model.config.num_attention_heads
        attn.num_key_value_heads = model.config.num_key_value_heads
        attn.head_dim = model.config.hidden_size // model.config.num_attention_heads
        attn.q_size = attn.num_heads * attn.head_dim
        attn.kv_size = attn.num_key_value_heads * attn.head_dim
        attn.rope_theta = rope_theta
        attn.rope_scale = rope_scale
        attn.qkv_proj = _fuse_qkv_proj_plain(attn)
        del attn.q_proj, attn.k_proj, attn.v_proj
        attn.forward = patched_llama_attention_forward.__get__(attn, LlamaAttention)
