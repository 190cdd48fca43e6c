"""Device-side step tables (the Python loops of the reference's StepExecutor).

`build_decode_tables` / `build_prefill_tables` produce, on the device, the
CSR page tables, batch indices and positions that
src/engine/runtime/step_executor.py builds in Python lists every step
(:98-155 for prefill chunks, :204-225 for decode) and then copies to the GPU.
Inputs are the sequences' block tables as a padded int32 matrix plus their
lengths, already on the device; nothing is synchronised, so a step built
this way can be captured in a CUDA graph. Results are bit-identical to the
reference's lists.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from . import _lib


def _i32(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.int32:
        raise TypeError(f"{name} must be int32")
    if not t.is_cuda:
        raise ValueError(f"{name} must be on the GPU")
    return t.contiguous()


def _block_tables(block_tables: torch.Tensor):
    if block_tables.dim() != 2 or block_tables.stride(1) != 1:
        raise ValueError("block_tables must be [batch, max_blocks] with contiguous rows")
    if block_tables.dtype != torch.int32 or not block_tables.is_cuda:
        raise TypeError("block_tables must be int32 on the GPU")
    return block_tables, block_tables.stride(0)


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def build_decode_tables(block_tables: torch.Tensor, num_blocks: torch.Tensor,
                        seq_lens: torch.Tensor, page_size: int,
                        kv_indices_capacity: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """Decode tables for sequences with get_len = seq_lens and block tables
    block_tables[b, :num_blocks[b]] (the whole table is used, as the
    reference does). counts = [batch, batch, error]."""
    bt, stride = _block_tables(block_tables)
    num_blocks = _i32(num_blocks, "num_blocks")
    seq_lens = _i32(seq_lens, "seq_lens")
    B = seq_lens.numel()
    dev = seq_lens.device
    cap = bt.numel() if kv_indices_capacity is None else int(kv_indices_capacity)
    out = {
        "kv_indptr": torch.empty(B + 1, dtype=torch.int32, device=dev),
        "kv_indices": torch.empty(max(cap, 1), dtype=torch.int32, device=dev),
        "kv_last_page_len": torch.empty(B, dtype=torch.int32, device=dev),
        "batch_indices": torch.empty(B, dtype=torch.int32, device=dev),
        "positions": torch.empty(B, dtype=torch.int32, device=dev),
        "counts": torch.empty(3, dtype=torch.int32, device=dev),
    }
    _lib.check(_lib.load().pa_build_decode_tables(
        _p(bt), stride, _p(num_blocks), _p(seq_lens), B, int(page_size), _p(out["kv_indptr"]),
        _p(out["kv_indices"]), cap, _p(out["kv_last_page_len"]), _p(out["batch_indices"]),
        _p(out["positions"]), _p(out["counts"]), _stream()), "build_decode_tables")
    return out


def build_prefill_tables(block_tables: torch.Tensor, num_blocks: torch.Tensor,
                         prompt_lens: torch.Tensor, computed_lens: torch.Tensor,
                         chunk_lens: torch.Tensor, page_size: int, rows_capacity: int,
                         kv_indices_capacity: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """Prefill-chunk tables: chunk = min(chunk_lens, prompt_lens -
    computed_lens); sequences with an empty chunk are dropped and `active`
    lists the input index of each output slot. counts = [active sequences,
    rows, error]; rows_capacity bounds the total chunk rows."""
    bt, stride = _block_tables(block_tables)
    num_blocks = _i32(num_blocks, "num_blocks")
    prompt_lens = _i32(prompt_lens, "prompt_lens")
    computed_lens = _i32(computed_lens, "computed_lens")
    chunk_lens = _i32(chunk_lens, "chunk_lens")
    B = computed_lens.numel()
    dev = computed_lens.device
    cap = bt.numel() if kv_indices_capacity is None else int(kv_indices_capacity)
    rows = int(rows_capacity)
    out = {
        "qo_indptr": torch.empty(B + 1, dtype=torch.int32, device=dev),
        "kv_indptr": torch.empty(B + 1, dtype=torch.int32, device=dev),
        "kv_indices": torch.empty(max(cap, 1), dtype=torch.int32, device=dev),
        "kv_last_page_len": torch.empty(B, dtype=torch.int32, device=dev),
        "seq_lens": torch.empty(B, dtype=torch.int32, device=dev),
        "active": torch.empty(B, dtype=torch.int32, device=dev),
        "batch_indices": torch.empty(max(rows, 1), dtype=torch.int32, device=dev),
        "positions": torch.empty(max(rows, 1), dtype=torch.int32, device=dev),
        "counts": torch.empty(3, dtype=torch.int32, device=dev),
    }
    _lib.check(_lib.load().pa_build_prefill_tables(
        _p(bt), stride, _p(num_blocks), _p(prompt_lens), _p(computed_lens), _p(chunk_lens), B,
        int(page_size), _p(out["qo_indptr"]), _p(out["kv_indptr"]), _p(out["kv_indices"]), cap,
        _p(out["kv_last_page_len"]), _p(out["seq_lens"]), _p(out["active"]),
        _p(out["batch_indices"]), _p(out["positions"]), rows, _p(out["counts"]), _stream()),
        "build_prefill_tables")
    return out


def fork_pages(kv_pool: torch.Tensor, src_pages: torch.Tensor, dst_pages: torch.Tensor) -> None:
    """Copy-on-write fork: page src_pages[i] -> dst_pages[i] in every layer of
    the engine's pool [L, N, 2, H_kv, P, D] (or one layer [N, 2, H_kv, P, D]),
    K and V of every head. dst pages must be distinct and not sources."""
    pool = kv_pool if kv_pool.dim() == 6 else kv_pool.unsqueeze(0)
    if pool.dim() != 6 or not pool.is_cuda:
        raise ValueError("kv_pool must be [L, N, 2, H_kv, P, D] (or one layer) on the GPU")
    if pool[0, 0].is_contiguous() is False or pool.stride(1) != pool[0, 0].numel():
        raise ValueError("each page of a layer must be one contiguous block")
    src = _i32(src_pages, "src_pages")
    dst = _i32(dst_pages, "dst_pages")
    if src.numel() != dst.numel():
        raise ValueError("src_pages and dst_pages must have the same length")
    es = pool.element_size()
    _lib.check(_lib.load().pa_fork_pages(
        _p(pool), pool.stride(0) * es, pool.size(0), pool.stride(1) * es, pool[0, 0].numel() * es,
        pool.size(1), _p(src), _p(dst), src.numel(), _stream()), "fork_pages")
