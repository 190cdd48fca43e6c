"""fp32 attention over gathered pages — the oracle for decode and prefill.

Test infrastructure (see oracle/__init__.py).

The reference's attention is FlashInfer (GPU only). The eager path it
patches out is transformers' LlamaAttention: ``repeat_kv`` then
``eager_attention_forward`` (transformers/models/llama/modeling_llama.py,
repeat_kv and eager_attention_forward: scores = q k^T * head_dim**-0.5 +
causal mask, softmax in float32, then @ v). This module applies that math,
in float32, to K/V gathered from the paged pool with the engine's CSR
contract (kv_indptr / kv_indices / kv_last_page_len, HND or NHD pages):

  K_b = pool[kv_indices[kv_indptr[b]:kv_indptr[b+1]], 0] -> [H_kv, pages*P, D],
  truncated to kv_len_b = (pages - 1) * P + kv_last_page_len[b]; same for V.

Causal masks are bottom-right aligned like FlashInfer's prefill
(src/models/llama.py:221 passes causal=True): query row i of a request with
qo_len rows sees key j iff j <= i + kv_len - qo_len.
"""

from __future__ import annotations

import math

import numpy as np
import torch

LOG2E = 1.4426950408889634


def _np_i64(x):
    if isinstance(x, torch.Tensor):
        x = x.detach().cpu().numpy()
    return np.asarray(x, dtype=np.int64)


def kv_len(kv_indptr, kv_last_page_len, b: int, page_size: int) -> int:
    kv_indptr = _np_i64(kv_indptr)
    n = int(kv_indptr[b + 1] - kv_indptr[b])
    return 0 if n == 0 else (n - 1) * page_size + int(_np_i64(kv_last_page_len)[b])


def gather_kv(pool_layer: torch.Tensor, kv_indptr, kv_indices, kv_last_page_len, b: int,
              layout: str = "HND"):
    """K, V of request b as float32 [H_kv, kv_len, D]."""
    kv_indptr = _np_i64(kv_indptr)
    kv_indices = _np_i64(kv_indices)
    pages = torch.as_tensor(kv_indices[kv_indptr[b]:kv_indptr[b + 1]], dtype=torch.long)
    blk = pool_layer.index_select(0, pages.to(pool_layer.device)).to(torch.float32).cpu()
    if layout == "HND":
        n, _, h, p, d = blk.shape
        k = blk[:, 0].permute(1, 0, 2, 3).reshape(h, n * p, d)
        v = blk[:, 1].permute(1, 0, 2, 3).reshape(h, n * p, d)
    else:
        n, _, p, h, d = blk.shape
        k = blk[:, 0].permute(2, 0, 1, 3).reshape(h, n * p, d)
        v = blk[:, 1].permute(2, 0, 1, 3).reshape(h, n * p, d)
    L = kv_len(kv_indptr, kv_last_page_len, b, p)
    return k[:, :L], v[:, :L]


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """[H_kv, L, D] -> [H_kv * n_rep, L, D]; q head h reads kv head h // n_rep."""
    h, L, d = x.shape
    return x[:, None].expand(h, n_rep, L, d).reshape(h * n_rep, L, d)


def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
           causal: bool = False):
    """q [R, Hq, D], k/v [H_kv, L, D] float32 -> (o [R, Hq, D], lse2 [R, Hq]).

    Rows are the last R query positions of the request (bottom-right causal).
    lse2 is the base-2 log-sum-exp of scale * log2(e) * q.k (FlashInfer's).
    """
    R, hq, d = q.shape
    hkv, L, _ = k.shape
    if L == 0:
        return torch.zeros((R, hq, d)), torch.full((R, hq), -math.inf)
    kk = repeat_kv(k, hq // hkv)
    vv = repeat_kv(v, hq // hkv)
    scores = torch.einsum("rhd,hld->hrl", q.to(torch.float32), kk) * scale
    if causal:
        qpos = torch.arange(R)[:, None] + (L - R)
        kpos = torch.arange(L)[None, :]
        scores = scores.masked_fill((kpos > qpos)[None], float("-inf"))
    lse = torch.logsumexp(scores, dim=-1)
    probs = torch.softmax(scores, dim=-1, dtype=torch.float32)
    o = torch.einsum("hrl,hld->rhd", probs, vv)
    return o, (lse * LOG2E).transpose(0, 1)


def decode(q: torch.Tensor, pool_layer: torch.Tensor, kv_indptr, kv_indices, kv_last_page_len,
           layout: str = "HND", sm_scale: float | None = None, requests=None):
    """Batched decode: q [B, Hq, D] -> (o [B, Hq, D], lse2 [B, Hq]) float32.

    ``requests`` restricts the work to a subset of request ids (the other
    rows are left zero), for sampled checks at full size.
    """
    B, hq, d = q.shape
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(d)
    out = torch.zeros((B, hq, d), dtype=torch.float32)
    lse = torch.full((B, hq), -math.inf, dtype=torch.float32)
    qf = q.detach().to(torch.float32).cpu()
    for b in (range(B) if requests is None else requests):
        k, v = gather_kv(pool_layer, kv_indptr, kv_indices, kv_last_page_len, b, layout)
        o, l2 = attend(qf[b:b + 1], k, v, scale, causal=False)
        out[b] = o[0]
        lse[b] = l2[0]
    return out, lse


def prefill(q: torch.Tensor, qo_indptr, pool_layer: torch.Tensor, kv_indptr, kv_indices,
            kv_last_page_len, causal: bool = True, layout: str = "HND",
            sm_scale: float | None = None, requests=None):
    """Ragged prefill: q [nnz, Hq, D] -> (o [nnz, Hq, D], lse2 [nnz, Hq]) float32."""
    qo_indptr = _np_i64(qo_indptr)
    nnz, hq, d = q.shape
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(d)
    out = torch.zeros((nnz, hq, d), dtype=torch.float32)
    lse = torch.full((nnz, hq), -math.inf, dtype=torch.float32)
    qf = q.detach().to(torch.float32).cpu()
    B = len(qo_indptr) - 1
    for b in (range(B) if requests is None else requests):
        s, e = int(qo_indptr[b]), int(qo_indptr[b + 1])
        if e == s:
            continue
        k, v = gather_kv(pool_layer, kv_indptr, kv_indices, kv_last_page_len, b, layout)
        o, l2 = attend(qf[s:e], k, v, scale, causal=causal)
        out[s:e] = o
        lse[s:e] = l2
    return out, lse


def compare(got: torch.Tensor, want: torch.Tensor, max_abs: float = 2e-2,
            mean_abs: float = 2e-3):
    """Tolerance of the north star for bf16 outputs against this fp32 oracle."""
    diff = (got.detach().to(torch.float32).cpu() - want.to(torch.float32)).abs()
    return float(diff.max()), float(diff.mean()), bool(diff.max() <= max_abs
                                                       and diff.mean() <= mean_abs)
