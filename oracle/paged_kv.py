"""Integer / byte work of the paged-KV path, restated in numpy.

Test infrastructure (see oracle/__init__.py). Bit-exact targets.
"""

from __future__ import annotations

import numpy as np


def batch_indices_positions(append_indptr, seq_lens, nnz: int | None = None):
    """flashinfer.get_batch_indices_positions (src/models/llama.py:70-83).

    FlashInfer 0.6.11 (flashinfer/page.py get_batch_indices_positions and its
    kernel flashinfer/triton/page.py): batch_indices pre-filled with -1,
    positions with 0; row t of request b gets b and
    seq_lens[b] - (append_indptr[b+1] - append_indptr[b]) + (t - append_indptr[b]).
    """
    append_indptr = np.asarray(append_indptr, dtype=np.int64)
    seq_lens = np.asarray(seq_lens, dtype=np.int64)
    if nnz is None:
        nnz = int(append_indptr[-1])
    bi = np.full(nnz, -1, dtype=np.int32)
    pos = np.zeros(nnz, dtype=np.int32)
    for b in range(len(append_indptr) - 1):
        s, e = int(append_indptr[b]), int(append_indptr[b + 1])
        t = np.arange(s, min(e, nnz))
        bi[t] = b
        pos[t] = seq_lens[b] - (e - s) + (t - s)
    return bi, pos


def seq_lens(kv_indptr, kv_last_page_len, page_size: int):
    """flashinfer.get_seq_lens: (pages - 1) * P + last, 0 for requests without pages."""
    kv_indptr = np.asarray(kv_indptr, dtype=np.int64)
    last = np.asarray(kv_last_page_len, dtype=np.int64)
    pages = kv_indptr[1:] - kv_indptr[:-1]
    return np.where(pages > 0, (pages - 1) * page_size + last, 0)


def append_paged_kv_cache(key, value, batch_indices, positions, pool_layer, kv_indices,
                          kv_indptr, layout: str = "HND"):
    """flashinfer.append_paged_kv_cache (src/models/llama.py:188-210), in place.

    pool_layer: [N, 2, H, P, D] ("HND") or [N, 2, P, H, D] ("NHD"), a numpy
    array or torch tensor of any dtype, with key/value of the same kind (the
    copy is bit-exact). Row t of request b = batch_indices[t] at
    position pos lands in page kv_indices[kv_indptr[b] + pos // P], slot pos % P.
    Rows with batch index -1 are skipped.
    """
    kv_indices = np.asarray(kv_indices)
    kv_indptr = np.asarray(kv_indptr)
    P = pool_layer.shape[3] if layout == "HND" else pool_layer.shape[2]
    for t in range(key.shape[0]):
        b = int(batch_indices[t])
        if b < 0:
            continue
        pos = int(positions[t])
        page = int(kv_indices[int(kv_indptr[b]) + pos // P])
        slot = pos % P
        if layout == "HND":
            pool_layer[page, 0, :, slot, :] = key[t]
            pool_layer[page, 1, :, slot, :] = value[t]
        else:
            pool_layer[page, 0, slot, :, :] = key[t]
            pool_layer[page, 1, slot, :, :] = value[t]
    return pool_layer


def rope_reference(x, pos_ids, rotary_dim: int | None = None, interleave: bool = False,
                   rope_scale: float = 1.0, rope_theta: float = 1e4):
    """flashinfer.apply_rope_pos_ids_inplace math in float64 (llama.py:175-182).

    x: [nnz, H, D]. For i < rotary_dim/2: angle = pos / rope_scale *
    rope_theta^(-2i/rotary_dim); non-interleaved pairs (i, i + rotary_dim/2),
    interleaved pairs (2i, 2i+1). Dims >= rotary_dim are unchanged.
    """
    x = np.asarray(x, dtype=np.float64).copy()
    d = x.shape[-1]
    rd = d if rotary_dim is None else rotary_dim
    half = rd // 2
    i = np.arange(half, dtype=np.float64)
    freq = rope_theta ** (-2.0 * i / rd) / rope_scale
    ang = np.asarray(pos_ids, dtype=np.float64)[:, None] * freq[None, :]
    cs, sn = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    if interleave:
        a, b = x[..., 0:rd:2].copy(), x[..., 1:rd:2].copy()
        x[..., 0:rd:2] = a * cs - b * sn
        x[..., 1:rd:2] = b * cs + a * sn
    else:
        a, b = x[..., :half].copy(), x[..., half:rd].copy()
        x[..., :half] = a * cs - b * sn
        x[..., half:rd] = b * cs + a * sn
    return x


def merge_states(v, s):
    """Log-sum-exp merge of attention states (flashinfer.merge_states), float64.

    v [n, S, H, D], s [n, S, H] base-2 LSE -> (v_merged [n, H, D], s_merged [n, H]).
    """
    v = np.asarray(v, dtype=np.float64)
    s = np.asarray(s, dtype=np.float64)
    smax = s.max(axis=1, keepdims=True)
    w = np.exp2(s - smax)
    wsum = w.sum(axis=1)
    vm = (w[..., None] * v).sum(axis=1) / wsum[..., None]
    return vm, smax[:, 0] + np.log2(wsum)
