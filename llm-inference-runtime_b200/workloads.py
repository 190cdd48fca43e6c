"""Seeded synthetic workloads of the benchmark configurations.

The reference measures with live HTTP traffic (ShareGPT prompts, absent
here); these generators stand in with the shapes, sizes and value
distributions of the five configurations the paged-attention path is
judged on. Draw order is fixed per seed: lengths -> page permutation ->
q -> new K/V rows; the pool itself is filled from a second generator
(seed + 1), on the device for large pools.

Page tables follow the engine's contract (src/engine/runtime/
step_executor.py:132-155, 204-225): kv_indptr [B+1], kv_indices
[sum pages], kv_last_page_len [B] in [1, P], int32.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch


@dataclass(frozen=True)
class Geometry:
    num_qo_heads: int
    num_kv_heads: int
    head_dim: int
    page_size: int = 16
    num_layers: int = 1

    @property
    def group(self) -> int:
        return self.num_qo_heads // self.num_kv_heads

    @property
    def kv_bytes_per_token(self) -> int:
        """K + V bytes of one token of one layer at 2 bytes per element."""
        return 2 * self.num_kv_heads * self.head_dim * 2


TINYLLAMA = Geometry(num_qo_heads=32, num_kv_heads=4, head_dim=64, page_size=16, num_layers=22)
LLAMA3_8B = Geometry(num_qo_heads=32, num_kv_heads=8, head_dim=128, page_size=16, num_layers=1)


def tables_from_lengths(lengths: np.ndarray, page_ids: np.ndarray, page_size: int):
    """CSR tables for requests of the given KV lengths over the given pages."""
    lengths = np.asarray(lengths, dtype=np.int64)
    npages = (lengths + page_size - 1) // page_size
    indptr = np.zeros(len(lengths) + 1, dtype=np.int64)
    np.cumsum(npages, out=indptr[1:])
    indices = np.asarray(page_ids[: indptr[-1]], dtype=np.int32)
    last = np.where(npages > 0, lengths - (npages - 1) * page_size, 0).astype(np.int32)
    return indptr.astype(np.int32), indices, last


@dataclass
class DecodeProblem:
    geom: Geometry
    lengths: np.ndarray          # KV length of each request (the appended token included)
    kv_indptr: np.ndarray
    kv_indices: np.ndarray
    kv_last_page_len: np.ndarray
    num_pages: int
    pool: torch.Tensor           # [layers, N, 2, H_kv, P, D] ("HND")
    q: torch.Tensor              # [B, H_q, D]
    k_new: torch.Tensor          # [B, H_kv, D]
    v_new: torch.Tensor
    positions: np.ndarray        # position of the appended token = length - 1
    extra: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return len(self.lengths)

    def device_tables(self, device):
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
        return t(self.kv_indptr), t(self.kv_indices), t(self.kv_last_page_len)

    def decode_bytes_per_layer(self) -> int:
        """Algorithmic HBM bytes of one decode launch: every key and value of
        every request once, q read once, o written once."""
        g = self.geom
        return int(self.lengths.sum()) * g.kv_bytes_per_token + \
            2 * self.batch * g.num_qo_heads * g.head_dim * 2

    def append_bytes_per_layer(self) -> int:
        """One new K and V row per request: read once, written once."""
        g = self.geom
        return 2 * self.batch * g.num_kv_heads * g.head_dim * 2 * 2


def _fill_normal(t: torch.Tensor, seed: int) -> None:
    gen = torch.Generator(device=t.device).manual_seed(seed)
    flat = t.view(-1)
    step = 1 << 28
    for s in range(0, flat.numel(), step):
        chunk = flat[s:s + step]
        chunk.copy_(torch.randn(chunk.shape, generator=gen, device=t.device, dtype=torch.float32))


def make_decode_problem(geom: Geometry, batch: int, lo: int, hi: int, seed: int = 0,
                        device: str | torch.device = "cpu", dtype=torch.bfloat16,
                        num_layers: Optional[int] = None, pool_pages: Optional[int] = None,
                        append: bool = True, lengths: Optional[np.ndarray] = None,
                        ) -> DecodeProblem:
    """Decode batch: context lengths ~ U[lo, hi], +1 appended token if `append`.

    Page ids are a random permutation of the pool; q, new K/V rows and the
    pool are i.i.d. N(0, 1) rounded to `dtype`.
    """
    layers = num_layers or geom.num_layers
    P = geom.page_size
    g = torch.Generator().manual_seed(seed)
    if lengths is None:
        ctx = torch.randint(lo, hi + 1, (batch,), generator=g).numpy().astype(np.int64)
        lengths = ctx + (1 if append else 0)
    lengths = np.asarray(lengths, dtype=np.int64)
    total_pages = int(((lengths + P - 1) // P).sum())
    N = pool_pages if pool_pages is not None else total_pages
    if N < total_pages:
        raise ValueError(f"pool of {N} pages cannot hold {total_pages}")
    perm = torch.randperm(N, generator=g).numpy()
    indptr, indices, last = tables_from_lengths(lengths, perm, P)
    q = torch.randn((batch, geom.num_qo_heads, geom.head_dim), generator=g)
    k_new = torch.randn((batch, geom.num_kv_heads, geom.head_dim), generator=g)
    v_new = torch.randn((batch, geom.num_kv_heads, geom.head_dim), generator=g)
    pool = torch.empty((layers, N, 2, geom.num_kv_heads, P, geom.head_dim), dtype=dtype,
                       device=device)
    _fill_normal(pool, seed + 1)
    return DecodeProblem(geom=geom, lengths=lengths, kv_indptr=indptr, kv_indices=indices,
                         kv_last_page_len=last, num_pages=N, pool=pool,
                         q=q.to(dtype).to(device), k_new=k_new.to(dtype).to(device),
                         v_new=v_new.to(dtype).to(device), positions=lengths - 1)


def make_shared_prefix_problem(geom: Geometry, batch: int = 64, prefix: int = 2048,
                               lo: int = 32, hi: int = 256, seed: int = 0,
                               device: str | torch.device = "cpu", dtype=torch.bfloat16,
                               num_layers: int = 1) -> DecodeProblem:
    """Configuration 4: `batch` requests whose tables start with the same
    prefix / P page ids (the refcounted pages a radix-cache hit hands out),
    followed by unique suffix pages for suffixes ~ U[lo, hi] (+1 appended
    token). extra["unique_pages"] counts the distinct pages referenced."""
    P = geom.page_size
    assert prefix % P == 0
    g = torch.Generator().manual_seed(seed)
    suffix = torch.randint(lo, hi + 1, (batch,), generator=g).numpy().astype(np.int64) + 1
    lengths = prefix + suffix
    shared_pages = prefix // P
    suffix_pages = (suffix + P - 1) // P
    N = shared_pages + int(suffix_pages.sum())
    perm = torch.randperm(N, generator=g).numpy().astype(np.int32)
    shared = perm[:shared_pages]
    rest = perm[shared_pages:]
    tables, o = [], 0
    for n in suffix_pages:
        tables.append(np.concatenate([shared, rest[o:o + n]]))
        o += n
    indptr = np.zeros(batch + 1, dtype=np.int32)
    np.cumsum([len(t) for t in tables], out=indptr[1:])
    indices = np.concatenate(tables).astype(np.int32)
    last = (suffix - (suffix_pages - 1) * P).astype(np.int32)
    q = torch.randn((batch, geom.num_qo_heads, geom.head_dim), generator=g)
    k_new = torch.randn((batch, geom.num_kv_heads, geom.head_dim), generator=g)
    v_new = torch.randn((batch, geom.num_kv_heads, geom.head_dim), generator=g)
    pool = torch.empty((num_layers, N, 2, geom.num_kv_heads, P, geom.head_dim), dtype=dtype,
                       device=device)
    _fill_normal(pool, seed + 1)
    return DecodeProblem(geom=geom, lengths=lengths, kv_indptr=indptr, kv_indices=indices,
                         kv_last_page_len=last, num_pages=N, pool=pool,
                         q=q.to(dtype).to(device), k_new=k_new.to(dtype).to(device),
                         v_new=v_new.to(dtype).to(device), positions=lengths - 1,
                         extra={"unique_pages": N, "shared_pages": shared_pages})


@dataclass
class PrefillProblem:
    geom: Geometry
    qo_lens: np.ndarray
    prefix_lens: np.ndarray
    qo_indptr: np.ndarray
    kv_indptr: np.ndarray
    kv_indices: np.ndarray
    kv_last_page_len: np.ndarray
    num_pages: int
    pool: torch.Tensor   # [layers, N, 2, H_kv, P, D], chunk K/V already in place
    q: torch.Tensor      # [sum qo, H_q, D]

    @property
    def kv_lens(self) -> np.ndarray:
        return self.prefix_lens + self.qo_lens

    def flops(self, causal: bool = True) -> int:
        """4 * D * H_q * (visible query-key pairs); causal counts pairs j <= i + prefix."""
        g = self.geom
        pairs = 0
        for n, p in zip(self.qo_lens.tolist(), self.prefix_lens.tolist()):
            pairs += n * p + n * (n + 1) // 2 if causal else n * (n + p)
        return 4 * g.head_dim * g.num_qo_heads * pairs

    def device_tables(self, device):
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
        return (t(self.qo_indptr), t(self.kv_indptr), t(self.kv_indices),
                t(self.kv_last_page_len))


def make_prefill_problem(geom: Geometry, qo_lens, prefix_lens, seed: int = 0,
                         device: str | torch.device = "cpu", dtype=torch.bfloat16,
                         num_layers: int = 1, extra_pages: int = 0) -> PrefillProblem:
    """Chunked prefill: request b appends qo_lens[b] rows after prefix_lens[b] cached keys."""
    P = geom.page_size
    g = torch.Generator().manual_seed(seed)
    qo_lens = np.asarray(qo_lens, dtype=np.int64)
    prefix_lens = np.asarray(prefix_lens, dtype=np.int64)
    kv_lens = qo_lens + prefix_lens
    total_pages = int(((kv_lens + P - 1) // P).sum())
    N = total_pages + extra_pages
    perm = torch.randperm(N, generator=g).numpy()
    indptr, indices, last = tables_from_lengths(kv_lens, perm, P)
    qo_indptr = np.zeros(len(qo_lens) + 1, dtype=np.int32)
    np.cumsum(qo_lens, out=qo_indptr[1:])
    q = torch.randn((int(qo_lens.sum()), geom.num_qo_heads, geom.head_dim), generator=g)
    pool = torch.empty((num_layers, N, 2, geom.num_kv_heads, P, geom.head_dim), dtype=dtype,
                       device=device)
    _fill_normal(pool, seed + 1)
    return PrefillProblem(geom=geom, qo_lens=qo_lens, prefix_lens=prefix_lens,
                          qo_indptr=qo_indptr, kv_indptr=indptr, kv_indices=indices,
                          kv_last_page_len=last, num_pages=N, pool=pool,
                          q=q.to(dtype).to(device))


def config3_prefill(seed: int = 0, device="cpu", dtype=torch.bfloat16,
                    chunks: int = 16, chunk: int = 512, max_prefix: int = 2048) -> PrefillProblem:
    """Configuration 3, prefill part: 16 chunks of 512 rows over prefixes ~ U[0, 2048]."""
    g = torch.Generator().manual_seed(seed)
    prefix = torch.randint(0, max_prefix + 1, (chunks,), generator=g).numpy()
    return make_prefill_problem(LLAMA3_8B, [chunk] * chunks, prefix, seed=seed + 7,
                                device=device, dtype=dtype)


def round_robin(batch: int, world: int, rank: int) -> np.ndarray:
    """Request ids that GPU `rank` of `world` owns: i with i mod world == rank."""
    return np.arange(rank, batch, world)


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


__all__ = ["Geometry", "TINYLLAMA", "LLAMA3_8B", "DecodeProblem", "PrefillProblem",
           "make_decode_problem", "make_prefill_problem", "config3_prefill", "tables_from_lengths",
           "round_robin", "ceil_div", "math"]
