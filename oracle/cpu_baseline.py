"""Timed CPU arm: the oracle's fp32 eager attention over gathered pages.

Test / benchmark infrastructure (see oracle/__init__.py). Used only by
bench.py's cpu_baseline leg and its ``--impl reference`` arm. It restates
what the reference's eager path computes (oracle/attention.py) and runs it
with torch on every host core, on a seeded sample of the benchmark's
requests; throughput is reported in the GPU arm's unit (GB/s of bf16 KV
bytes the attention reads, plus q read and o written).
"""

from __future__ import annotations

import os
import time

import numpy as np
import torch

from . import attention


def _sample_problem(lengths: np.ndarray, geom, sample: int, seed: int = 2024):
    rng = np.random.default_rng(seed)
    idx = np.sort(rng.choice(len(lengths), size=min(sample, len(lengths)), replace=False))
    lens = lengths[idx].astype(np.int64)
    P = geom.page_size
    npages = (lens + P - 1) // P
    indptr = np.zeros(len(lens) + 1, dtype=np.int64)
    np.cumsum(npages, out=indptr[1:])
    N = int(indptr[-1])
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(N, generator=g).numpy()
    last = (lens - (npages - 1) * P).astype(np.int64)
    pool = torch.randn((N, 2, geom.num_kv_heads, P, geom.head_dim), generator=g)
    pool = pool.to(torch.bfloat16).to(torch.float32)
    q = torch.randn((len(lens), geom.num_qo_heads, geom.head_dim), generator=g)
    q = q.to(torch.bfloat16).to(torch.float32)
    nbytes = int(lens.sum()) * geom.kv_bytes_per_token + \
        2 * len(lens) * geom.num_qo_heads * geom.head_dim * 2
    return dict(idx=idx, lens=lens, indptr=indptr, indices=perm, last=last, pool=pool, q=q,
                nbytes=nbytes)


def _cores() -> int:
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def time_decode_sample(lengths: np.ndarray, geom, budget_s: float = 15.0,
                       sample: int = 16) -> dict:
    """Repeats the oracle decode of `sample` requests for about budget_s seconds."""
    cores = _cores()
    sp = _sample_problem(lengths, geom, sample)
    attention.decode(sp["q"], sp["pool"], sp["indptr"], sp["indices"], sp["last"])  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        attention.decode(sp["q"], sp["pool"], sp["indptr"], sp["indices"], sp["last"])
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    gbs = sp["nbytes"] * reps / el / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{len(sp['lens'])} requests of one layer (seeded), {reps} passes in "
                      f"{el:.1f} s; fp32 torch eager attention over gathered pages"}


def run_reference_arm(lengths: np.ndarray, geom, steps: int, warmup: int,
                      sample: int = 32) -> dict:
    """bench.py --impl reference: each step times the oracle on a bounded
    sample (`sample` requests of one layer) of the workload."""
    cores = _cores()
    sp = _sample_problem(lengths, geom, sample)
    for _ in range(warmup):
        attention.decode(sp["q"], sp["pool"], sp["indptr"], sp["indices"], sp["last"])
    t0 = time.perf_counter()
    for _ in range(steps):
        attention.decode(sp["q"], sp["pool"], sp["indptr"], sp["indices"], sp["last"])
    el = time.perf_counter() - t0
    return {"value": sp["nbytes"] * steps / el / 1e9, "ms_per_step": round(el / steps * 1e3, 3),
            "cores": cores,
            "sample": f"{len(sp['lens'])} requests of one layer per step (seeded); fp32 torch "
                      "eager attention over gathered pages"}


def time_prefill_sample(qo_lens: np.ndarray, prefix_lens: np.ndarray, geom,
                        budget_s: float = 10.0, sample: int = 2, seed: int = 2025) -> dict:
    """Repeats the oracle's causal prefill of `sample` chunks (seeded choice
    among the workload's chunks) for about budget_s seconds; TFLOP/s of the
    visible (unmasked) query-key pairs, 4 * D FLOPs each, as the GPU arm
    counts them."""
    cores = _cores()
    rng = np.random.default_rng(seed)
    idx = np.sort(rng.choice(len(qo_lens), size=min(sample, len(qo_lens)), replace=False))
    qo = np.asarray(qo_lens)[idx].astype(np.int64)
    pre = np.asarray(prefix_lens)[idx].astype(np.int64)
    kv = qo + pre
    P = geom.page_size
    npages = (kv + P - 1) // P
    kv_indptr = np.zeros(len(kv) + 1, dtype=np.int64)
    np.cumsum(npages, out=kv_indptr[1:])
    qo_indptr = np.zeros(len(qo) + 1, dtype=np.int64)
    np.cumsum(qo, out=qo_indptr[1:])
    N = int(kv_indptr[-1])
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(N, generator=g).numpy()
    last = (kv - (npages - 1) * P).astype(np.int64)
    pool = torch.randn((N, 2, geom.num_kv_heads, P, geom.head_dim), generator=g)
    pool = pool.to(torch.bfloat16).to(torch.float32)
    q = torch.randn((int(qo.sum()), geom.num_qo_heads, geom.head_dim), generator=g)
    q = q.to(torch.bfloat16).to(torch.float32)
    pairs = float(sum(int(n) * int(p) + int(n) * (int(n) + 1) // 2 for n, p in zip(qo, pre)))
    flops = 4.0 * geom.head_dim * geom.num_qo_heads * pairs
    attention.prefill(q, qo_indptr, pool, kv_indptr, perm, last)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        attention.prefill(q, qo_indptr, pool, kv_indptr, perm, last)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return {"value": round(flops * reps / el / 1e12, 5), "unit": "TFLOP/s", "cores": cores,
            "kind": "port",
            "sample": f"{len(qo)} of the workload's prefill chunks (seeded), {reps} passes in "
                      f"{el:.1f} s; fp32 torch eager causal attention over gathered pages"}
