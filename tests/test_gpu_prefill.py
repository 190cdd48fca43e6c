"""Ragged / chunked prefill attention (tcgen05 kernel) against the CPU oracle.

Tolerance (bf16/fp16 in, fp32 accumulate): max-abs 2e-2, mean-abs 2e-3
against the fp32 gathered-page oracle with a bottom-right causal mask.
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_attention_cases
from oracle import attention

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3
DEV = "cuda"


def _t(a):
    return torch.as_tensor(np.asarray(a, dtype=np.int32)).to(DEV)


def _prefill(fi, q, pool_layer, qo_indptr, indptr, indices, last, causal=True, layout="HND",
             return_lse=False):
    hq, d = q.shape[1], q.shape[2]
    hkv = pool_layer.shape[2] if layout == "HND" else pool_layer.shape[3]
    ws = torch.empty(128 << 20, dtype=torch.uint8, device=DEV)
    w = fi.BatchPrefillWithPagedKVCacheWrapper(ws, layout)
    w.plan(_t(qo_indptr), _t(indptr), _t(indices), _t(last), hq, hkv, d, 16,
           q_data_type=q.dtype)
    if return_lse:
        w._causal = causal
        return w.run(q.to(DEV), pool_layer.to(DEV), return_lse=True)
    return w.forward(q.to(DEV), pool_layer.to(DEV), causal=causal)


def _check(got, want):
    mx, mean, ok = attention.compare(got, want, MAX_ABS, MEAN_ABS)
    assert ok, f"max-abs {mx:.3e} mean-abs {mean:.3e}"


@pytest.mark.parametrize("case", [c for c in load_attention_cases() if c["mode"] == "prefill"],
                         ids=lambda c: c["name"])
def test_prefill_matches_eager_and_flashinfer_fixtures(fi, case):
    got = _prefill(fi, case["q"], case["pool"], case["qo_indptr"], case["kv_indptr"],
                   case["kv_indices"], case["kv_last_page_len"], layout=case["layout"])
    _check(got, case["out"])
    z = np.load(os.path.join(GOLDEN, "flashinfer_outputs.npz"))
    _check(got, torch.from_numpy(z[case["name"] + "__out"]))


def _problem(workloads, geom, qo, prefix, seed, dtype=torch.bfloat16, extra_pages=5):
    return workloads.make_prefill_problem(geom, qo, prefix, seed=seed, dtype=dtype,
                                          extra_pages=extra_pages)


def _oracle(prob, causal=True, layout="HND", pool=None, requests=None):
    return attention.prefill(prob.q, prob.qo_indptr, (prob.pool[0] if pool is None else pool)
                             .float(), prob.kv_indptr, prob.kv_indices, prob.kv_last_page_len,
                             causal=causal, layout=layout, requests=requests)


def test_config3_shape_llama3_chunks_over_prefixes(fi, workloads):
    """Configuration 3 shape (reduced batch): 512-row chunks over cached
    prefixes U[0, 2048], Llama-3 attention geometry (32 q / 8 kv heads, D=128)."""
    g = torch.Generator().manual_seed(30)
    prefix = torch.randint(0, 2049, (4,), generator=g).numpy()
    prob = _problem(workloads, workloads.LLAMA3_8B, [512] * 4, prefix, seed=31)
    got = _prefill(fi, prob.q, prob.pool[0], prob.qo_indptr, prob.kv_indptr, prob.kv_indices,
                   prob.kv_last_page_len)
    want, _ = _oracle(prob)
    _check(got, want)


def test_tinyllama_geometry_ragged_chunks(fi, workloads):
    """TinyLlama geometry (g = 8, D = 64): ragged chunk lengths and prefixes,
    including a single-row chunk and a chunk starting mid-page."""
    prob = _problem(workloads, workloads.TINYLLAMA, [37, 1, 300, 16, 129],
                    [0, 100, 17, 16, 1000], seed=32)
    got = _prefill(fi, prob.q, prob.pool[0], prob.qo_indptr, prob.kv_indptr, prob.kv_indices,
                   prob.kv_last_page_len)
    want, _ = _oracle(prob)
    _check(got, want)


@pytest.mark.parametrize("geom_name", ["TINYLLAMA", "LLAMA3_8B"])
def test_non_causal_and_lse(fi, workloads, geom_name):
    geom = getattr(workloads, geom_name)
    prob = _problem(workloads, geom, [64, 200, 5], [10, 0, 300], seed=33)
    got, lse = _prefill(fi, prob.q, prob.pool[0], prob.qo_indptr, prob.kv_indptr,
                        prob.kv_indices, prob.kv_last_page_len, causal=False, return_lse=True)
    want, want_lse = _oracle(prob, causal=False)
    _check(got, want)
    assert torch.allclose(lse.cpu(), want_lse, atol=2e-3, rtol=1e-4)


def test_fp16_nhd_and_empty_request(fi, workloads):
    prob = _problem(workloads, workloads.LLAMA3_8B, [40, 0, 77], [20, 33, 0], seed=34,
                    dtype=torch.float16)
    got = _prefill(fi, prob.q, prob.pool[0], prob.qo_indptr, prob.kv_indptr, prob.kv_indices,
                   prob.kv_last_page_len)
    want, _ = _oracle(prob)
    _check(got, want)
    nhd = prob.pool[0].permute(0, 1, 3, 2, 4).contiguous()
    got2 = _prefill(fi, prob.q, nhd, prob.qo_indptr, prob.kv_indptr, prob.kv_indices,
                    prob.kv_last_page_len, layout="NHD")
    assert torch.equal(got.cpu(), got2.cpu())


def test_strided_q_from_fused_qkv(fi, workloads):
    """q as a view of the fused QKV projection output (llama.py:163-171)."""
    geom = workloads.TINYLLAMA
    prob = _problem(workloads, geom, [50, 70], [30, 0], seed=35)
    n = prob.q.shape[0]
    qkv = torch.randn(n, (32 + 8) * 64).to(torch.bfloat16)
    qkv[:, :32 * 64] = prob.q.reshape(n, -1)
    q_view = qkv.to(DEV).split([32 * 64, 4 * 64, 4 * 64], dim=-1)[0].view(-1, 32, 64)
    got = _prefill(fi, q_view, prob.pool[0], prob.qo_indptr, prob.kv_indptr, prob.kv_indices,
                   prob.kv_last_page_len)
    want, _ = _oracle(prob)
    _check(got, want)


@pytest.mark.parametrize("geom_name", ["TINYLLAMA", "LLAMA3_8B"])
def test_many_one_tile_items(fi, workloads, geom_name):
    """Runs of items with a single key tile: the output rows of tile 1 wait
    in the V ring stage of their item's last key tile until the next V load
    into that stage, so several stages hold rows at once (the ring has 2
    stages at head_dim 128, 4 at 64). Chunks of one or two item spans over
    prefixes shorter than a key tile, some ending inside tile 1 (rows
    written directly), then two launches on the same plan: identical
    outputs, both equal to the oracle's."""
    geom = getattr(workloads, geom_name)
    span = 2 * (128 // (geom.num_qo_heads // geom.num_kv_heads))
    g = torch.Generator().manual_seed(37)
    n = 48
    qo = [span * (1 + int(i % 3 == 0)) - (int(torch.randint(0, span // 2, (1,), generator=g))
                                          if i % 4 == 1 else 0) for i in range(n)]
    prefix = torch.randint(0, 128 - 2 * span + 1, (n,), generator=g).tolist()
    prob = _problem(workloads, geom, qo, prefix, seed=38)
    hq, d = prob.q.shape[1], prob.q.shape[2]
    hkv = prob.pool.shape[3]
    ws = torch.empty(128 << 20, dtype=torch.uint8, device=DEV)
    w = fi.BatchPrefillWithPagedKVCacheWrapper(ws, "HND")
    w.plan(_t(prob.qo_indptr), _t(prob.kv_indptr), _t(prob.kv_indices),
           _t(prob.kv_last_page_len), hq, hkv, d, 16, q_data_type=prob.q.dtype)
    q, pool = prob.q.to(DEV), prob.pool[0].to(DEV)
    first = w.forward(q, pool, causal=True)
    second = w.forward(q, pool, causal=True)
    assert torch.equal(first, second)
    want, _ = _oracle(prob)
    _check(first.cpu(), want)


def test_full_config3_sampled(fi, workloads):
    """Configuration 3 prefill part at full size: 16 chunks x 512 rows over
    prefixes U[0, 2048]; the oracle checks a sample of requests."""
    prob = workloads.config3_prefill(seed=0, device="cpu")
    got = _prefill(fi, prob.q, prob.pool[0], prob.qo_indptr, prob.kv_indptr, prob.kv_indices,
                   prob.kv_last_page_len)
    assert torch.isfinite(got).all()
    sample = [0, 5, 15]
    want, _ = _oracle(prob, requests=sample)
    rows = np.concatenate([np.arange(prob.qo_indptr[b], prob.qo_indptr[b + 1]) for b in sample])
    _check(got.cpu()[rows], want[rows])


def test_prefill_rejects_chunk_longer_than_cache(fi, lir, workloads):
    import importlib
    fa = importlib.import_module("llm-inference-runtime_b200.flashinfer_api")
    prob = _problem(workloads, workloads.TINYLLAMA, [20], [0], seed=36)
    saved = fa._CHECK
    fa._CHECK = False
    try:
        torch.cuda.synchronize()
        lir._lib.device_status()
        last = prob.kv_last_page_len.copy()
        last[0] = 3  # kv_len 3 < 20 query rows
        _prefill(fi, prob.q, prob.pool[0], prob.qo_indptr, prob.kv_indptr, prob.kv_indices, last)
        assert lir._lib.device_status() == lir._lib.PA_ERR_DEVICE_CHECK
    finally:
        fa._CHECK = saved


@pytest.mark.parametrize("hq,hkv,d", [(8, 8, 128), (16, 8, 64), (32, 2, 128), (64, 4, 64),
                                      (16, 16, 64)])
def test_every_gqa_group_size(fi, workloads, hq, hkv, d):
    """GQA packing for group sizes 1, 2, 16 (8 and 4 are the model configs):
    rows per tile = 128 / g queries x g heads."""
    geom = workloads.Geometry(num_qo_heads=hq, num_kv_heads=hkv, head_dim=d)
    prob = _problem(workloads, geom, [70, 1, 200], [33, 0, 500], seed=40 + hq + hkv)
    got, lse = _prefill(fi, prob.q, prob.pool[0], prob.qo_indptr, prob.kv_indptr,
                        prob.kv_indices, prob.kv_last_page_len, return_lse=True)
    want, want_lse = _oracle(prob)
    _check(got, want)
    assert torch.allclose(lse.cpu(), want_lse, atol=2e-3, rtol=1e-4)
