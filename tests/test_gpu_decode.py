"""Paged decode attention on the GPU against the CPU oracle.

Tolerance (bf16/fp16 in, fp32 accumulate): max-abs 2e-2, mean-abs 2e-3
against the fp32 gathered-page oracle (oracle/attention.py).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import load_attention_cases
from oracle import attention, bookkeeping

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3
DEV = "cuda"


def _ws():
    return torch.empty(128 << 20, dtype=torch.uint8, device=DEV)


def _decode(fi, q, pool_layer, indptr, indices, last, layout="HND", return_lse=False,
            wrapper=None):
    hq, d = q.shape[1], q.shape[2]
    hkv = pool_layer.shape[2] if layout == "HND" else pool_layer.shape[3]
    t = lambda a: torch.as_tensor(np.asarray(a, dtype=np.int32)).to(DEV)  # noqa: E731
    w = wrapper or fi.BatchDecodeWithPagedKVCacheWrapper(_ws(), layout)
    w.plan(t(indptr), t(indices), t(last), hq, hkv, d, 16, q_data_type=q.dtype)
    return w.run(q.to(DEV), pool_layer.to(DEV), return_lse=return_lse)


def _check(got, want):
    mx, mean, ok = attention.compare(got, want, MAX_ABS, MEAN_ABS)
    assert ok, f"max-abs {mx:.3e} mean-abs {mean:.3e}"
    return mx, mean


def test_config1_tinyllama_decode_with_append(fi, workloads):
    """Configuration 1: B=8, L~U[16,512], 1024 permuted pages, +1 appended token."""
    from oracle import paged_kv
    prob = workloads.make_decode_problem(workloads.TINYLLAMA, 8, 16, 512, seed=0, device="cpu",
                                         num_layers=1, pool_pages=1024)
    pool_cpu = prob.pool[0].clone()
    pool = prob.pool[0].to(DEV)
    indptr, indices, last = prob.device_tables(DEV)
    seq = torch.from_numpy(prob.lengths.astype(np.int32)).to(DEV)
    bi, pos = fi.get_batch_indices_positions(
        torch.arange(prob.batch + 1, dtype=torch.int32, device=DEV), seq, prob.batch)
    assert pos.cpu().numpy().tolist() == prob.positions.tolist()
    fi.append_paged_kv_cache(prob.k_new.to(DEV), prob.v_new.to(DEV), bi, pos, pool, indices,
                             indptr, last, kv_layout="HND")
    paged_kv.append_paged_kv_cache(prob.k_new, prob.v_new, np.arange(prob.batch),
                                   prob.positions, pool_cpu, prob.kv_indices, prob.kv_indptr)
    assert torch.equal(pool.cpu(), pool_cpu)
    got = _decode(fi, prob.q, pool, prob.kv_indptr, prob.kv_indices, prob.kv_last_page_len)
    want, _ = attention.decode(prob.q, pool_cpu.float(), prob.kv_indptr, prob.kv_indices,
                               prob.kv_last_page_len)
    _check(got, want)


@pytest.mark.parametrize("case", [c for c in load_attention_cases() if c["mode"] == "decode"],
                         ids=lambda c: c["name"])
def test_decode_matches_transformers_eager_fixture(fi, case):
    got = _decode(fi, case["q"], case["pool"], case["kv_indptr"], case["kv_indices"],
                  case["kv_last_page_len"], layout=case["layout"])
    _check(got, case["out"])


@pytest.mark.parametrize("case", [c for c in load_attention_cases() if c["mode"] == "decode"],
                         ids=lambda c: c["name"])
def test_decode_matches_flashinfer_outputs(fi, case):
    """Against FlashInfer 0.6.11's own B200 outputs on the same inputs
    (tests/golden/flashinfer_outputs.npz)."""
    import os
    from conftest import GOLDEN
    z = np.load(os.path.join(GOLDEN, "flashinfer_outputs.npz"))
    got = _decode(fi, case["q"], case["pool"], case["kv_indptr"], case["kv_indices"],
                  case["kv_last_page_len"], layout=case["layout"])
    _check(got, torch.from_numpy(z[case["name"] + "__out"]))


@pytest.mark.parametrize("geom_name,lengths", [
    ("TINYLLAMA", [1, 15, 16, 17, 31, 32, 33, 255, 256, 257]),
    ("LLAMA3_8B", [1, 16, 17, 100, 4000]),
])
def test_decode_edge_lengths(fi, workloads, geom_name, lengths):
    geom = getattr(workloads, geom_name)
    prob = workloads.make_decode_problem(geom, len(lengths), 0, 0, seed=3, num_layers=1,
                                         lengths=np.array(lengths), pool_pages=600)
    got = _decode(fi, prob.q, prob.pool[0], prob.kv_indptr, prob.kv_indices,
                  prob.kv_last_page_len)
    want, _ = attention.decode(prob.q, prob.pool[0].float(), prob.kv_indptr, prob.kv_indices,
                               prob.kv_last_page_len)
    _check(got, want)


def test_decode_long_context_split_merge_and_lse(fi, workloads):
    """Few long requests: every segment spans many warps and is LSE-merged."""
    prob = workloads.make_decode_problem(workloads.LLAMA3_8B, 3, 6000, 9000, seed=5,
                                         num_layers=1)
    got, lse = _decode(fi, prob.q, prob.pool[0], prob.kv_indptr, prob.kv_indices,
                       prob.kv_last_page_len, return_lse=True)
    want, want_lse = attention.decode(prob.q, prob.pool[0].float(), prob.kv_indptr,
                                      prob.kv_indices, prob.kv_last_page_len)
    _check(got, want)
    assert torch.allclose(lse.cpu(), want_lse, atol=1e-3, rtol=1e-4)


def test_decode_empty_request_gives_zeros(fi, workloads):
    lengths = np.array([40, 0, 17, 0])
    prob = workloads.make_decode_problem(workloads.TINYLLAMA, 4, 0, 0, seed=2, num_layers=1,
                                         lengths=lengths, pool_pages=16)
    got, lse = _decode(fi, prob.q, prob.pool[0], prob.kv_indptr, prob.kv_indices,
                       prob.kv_last_page_len, return_lse=True)
    want, _ = attention.decode(prob.q, prob.pool[0].float(), prob.kv_indptr, prob.kv_indices,
                               prob.kv_last_page_len)
    _check(got, want)
    assert torch.count_nonzero(got[1]) == 0 and torch.count_nonzero(got[3]) == 0
    assert torch.isinf(lse[1]).all() and torch.isinf(lse[3]).all()


def test_decode_honours_over_reserved_page_table(fi, workloads):
    """The reference's decode table can carry one page more than get_len needs
    (admission_controller.py:275 reserves ceil((L+1)/P)); with last_page_len = P
    the attention covers L + P keys. The kernel follows the table exactly."""
    L = 48
    prob = workloads.make_decode_problem(workloads.TINYLLAMA, 2, 0, 0, seed=9, num_layers=1,
                                         lengths=np.array([L + 16, 20]), pool_pages=12)
    # request 0: 4 pages, last_page_len 16 (the step executor's table for get_len = 48)
    assert prob.kv_indptr.tolist()[:2] == [0, 4] and prob.kv_last_page_len[0] == 16
    got = _decode(fi, prob.q, prob.pool[0], prob.kv_indptr, prob.kv_indices,
                  prob.kv_last_page_len)
    want_table, _ = attention.decode(prob.q, prob.pool[0].float(), prob.kv_indptr,
                                     prob.kv_indices, prob.kv_last_page_len)
    _check(got, want_table)
    # truncating to ceil(L/P) pages changes request 0's output
    trunc_indptr = prob.kv_indptr.copy()
    trunc_indices = np.concatenate([prob.kv_indices[:3], prob.kv_indices[4:]])
    trunc_indptr[1:] -= 1
    want_trunc, _ = attention.decode(prob.q, prob.pool[0].float(), trunc_indptr, trunc_indices,
                                     prob.kv_last_page_len)
    assert (want_trunc[0] - want_table[0]).abs().max() > 1e-3


def test_decode_fp16_and_nhd(fi, workloads):
    prob = workloads.make_decode_problem(workloads.TINYLLAMA, 6, 10, 300, seed=11, num_layers=1,
                                         dtype=torch.float16)
    got = _decode(fi, prob.q, prob.pool[0], prob.kv_indptr, prob.kv_indices,
                  prob.kv_last_page_len)
    want, _ = attention.decode(prob.q, prob.pool[0].float(), prob.kv_indptr, prob.kv_indices,
                               prob.kv_last_page_len)
    _check(got, want)
    nhd = prob.pool[0].permute(0, 1, 3, 2, 4).contiguous()  # [N, 2, P, H, D]
    got2 = _decode(fi, prob.q, nhd, prob.kv_indptr, prob.kv_indices, prob.kv_last_page_len,
                   layout="NHD")
    assert torch.equal(got.cpu(), got2.cpu())


def test_decode_strided_q_from_fused_qkv(fi, workloads):
    """q is a view of the fused QKV projection output (llama.py:163-171)."""
    prob = workloads.make_decode_problem(workloads.TINYLLAMA, 5, 30, 200, seed=4, num_layers=1)
    qkv = torch.randn(5, (32 + 8) * 64, dtype=torch.bfloat16)
    qkv[:, :32 * 64] = prob.q.reshape(5, -1)
    q_view = qkv.to(DEV).split([32 * 64, 4 * 64, 4 * 64], dim=-1)[0].view(-1, 32, 64)
    assert not q_view.is_contiguous()
    got = _decode(fi, q_view, prob.pool[0], prob.kv_indptr, prob.kv_indices,
                  prob.kv_last_page_len)
    want, _ = attention.decode(prob.q, prob.pool[0].float(), prob.kv_indptr, prob.kv_indices,
                               prob.kv_last_page_len)
    _check(got, want)


def test_decode_plan_reuse_is_deterministic(fi, workloads):
    """One plan serves every layer; split merges reset their counters per launch."""
    prob = workloads.make_decode_problem(workloads.LLAMA3_8B, 7, 500, 3000, seed=8,
                                         num_layers=2)
    t = lambda a: torch.as_tensor(a).to(DEV)  # noqa: E731
    w = fi.BatchDecodeWithPagedKVCacheWrapper(_ws(), "HND")
    w.plan(t(prob.kv_indptr), t(prob.kv_indices), t(prob.kv_last_page_len), 32, 8, 128, 16)
    q = prob.q.to(DEV)
    pool = prob.pool.to(DEV)
    outs = [w.run(q, pool[i % 2]) for i in range(4)]
    assert torch.equal(outs[0], outs[2]) and torch.equal(outs[1], outs[3])
    want, _ = attention.decode(prob.q, prob.pool[1].float(), prob.kv_indptr, prob.kv_indices,
                               prob.kv_last_page_len)
    _check(outs[1], want)


def test_mid_size_batch_capped_pieces(fi, workloads):
    """32 TinyLlama requests of 256-2048 tokens: the plan's runs would be 6
    pages (12 pieces per segment); they are raised so each segment splits
    into about 8 pieces. Two launches on one plan agree bit for bit and
    match the oracle."""
    prob = workloads.make_decode_problem(workloads.TINYLLAMA, 32, 256, 2048, seed=13,
                                         num_layers=1)
    t = lambda a: torch.as_tensor(a).to(DEV)  # noqa: E731
    w = fi.BatchDecodeWithPagedKVCacheWrapper(_ws(), "HND")
    w.plan(t(prob.kv_indptr), t(prob.kv_indices), t(prob.kv_last_page_len), 32, 4, 64, 16)
    q, pool = prob.q.to(DEV), prob.pool[0].to(DEV)
    first, second = w.run(q, pool), w.run(q, pool)
    assert torch.equal(first, second)
    want, _ = attention.decode(prob.q, prob.pool[0].float(), prob.kv_indptr, prob.kv_indices,
                               prob.kv_last_page_len)
    _check(first, want)


def test_config4_radix_shared_prefix_decode(fi, workloads):
    """Configuration 4: 64 requests share one 2048-token prefix (128 refcounted
    page ids from the radix cache) plus unique suffixes U[32, 256]; decode all,
    then evict 25 % of the unshared pages and check tables and refcounts."""
    P = 16
    rng = np.random.default_rng(4)
    alloc = bookkeeping.BlockAllocator(2048)
    cache = bookkeeping.RadixCache(P, alloc)
    prefix = rng.integers(0, 32000, 2048).tolist()
    tables_, lens = [], []
    for r in range(64):
        toks = prefix + rng.integers(0, 32000, int(rng.integers(32, 257))).tolist()
        mt, mb = bookkeeping.match_prefix_for_new_run(cache, alloc, toks)
        table = mb + alloc.allocate(math.ceil(len(toks) / P) - len(mb))
        cache.insert(toks, table)
        tables_.append(table)
        lens.append(len(toks))
    shared = tables_[0][:128]
    assert all(t[:128] == shared for t in tables_)
    assert all(alloc.ref_counts[b] == 65 for b in shared)  # 64 sequences + 1 cache
    geom = workloads.LLAMA3_8B
    indptr = np.zeros(65, dtype=np.int32)
    np.cumsum([len(t) for t in tables_], out=indptr[1:])
    indices = np.array([b for t in tables_ for b in t], dtype=np.int32)
    last = np.array([L - (math.ceil(L / P) - 1) * P for L in lens], dtype=np.int32)
    # q and a 2048-page pool; the tables come from the radix cache above
    prob = workloads.make_decode_problem(geom, 64, 0, 0, seed=12, num_layers=1,
                                         lengths=np.ones(64, dtype=np.int64), pool_pages=2048)
    got = _decode(fi, prob.q, prob.pool[0], indptr, indices, last)
    want, _ = attention.decode(prob.q, prob.pool[0].float(), indptr, indices, last)
    _check(got, want)
    # sequences finish; evict 25 % of the pages only the cache holds (unshared)
    for t in tables_:
        alloc.decref(t)
    unshared = [b for b, c in enumerate(alloc.ref_counts) if c == 1 and b not in shared]
    evicted = cache.evict_lru(len(unshared) // 4)
    assert len(evicted) == len(unshared) // 4
    assert not set(evicted) & set(shared)
    assert all(alloc.ref_counts[b] == 0 for b in evicted)
    assert all(alloc.ref_counts[b] == 1 for b in shared)
    # a new request still matches the whole shared prefix afterwards
    mt, mb = cache.match_prefix(prefix + [1])
    assert mb == shared


def test_full_size_config2_layer_sampled(fi, workloads):
    """Configuration 2 size, one layer: B=256, L~U[1024,4096]; oracle on a sample."""
    prob = workloads.make_decode_problem(workloads.TINYLLAMA, 256, 1024, 4096, seed=0,
                                         device=DEV, num_layers=1)
    got = _decode(fi, prob.q, prob.pool[0], prob.kv_indptr, prob.kv_indices,
                  prob.kv_last_page_len)
    assert torch.isfinite(got).all()
    sample = [0, 1, 77, 128, 200, 255]
    want, _ = attention.decode(prob.q.cpu(), prob.pool[0], prob.kv_indptr, prob.kv_indices,
                               prob.kv_last_page_len, requests=sample)
    _check(got.cpu()[sample], want[sample])


def test_device_check_flags_bad_page_id(fi, lir, workloads):
    prob = workloads.make_decode_problem(workloads.TINYLLAMA, 3, 20, 60, seed=1, num_layers=1,
                                         pool_pages=20)
    indices = prob.kv_indices.copy()
    indices[1] = 10_000  # beyond the pool
    torch.cuda.synchronize()
    lir._lib.device_status()  # clear
    t = lambda a: torch.as_tensor(a).to(DEV)  # noqa: E731
    w = fi.BatchDecodeWithPagedKVCacheWrapper(_ws(), "HND")
    import importlib
    fa = importlib.import_module("llm-inference-runtime_b200.flashinfer_api")
    saved = fa._CHECK
    fa._CHECK = False
    try:
        w.plan(t(prob.kv_indptr), t(indices), t(prob.kv_last_page_len), 32, 4, 64, 16)
        w.run(prob.q.to(DEV), prob.pool[0].to(DEV))
        assert lir._lib.device_status() == lir._lib.PA_ERR_DEVICE_CHECK
        bad_last = prob.kv_last_page_len.copy()
        bad_last[0] = 17  # > page size
        w.plan(t(prob.kv_indptr), t(prob.kv_indices), t(bad_last), 32, 4, 64, 16)
        assert lir._lib.device_status() == lir._lib.PA_ERR_DEVICE_CHECK
        bad_indptr = prob.kv_indptr.copy()
        bad_indptr[1], bad_indptr[2] = bad_indptr[2], bad_indptr[1]  # not monotone
        w.plan(t(bad_indptr), t(prob.kv_indices), t(prob.kv_last_page_len), 32, 4, 64, 16)
        assert lir._lib.device_status() == lir._lib.PA_ERR_DEVICE_CHECK
    finally:
        fa._CHECK = saved
    # with checking on, the same error surfaces as RuntimeError
    with pytest.raises(RuntimeError, match="device"):
        w.plan(t(prob.kv_indptr), t(prob.kv_indices), t(bad_last), 32, 4, 64, 16)


def test_run_without_plan_raises(fi):
    w = fi.BatchDecodeWithPagedKVCacheWrapper(_ws(), "HND")
    with pytest.raises(RuntimeError, match="plan"):
        w.run(torch.zeros(1, 32, 64, dtype=torch.bfloat16, device=DEV),
              torch.zeros(4, 2, 4, 16, 64, dtype=torch.bfloat16, device=DEV))


def test_unsupported_options_raise(fi):
    w = fi.BatchDecodeWithPagedKVCacheWrapper(_ws(), "HND")
    t = torch.zeros(2, dtype=torch.int32, device=DEV)
    with pytest.raises(NotImplementedError):
        w.plan(t, t[:1], t[:1], 32, 4, 64, 16, logits_soft_cap=30.0)
    with pytest.raises(NotImplementedError):
        w.plan(t, t[:1], t[:1], 32, 4, 64, 16, window_left=128)


def test_bounded_wait_times_out_and_context_stays_usable(fi, lir, workloads):
    """The bounded-wait path without a fault: a kernel waits on a barrier
    nothing completes, gives up after ~1 ms of SM clocks, reports
    PA_ERR_TIMEOUT; the next decode on the same context is correct."""
    torch.cuda.synchronize()
    lir._lib.device_status()
    lib = lir._lib.load()
    assert lib.pa_selftest_wait_timeout(2_000_000, torch.cuda.current_stream().cuda_stream) == 0
    assert lir._lib.device_status() == lir._lib.PA_ERR_TIMEOUT
    assert lir._lib.device_status() == 0  # read and cleared
    geom = workloads.TINYLLAMA
    prob = workloads.make_decode_problem(geom, 4, 50, 300, seed=21, device=DEV, num_layers=1,
                                         append=False)
    got = _decode(fi, prob.q, prob.pool[0], prob.kv_indptr, prob.kv_indices,
                  prob.kv_last_page_len)
    want, _ = attention.decode(prob.q, prob.pool[0].float(), prob.kv_indptr, prob.kv_indices,
                               prob.kv_last_page_len)
    _check(got, want)


@pytest.mark.parametrize("hq,hkv,d", [(8, 8, 128), (16, 8, 64), (32, 2, 128), (64, 4, 64),
                                      (16, 16, 64), (32, 16, 128)])
def test_decode_every_gqa_group_and_head_block(fi, workloads, hq, hkv, d):
    """Group sizes 1..16 and kv-head counts above 8 (two head blocks per
    page): the head-block split of the stream and the GQA rows of the MMA."""
    geom = workloads.Geometry(num_qo_heads=hq, num_kv_heads=hkv, head_dim=d)
    prob = workloads.make_decode_problem(geom, 9, 1, 1500, seed=hq * 7 + hkv, num_layers=1)
    got, lse = _decode(fi, prob.q, prob.pool[0], prob.kv_indptr, prob.kv_indices,
                       prob.kv_last_page_len, return_lse=True)
    want, want_lse = attention.decode(prob.q, prob.pool[0].float(), prob.kv_indptr,
                                      prob.kv_indices, prob.kv_last_page_len)
    _check(got, want)
    assert torch.allclose(lse.cpu(), want_lse, atol=2e-3, rtol=1e-4)
