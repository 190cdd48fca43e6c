"""Pins the CPU oracle to fixtures produced by the reference's own code.

CPU only. Every fixture comes from tests/golden/make_golden.py, which ran the
reference (BlockAllocator, RadixCache, match_prefix_for_new_run,
StepExecutor) and transformers' eager attention.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import load_attention_cases, load_json
from oracle import attention, bookkeeping, paged_kv, tables


# ------------------------------------------------------------ bookkeeping
def _replay_config4(sc):
    P = 16
    a = bookkeeping.BlockAllocator(4096)
    cache = bookkeeping.RadixCache(P, a, clock=bookkeeping.counter_clock())
    prefix = sc["prefix"]
    ops = iter(sc["ops"])
    import random
    rng = random.Random(sc["seed"])
    assert [rng.randrange(32000) for _ in range(2048)] == prefix
    tables_ = []
    for r in range(64):
        rec = next(ops)
        assert rec["op"] == "admit"
        suffix_len = rng.randint(32, 256)
        assert suffix_len == rec["suffix_len"]
        toks = prefix + [rng.randrange(32000) for _ in range(suffix_len)]
        mt, mb = bookkeeping.match_prefix_for_new_run(cache, a, toks)
        assert len(mt) == rec["matched_tokens"] and mb == rec["matched_blocks"]
        new = a.allocate(math.ceil(len(toks) / P) - len(mb))
        assert new == rec["allocated"]
        table = mb + new
        tables_.append(table)
        rec = next(ops)
        assert cache.insert(toks, table) == rec["new"]
    assert tables_ == sc["tables"]
    assert a.free_blocks == sc["state_before_finish"]["free_blocks"]
    assert a.ref_counts == sc["state_before_finish"]["ref_counts"]
    for t in tables_:
        a.decref(t)
    rec = next(ops)
    assert cache.evict_lru(rec["num_blocks"]) == rec["evicted"]
    assert a.free_blocks == sc["final"]["free_blocks"]
    assert a.ref_counts == sc["final"]["ref_counts"]
    return tables_


def _replay_fuzz(sc):
    import random
    P = 16
    rng = random.Random(sc["seed"])
    a = bookkeeping.BlockAllocator(96)
    cache = bookkeeping.RadixCache(P, a, clock=bookkeeping.counter_clock())
    corpus = [[rng.randrange(50) for _ in range(rng.randint(1, 70))] for _ in range(6)]
    assert corpus == sc["corpus"]
    live = []
    ops = iter(sc["ops"])
    for _ in range(160):
        kind = rng.choice(["admit", "admit", "finish", "evict", "decode_grow"])
        if kind == "admit":
            base = rng.choice(corpus)
            toks = base[:rng.randint(1, len(base))] + [rng.randrange(50)
                                                       for _ in range(rng.randint(0, 20))]
            rec = next(ops)
            assert rec["op"] == "admit" and toks == rec["tokens"]
            mt, mb = bookkeeping.match_prefix_for_new_run(cache, a, toks)
            assert (len(mt), mb) == (rec["matched_tokens"], rec["matched_blocks"])
            need = math.ceil(len(toks) / P) - len(mb)
            ok = a.try_allocate(need, cache)
            assert ok == rec["ok"]
            if ok:
                new = a.allocate(need)
                assert new == rec["allocated"]
                table = mb + new
                assert cache.insert(toks, table) == rec["inserted"]
                live.append((toks, table))
            else:
                a.decref(mb)
        elif kind == "finish" and live:
            i = rng.randrange(len(live))
            rec = next(ops)
            assert rec["op"] == "finish" and rec["index"] == i
            toks, table = live.pop(i)
            assert cache.insert(toks, table) == rec["inserted"]
            a.decref(table)
        elif kind == "evict":
            n = rng.randint(1, 8)
            rec = next(ops)
            assert rec["op"] == "evict_lru" and cache.evict_lru(n) == rec["evicted"]
        elif kind == "decode_grow" and live:
            i = rng.randrange(len(live))
            toks, table = live[i]
            toks = toks + [rng.randrange(50)]
            rec = next(ops)
            assert rec["op"] == "decode_grow" and rec["token"] == toks[-1]
            need = math.ceil((len(toks) + 1) / P) - len(table)
            got = []
            if need > 0 and a.try_allocate(need, cache):
                got = a.allocate(need)
            assert got == rec["allocated"]
            live[i] = (toks, table + got)
        else:
            continue
        assert a.free_blocks == rec["free_blocks"]
        assert a.ref_counts == rec["ref_counts"]


def test_bookkeeping_config4_matches_reference():
    trace = load_json("bookkeeping_trace.json")
    sc = next(s for s in trace["scenarios"] if s["name"] == "config4_shared_prefix")
    tables_ = _replay_config4(sc)
    # all 64 requests share the 128 prefix pages by id
    assert all(t[:128] == tables_[0][:128] for t in tables_)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_bookkeeping_fuzz_matches_reference(seed):
    trace = load_json("bookkeeping_trace.json")
    _replay_fuzz(next(s for s in trace["scenarios"] if s["name"] == f"fuzz_{seed}"))


def test_allocator_double_free_raises():
    a = bookkeeping.BlockAllocator(4)
    blocks = a.allocate(2)
    a.decref(blocks)
    with pytest.raises(bookkeeping.AllocationError):
        a.decref(blocks[:1])


# ----------------------------------------------------------------- tables
def test_prefill_tables_match_step_executor():
    st = load_json("step_tables.json")
    for case in st["prefill"]:
        got = tables.prefill_tables([tuple(s) for s in case["seqs"]], case["chunk_lens"], 16)
        cap = case["captured"]
        pp = cap["plan_prefill"]
        assert got["qo_indptr"] == pp["qo_indptr"]
        assert got["kv_indptr"] == pp["kv_indptr"]
        assert got["kv_indices"] == pp["kv_indices"]
        assert got["kv_last_page_len"] == pp["kv_last_page_len"]
        assert got["seq_lens"] == cap["bip"]["seq_lens"]
        assert got["qo_indptr"] == cap["bip"]["append_indptr"]
        assert got["positions"] == cap["position_ids"][0]
        bi, pos = paged_kv.batch_indices_positions(got["qo_indptr"], got["seq_lens"])
        assert pos.tolist() == cap["position_ids"][0]


def test_decode_tables_match_step_executor_including_reservation_quirk():
    st = load_json("step_tables.json")
    quirk_seen = False
    for case in st["decode"]:
        seqs = [tuple(s) for s in case["seqs"]]
        got = tables.decode_tables(seqs, 16)
        pd = case["captured"]["plan_decode"]
        assert got["kv_indptr"] == pd["kv_indptr"]
        assert got["kv_indices"] == pd["kv_indices"]
        assert got["kv_last_page_len"] == pd["kv_last_page_len"]
        assert got["batch_indices"] == case["captured"]["batch_indices"]
        assert got["positions"] == case["captured"]["positions"]
        for (L, table) in seqs:
            if L % 16 == 0:
                # the scheduler reserved ceil((L + 1) / 16) pages: one more than L needs
                assert len(table) == L // 16 + 1
                quirk_seen = True
    assert quirk_seen


# ------------------------------------------------------------- paged_kv
def test_batch_indices_positions_known_answers():
    ka = load_json("known_answers.json")["get_batch_indices_positions"]
    for ex in ka:
        bi, pos = paged_kv.batch_indices_positions(ex["append_indptr"], ex["seq_lens"], ex["nnz"])
        assert bi.tolist() == ex["batch_indices"]
        assert pos.tolist() == ex["positions"]
    ex = ka[1]
    assert paged_kv.seq_lens(ex["kv_page_indptr"], ex["kv_last_page_len"], 16).tolist() == \
        ex["seq_lens"]


def test_batch_indices_positions_tail_padding():
    bi, pos = paged_kv.batch_indices_positions([0, 2, 3], [5, 9], nnz=5)
    assert bi.tolist() == [0, 0, 1, -1, -1]
    assert pos.tolist() == [3, 4, 8, 0, 0]


def test_append_oracle_roundtrip():
    rng = np.random.default_rng(0)
    pool = np.zeros((8, 2, 2, 16, 8), dtype=np.float32)
    indptr = np.array([0, 2, 3])
    indices = np.array([5, 1, 6])
    k = rng.standard_normal((3, 2, 8)).astype(np.float32)
    v = rng.standard_normal((3, 2, 8)).astype(np.float32)
    paged_kv.append_paged_kv_cache(k, v, [0, 0, 1], [15, 16, 0], pool, indices, indptr)
    assert np.array_equal(pool[5, 0, :, 15], k[0])
    assert np.array_equal(pool[1, 1, :, 0], v[1])
    assert np.array_equal(pool[6, 0, :, 0], k[2])


# -------------------------------------------------------------- attention
@pytest.mark.parametrize("case", load_attention_cases(), ids=lambda c: c["name"])
def test_attention_oracle_matches_transformers_eager(case):
    pool = case["pool"].to(torch.float32)
    if case["mode"] == "decode":
        got, _ = attention.decode(case["q"], pool, case["kv_indptr"], case["kv_indices"],
                                  case["kv_last_page_len"], layout=case["layout"])
    else:
        got, _ = attention.prefill(case["q"], case["qo_indptr"], pool, case["kv_indptr"],
                                   case["kv_indices"], case["kv_last_page_len"], causal=True,
                                   layout=case["layout"])
    assert torch.allclose(got, case["out"], atol=1e-5, rtol=1e-5)


def test_lse_merge_identity():
    """Splitting keys into two halves and merging by LSE reproduces the whole."""
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 4, 16, generator=g)
    k = torch.randn(2, 40, 16, generator=g)
    v = torch.randn(2, 40, 16, generator=g)
    o, l2 = attention.attend(q, k, v, 0.25)
    oa, la = attention.attend(q, k[:, :13], v[:, :13], 0.25)
    ob, lb = attention.attend(q, k[:, 13:], v[:, 13:], 0.25)
    vm, sm = paged_kv.merge_states(torch.stack([oa, ob], 1).numpy(),
                                   torch.stack([la, lb], 1).numpy())
    assert np.allclose(vm, o.numpy(), atol=1e-5)
    assert np.allclose(sm, l2.numpy(), atol=1e-5)


def _flashinfer_outputs():
    import os
    from conftest import GOLDEN
    path = os.path.join(GOLDEN, "flashinfer_outputs.npz")
    return np.load(path) if os.path.exists(path) else None


@pytest.mark.parametrize("case", load_attention_cases(), ids=lambda c: c["name"])
def test_attention_oracle_matches_flashinfer_on_b200(case):
    """The oracle against FlashInfer 0.6.11 itself (the reference's GPU path),
    run on a B200 by tests/golden/make_flashinfer_golden.py. FlashInfer's
    outputs are bf16, so the north-star bf16 tolerance applies."""
    z = _flashinfer_outputs()
    assert z is not None, "tests/golden/flashinfer_outputs.npz missing"
    assert bytes(z["flashinfer_version"]).decode().startswith("0.6.11")
    want = torch.from_numpy(z[case["name"] + "__out"])
    pool = case["pool"].to(torch.float32)
    if case["mode"] == "decode":
        got, _ = attention.decode(case["q"], pool, case["kv_indptr"], case["kv_indices"],
                                  case["kv_last_page_len"], layout=case["layout"])
    else:
        got, _ = attention.prefill(case["q"], case["qo_indptr"], pool, case["kv_indptr"],
                                   case["kv_indices"], case["kv_last_page_len"], causal=True,
                                   layout=case["layout"])
    mx, mean, ok = attention.compare(want, got)
    assert ok, f"max-abs {mx:.3e} mean-abs {mean:.3e}"


def test_two_level_merge_equals_concatenated_tables():
    """The expected value the GPU cascade tests build — decode over the
    shared prefix pages and over each request's own pages separately, merged
    by base-2 log-sum-exp with a level of LSE -inf contributing nothing —
    equals the oracle decode over the concatenated tables (full shared pages;
    requests with no pages of their own included)."""
    g = torch.Generator().manual_seed(3)
    B, H, HKV, D, N = 5, 8, 2, 16, 40
    pool = torch.randn(N, 2, HKV, 16, D, generator=g)
    q = torch.randn(B, H, D, generator=g)
    perm = torch.randperm(N, generator=g).numpy().astype(np.int32)
    shared = perm[:3]
    counts = np.array([2, 0, 1, 3, 0])
    up = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    ui = perm[3:3 + up[-1]]
    ul = np.array([5, 16, 16, 1, 16], dtype=np.int32)
    o0, l0 = attention.decode(q, pool, np.arange(B + 1) * 3, np.tile(shared, B), np.full(B, 16))
    o1, l1 = attention.decode(q, pool, up, ui, ul)
    m = torch.maximum(l0, l1)
    m = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    w0, w1 = torch.exp2(l0 - m), torch.exp2(l1 - m)
    merged = (o0 * w0[..., None] + o1 * w1[..., None]) / (w0 + w1)[..., None]
    full_ptr = np.concatenate([[0], np.cumsum(3 + counts)]).astype(np.int32)
    full_idx = np.concatenate([np.concatenate([shared, ui[up[b]:up[b + 1]]]) for b in range(B)])
    full_last = np.where(counts > 0, ul, 16).astype(np.int32)
    want, want_lse = attention.decode(q, pool, full_ptr, full_idx, full_last)
    assert torch.allclose(merged, want, atol=1e-5)
    lse = m + torch.log2(w0 + w1)
    assert torch.allclose(lse, want_lse, atol=1e-5)
