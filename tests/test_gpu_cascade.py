"""Two-level (cascade) decode for radix-shared prefixes on the GPU.

The reference decodes a batch whose requests share prefix pages (identical
refcounted page ids at the head of every block table, from its RadixCache)
request by request (src/models/llama.py:230-245). The cascade wrapper attends
the shared pages once for all requests and merges with each request's own
pages. Checked against the plain decode over the full tables and against
the fp32 oracle: max-abs 2e-2, mean-abs 2e-3 (bf16 in, fp32 accumulate;
the level states are rounded to bf16 before the merge).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3
DEV = "cuda"


def _t(a):
    return torch.as_tensor(np.asarray(a, dtype=np.int32)).to(DEV)


def _split_tables(prob, shared_pages):
    """Level-0 (shared prefix) and level-1 (unique pages) tables of a problem
    whose tables all start with the same `shared_pages` page ids."""
    indptr, indices = prob.kv_indptr, prob.kv_indices
    B = len(indptr) - 1
    shared = indices[:shared_pages]
    uniq, uptr = [], [0]
    for b in range(B):
        pages = indices[indptr[b]:indptr[b + 1]]
        assert np.array_equal(pages[:shared_pages], shared)
        uniq.append(pages[shared_pages:])
        uptr.append(uptr[-1] + len(pages) - shared_pages)
    uindices = np.concatenate(uniq) if uniq else np.zeros(0, np.int32)
    return (np.array([0, shared_pages]), shared, np.array([16]),
            np.array(uptr), uindices, prob.kv_last_page_len)


def _cascade(fi, q, pool, levels, hq, hkv, d, return_lse=False):
    sp, si, sl, up, ui, ul = levels
    B = q.shape[0]
    nbytes = fi.cascade_workspace_bytes(B, hq, hkv, d)
    ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=DEV)
    w = fi.MultiLevelCascadeAttentionWrapper(2, ws, "HND")
    w.plan([torch.tensor([0, B], dtype=torch.int32), torch.arange(B + 1, dtype=torch.int32)],
           [_t(sp), _t(up)], [_t(si), _t(ui)], [_t(sl), _t(ul)], hq, hkv, d, 16)
    return w.run(q.to(DEV), pool.to(DEV), return_lse=return_lse)


def _plain(fi, prob, hq, hkv, d):
    w = fi.BatchDecodeWithPagedKVCacheWrapper(torch.empty(128 << 20, dtype=torch.uint8,
                                                          device=DEV), "HND")
    w.plan(_t(prob.kv_indptr), _t(prob.kv_indices), _t(prob.kv_last_page_len), hq, hkv, d, 16,
           q_data_type=prob.q.dtype)
    return w.run(prob.q.to(DEV), prob.pool[0].to(DEV))


def _check(got, want):
    mx, mean, ok = attention.compare(got, want, MAX_ABS, MEAN_ABS)
    assert ok, f"max-abs {mx:.3e} mean-abs {mean:.3e}"


@pytest.mark.parametrize("geom_name,batch,prefix", [
    ("LLAMA3_8B", 64, 2048),   # configuration 4
    ("TINYLLAMA", 37, 512),
    ("LLAMA3_8B", 3, 4096),
    ("TINYLLAMA", 300, 256),
    # 4 kv heads x one query span per chunk: the plan allows 37 chunks on 148
    # SMs and 296 prefix pages cut into 37 chunks of 8, so chunk states
    # 32-36 travel in the merge's second LSE slot
    ("TINYLLAMA", 6, 4736),
])
def test_cascade_matches_plain_decode_and_oracle(fi, workloads, geom_name, batch, prefix):
    geom = getattr(workloads, geom_name)
    prob = workloads.make_shared_prefix_problem(geom, batch, prefix, 32, 256, seed=batch)
    hq, hkv, d = geom.num_qo_heads, geom.num_kv_heads, geom.head_dim
    levels = _split_tables(prob, prefix // 16)
    got, lse = _cascade(fi, prob.q, prob.pool[0], levels, hq, hkv, d, return_lse=True)
    plain = _plain(fi, prob, hq, hkv, d)
    _check(got.cpu(), plain.cpu().float())
    sample = list(range(0, batch, max(1, batch // 6)))
    want, want_lse = attention.decode(prob.q, prob.pool[0].float(), prob.kv_indptr,
                                      prob.kv_indices, prob.kv_last_page_len, requests=sample)
    _check(got.cpu()[sample], want[sample])
    assert torch.allclose(lse.cpu()[sample], want_lse[sample], atol=2e-2)


def test_cascade_partial_prefix_page_and_empty_levels(fi, workloads):
    """A shared last page that is only partly filled, requests with no pages
    of their own, and a batch with no shared prefix at all: the result is the
    log-sum-exp merge of the two levels' oracle states."""
    geom = workloads.TINYLLAMA
    hq, hkv, d = geom.num_qo_heads, geom.num_kv_heads, geom.head_dim
    rng = np.random.default_rng(7)
    B, N = 9, 64
    pool = torch.randn((N, 2, hkv, 16, d)).to(torch.bfloat16)
    q = torch.randn((B, hq, d)).to(torch.bfloat16)
    perm = rng.permutation(N).astype(np.int32)
    for shared_pages, shared_last in ((5, 7), (0, 16)):
        shared = perm[:shared_pages]
        counts = np.array([0, 1, 3, 0, 2, 4, 1, 0, 5])[:B]
        up = np.concatenate([[0], np.cumsum(counts)])
        ui = perm[shared_pages:shared_pages + up[-1]]
        ul = rng.integers(1, 17, B).astype(np.int32)
        levels = (np.array([0, shared_pages]), shared, np.array([shared_last]), up, ui, ul)
        got = _cascade(fi, q, pool, levels, hq, hkv, d)
        o0, l0 = attention.decode(q, pool.float(), np.arange(B + 1) * shared_pages,
                                  np.tile(shared, B), np.full(B, shared_last))
        o1, l1 = attention.decode(q, pool.float(), up, ui, ul)
        m = torch.maximum(l0, l1)
        m = torch.where(torch.isinf(m), torch.zeros_like(m), m)
        w0, w1 = torch.exp2(l0 - m), torch.exp2(l1 - m)
        den = (w0 + w1).clamp_min(1e-30)
        want = (o0 * w0[..., None] + o1 * w1[..., None]) / den[..., None]
        _check(got.cpu(), want)


def test_cascade_rejects_unsupported_levels(fi):
    ws = torch.empty(1 << 20, dtype=torch.uint8, device=DEV)
    with pytest.raises(NotImplementedError):
        fi.MultiLevelCascadeAttentionWrapper(3, ws, "HND")
    w = fi.MultiLevelCascadeAttentionWrapper(2, ws, "HND")
    two_groups = torch.tensor([0, 2, 4], dtype=torch.int32)
    with pytest.raises(NotImplementedError):
        w.plan([two_groups, torch.arange(5, dtype=torch.int32)],
               [_t([0, 1, 2]), _t([0, 1, 2, 3, 4])], [_t([0, 1]), _t([2, 3, 4, 5])],
               [_t([16, 16]), _t([16] * 4)], 32, 4, 64, 16)


def test_cascade_fused_append_matches_append_then_run(fi, workloads):
    """run_with_append: the step's new K / V row lands in the request's own
    pages (global position minus the prefix keys) before level 1 reads it.
    The pool afterwards is bit-identical to append_paged_kv_cache + run, the
    shared prefix pages are untouched, and the outputs agree."""
    geom = workloads.LLAMA3_8B
    hq, hkv, d = geom.num_qo_heads, geom.num_kv_heads, geom.head_dim
    B, prefix = 24, 2048
    prob = workloads.make_shared_prefix_problem(geom, B, prefix, 32, 256, seed=11)
    sp = prefix // 16
    levels = _split_tables(prob, sp)
    pool_a = prob.pool[0].to(DEV)
    pool_b = pool_a.clone()
    seq = _t(prob.lengths)
    k_new, v_new = prob.k_new.to(DEV), prob.v_new.to(DEV)
    q = prob.q.to(DEV)
    bi, pos = fi.get_batch_indices_positions(torch.arange(B + 1, dtype=torch.int32, device=DEV),
                                             seq, B)
    # reference order: append over the full tables, then the cascade
    fi.append_paged_kv_cache(k_new, v_new, bi, pos, pool_a, _t(prob.kv_indices),
                             _t(prob.kv_indptr), _t(prob.kv_last_page_len), kv_layout="HND")
    want = _cascade(fi, q, pool_a, levels, hq, hkv, d)
    sp_, si, sl, up, ui, ul = levels
    ws = torch.empty(max(fi.cascade_workspace_bytes(B, hq, hkv, d), 1 << 20), dtype=torch.uint8,
                     device=DEV)
    w = fi.MultiLevelCascadeAttentionWrapper(2, ws, "HND")
    w.plan([torch.tensor([0, B], dtype=torch.int32), torch.arange(B + 1, dtype=torch.int32)],
           [_t(sp_), _t(up)], [_t(si), _t(ui)], [_t(sl), _t(ul)], hq, hkv, d, 16)
    got = w.run_with_append(q, pool_b, k_new, v_new, pos)
    torch.cuda.synchronize()
    assert torch.equal(pool_a, pool_b)
    assert torch.equal(pool_b[torch.as_tensor(si, dtype=torch.long, device=DEV)],
                       prob.pool[0].to(DEV)[torch.as_tensor(si, dtype=torch.long, device=DEV)])
    _check(got.cpu(), want.cpu().float())


def test_cascade_fused_append_into_shared_page_is_reported(fi, lir, workloads):
    """A position inside the shared prefix is a device-check error (the
    prefix pages belong to every request), and nothing is written."""
    import importlib
    fa = importlib.import_module("llm-inference-runtime_b200.flashinfer_api")
    geom = workloads.TINYLLAMA
    hq, hkv, d = geom.num_qo_heads, geom.num_kv_heads, geom.head_dim
    B = 4
    prob = workloads.make_shared_prefix_problem(geom, B, 256, 32, 64, seed=3)
    sp_, si, sl, up, ui, ul = _split_tables(prob, 16)
    pool = prob.pool[0].to(DEV)
    before = pool.clone()
    ws = torch.empty(max(fi.cascade_workspace_bytes(B, hq, hkv, d), 1 << 20), dtype=torch.uint8,
                     device=DEV)
    w = fi.MultiLevelCascadeAttentionWrapper(2, ws, "HND")
    w.plan([torch.tensor([0, B], dtype=torch.int32), torch.arange(B + 1, dtype=torch.int32)],
           [_t(sp_), _t(up)], [_t(si), _t(ui)], [_t(sl), _t(ul)], hq, hkv, d, 16)
    torch.cuda.synchronize()
    lir._lib.device_status()
    saved = fa._CHECK
    fa._CHECK = False
    try:
        w.run_with_append(prob.q.to(DEV), pool, prob.k_new.to(DEV), prob.v_new.to(DEV),
                          _t([100, 5, 255, 17]))  # all inside the 256-token prefix
        assert lir._lib.device_status() == lir._lib.PA_ERR_DEVICE_CHECK
    finally:
        fa._CHECK = saved
    assert torch.equal(pool, before)


@pytest.mark.parametrize("geom_name,dtype", [("TINYLLAMA", torch.float16), ("LLAMA3_8B", torch.float16),
                                             ("LLAMA3_8B", torch.bfloat16)])
def test_cascade_nhd_layout_strided_q_fp16(fi, workloads, geom_name, dtype):
    """The NHD pool layout ([N, 2, P, H, D]), fp16, and q as a strided view
    of a fused QKV row (as the patched attention passes it), against the
    plain decode over the full tables on the same pool."""
    geom = getattr(workloads, geom_name)
    hq, hkv, d = geom.num_qo_heads, geom.num_kv_heads, geom.head_dim
    B, prefix = 19, 768
    prob = workloads.make_shared_prefix_problem(geom, B, prefix, 1, 90, seed=23, dtype=dtype)
    sp_, si, sl, up, ui, ul = _split_tables(prob, prefix // 16)
    nhd = prob.pool[0].permute(0, 1, 3, 2, 4).contiguous().to(DEV)  # [N, 2, P, H, D]
    qkv = torch.randn(B, (hq + 2 * hkv) * d, dtype=dtype, device=DEV)
    q = qkv[:, :hq * d].view(B, hq, d)
    q.copy_(prob.q.to(DEV))
    assert not q.is_contiguous()
    ws = torch.empty(max(fi.cascade_workspace_bytes(B, hq, hkv, d), 1 << 20), dtype=torch.uint8,
                     device=DEV)
    w = fi.MultiLevelCascadeAttentionWrapper(2, ws, "NHD")
    w.plan([torch.tensor([0, B], dtype=torch.int32), torch.arange(B + 1, dtype=torch.int32)],
           [_t(sp_), _t(up)], [_t(si), _t(ui)], [_t(sl), _t(ul)], hq, hkv, d, 16)
    got = w.run(q, nhd)
    pw = fi.BatchDecodeWithPagedKVCacheWrapper(torch.empty(128 << 20, dtype=torch.uint8,
                                                           device=DEV), "NHD")
    pw.plan(_t(prob.kv_indptr), _t(prob.kv_indices), _t(prob.kv_last_page_len), hq, hkv, d, 16,
            q_data_type=dtype)
    plain = pw.run(q, nhd)
    _check(got.float().cpu(), plain.float().cpu())
    want, _ = attention.decode(prob.q.float(), prob.pool[0].float(), prob.kv_indptr,
                               prob.kv_indices, prob.kv_last_page_len, requests=[0, 7, 18])
    _check(got.float().cpu()[[0, 7, 18]], want[[0, 7, 18]])


@pytest.mark.parametrize("hq,hkv,d", [(8, 8, 128), (16, 8, 64), (32, 2, 128), (64, 4, 64)])
def test_cascade_gqa_groups(fi, workloads, hq, hkv, d):
    """GQA groups 1, 2 and 16 at both head sizes: the level-0 tiles pack
    128 / g queries x g heads per kv head, level 1 puts the g heads in one
    decode tile; both against the plain decode and the oracle."""
    geom = workloads.Geometry(num_qo_heads=hq, num_kv_heads=hkv, head_dim=d)
    B, prefix = 11, 1024
    prob = workloads.make_shared_prefix_problem(geom, B, prefix, 1, 200, seed=hq * 10 + hkv)
    levels = _split_tables(prob, prefix // 16)
    got = _cascade(fi, prob.q, prob.pool[0], levels, hq, hkv, d)
    plain = _plain(fi, prob, hq, hkv, d)
    _check(got.cpu(), plain.cpu().float())
    sample = [0, 5, 10]
    want, _ = attention.decode(prob.q, prob.pool[0].float(), prob.kv_indptr, prob.kv_indices,
                               prob.kv_last_page_len, requests=sample)
    _check(got.cpu()[sample], want[sample])


def test_cascade_prefix_table_past_its_page_ids_is_reported(fi, lir, workloads):
    """A level-0 table that names more pages than the shared index array
    holds is a device-check error from the plan; no kernel reads past the
    array (the level-0 work list is left empty)."""
    import importlib
    fa = importlib.import_module("llm-inference-runtime_b200.flashinfer_api")
    geom = workloads.TINYLLAMA
    hq, hkv, d = geom.num_qo_heads, geom.num_kv_heads, geom.head_dim
    B = 4
    prob = workloads.make_shared_prefix_problem(geom, B, 256, 32, 64, seed=5)
    sp_, si, sl, up, ui, ul = _split_tables(prob, 16)
    ws = torch.empty(max(fi.cascade_workspace_bytes(B, hq, hkv, d), 1 << 20), dtype=torch.uint8,
                     device=DEV)
    w = fi.MultiLevelCascadeAttentionWrapper(2, ws, "HND")
    torch.cuda.synchronize()
    lir._lib.device_status()
    saved = fa._CHECK
    fa._CHECK = False
    try:
        # 16 pages named, 5 page ids given
        w.plan([torch.tensor([0, B], dtype=torch.int32), torch.arange(B + 1, dtype=torch.int32)],
               [_t([0, 16]), _t(up)], [_t(si[:5]), _t(ui)], [_t(sl), _t(ul)], hq, hkv, d, 16)
        w.run(prob.q.to(DEV), prob.pool[0].to(DEV))
        assert lir._lib.device_status() == lir._lib.PA_ERR_DEVICE_CHECK
    finally:
        fa._CHECK = saved
