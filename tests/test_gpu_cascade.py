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
