"""Decode with the step's KV append in the same launch (pa_decode_append_run).

The reference's decode step runs, per layer, append_paged_kv_cache(k, v,
arange(B), positions) and then the decode forward (src/models/llama.py:188-210,
230-245). The fused call must leave the pool bit-identical to that sequence
and return bit-identical attention outputs; both are also checked against the
CPU oracle (append bit-exact, attention within max-abs 2e-2 / mean-abs 2e-3).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention, paged_kv

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3
DEV = "cuda"


def _t(a):
    return torch.as_tensor(np.asarray(a, dtype=np.int32)).to(DEV)


def _both_paths(fi, prob, pool_layer, layout, k_new, v_new, positions):
    """Returns (pool, out) of append + run and of run_with_append."""
    hq, d = prob.q.shape[1], prob.q.shape[2]
    hkv = k_new.shape[1]
    B = prob.batch
    indptr, indices, last = _t(prob.kv_indptr), _t(prob.kv_indices), _t(prob.kv_last_page_len)
    pos = _t(positions)
    q = prob.q.to(DEV)
    w = fi.BatchDecodeWithPagedKVCacheWrapper(torch.empty(128 << 20, dtype=torch.uint8,
                                                          device=DEV), layout)
    w.plan(indptr, indices, last, hq, hkv, d, 16, q_data_type=q.dtype)
    pool_a = pool_layer.to(DEV).clone()
    fi.append_paged_kv_cache(k_new, v_new, _t(np.arange(B)), pos, pool_a, indices, indptr, last,
                             kv_layout=layout)
    out_a = w.run(q, pool_a)
    pool_b = pool_layer.to(DEV).clone()
    out_b = w.run_with_append(q, pool_b, k_new, v_new, pos)
    torch.cuda.synchronize()
    return pool_a.cpu(), out_a.cpu(), pool_b.cpu(), out_b.cpu()


@pytest.mark.parametrize("geom_name,batch,lo,hi,dtype,layout", [
    ("TINYLLAMA", 8, 16, 512, torch.bfloat16, "HND"),     # configuration 1
    ("LLAMA3_8B", 5, 3000, 9000, torch.bfloat16, "HND"),  # every request split + merged
    ("TINYLLAMA", 6, 1, 300, torch.float16, "NHD"),
    ("LLAMA3_8B", 37, 1, 40, torch.bfloat16, "NHD"),
])
def test_fused_append_matches_append_then_decode(fi, workloads, geom_name, batch, lo, hi, dtype,
                                                 layout):
    geom = getattr(workloads, geom_name)
    prob = workloads.make_decode_problem(geom, batch, lo, hi, seed=batch + hi, num_layers=1,
                                         dtype=dtype, pool_pages=None)
    pool = prob.pool[0]
    if layout == "NHD":
        pool = pool.permute(0, 1, 3, 2, 4).contiguous()  # [N, 2, P, H, D]
    k_new, v_new = prob.k_new.to(DEV), prob.v_new.to(DEV)
    pool_a, out_a, pool_b, out_b = _both_paths(fi, prob, pool, layout, k_new, v_new,
                                               prob.positions)
    assert torch.equal(pool_a, pool_b)
    assert torch.equal(out_a, out_b)
    want_pool = pool.clone()
    paged_kv.append_paged_kv_cache(prob.k_new, prob.v_new, np.arange(prob.batch),
                                   prob.positions, want_pool, prob.kv_indices, prob.kv_indptr,
                                   layout=layout)
    assert torch.equal(pool_b, want_pool)
    hnd = want_pool if layout == "HND" else want_pool.permute(0, 1, 3, 2, 4)
    want, _ = attention.decode(prob.q, hnd.float(), prob.kv_indptr, prob.kv_indices,
                               prob.kv_last_page_len)
    mx, mean, ok = attention.compare(out_b, want, MAX_ABS, MEAN_ABS)
    assert ok, f"max-abs {mx:.3e} mean-abs {mean:.3e}"


def test_fused_append_strided_rows_from_fused_qkv(fi, workloads):
    """k and v are views of the fused QKV projection output (llama.py:163-171)."""
    g = workloads.TINYLLAMA
    prob = workloads.make_decode_problem(g, 7, 20, 260, seed=31, num_layers=1)
    qkv = torch.randn(7, (32 + 8) * 64, dtype=torch.bfloat16)
    qkv[:, 32 * 64:36 * 64] = prob.k_new.reshape(7, -1)
    qkv[:, 36 * 64:] = prob.v_new.reshape(7, -1)
    _, k_view, v_view = qkv.to(DEV).split([32 * 64, 4 * 64, 4 * 64], dim=-1)
    k_view, v_view = k_view.view(-1, 4, 64), v_view.view(-1, 4, 64)
    assert not k_view.is_contiguous()
    pool_a, out_a, pool_b, out_b = _both_paths(fi, prob, prob.pool[0], "HND", k_view, v_view,
                                               prob.positions)
    assert torch.equal(pool_a, pool_b)
    assert torch.equal(out_a, out_b)


def test_fused_append_over_reserved_table(fi, workloads):
    """The reference's decode table may carry one page more than get_len needs
    (admission_controller.py:275); the new token then lands in the page before
    the last one, and the fused call follows the given position exactly."""
    L = 48
    prob = workloads.make_decode_problem(workloads.TINYLLAMA, 2, 0, 0, seed=9, num_layers=1,
                                         lengths=np.array([L + 16, 20]), pool_pages=12)
    positions = np.array([L - 1, 19])  # request 0's token goes to page 2 of 4, slot 15
    pool_a, out_a, pool_b, out_b = _both_paths(fi, prob, prob.pool[0], "HND",
                                               prob.k_new.to(DEV), prob.v_new.to(DEV), positions)
    assert torch.equal(pool_a, pool_b)
    assert torch.equal(out_a, out_b)
    page = int(prob.kv_indices[2])
    assert torch.equal(pool_b[page, 0, :, 15], prob.k_new[0])


def test_fused_append_flags_out_of_range_position(fi, lir, workloads):
    import importlib
    fa = importlib.import_module("llm-inference-runtime_b200.flashinfer_api")
    prob = workloads.make_decode_problem(workloads.TINYLLAMA, 3, 10, 40, seed=5, num_layers=1)
    positions = prob.positions.copy()
    positions[1] = int(prob.kv_indptr[2] - prob.kv_indptr[1]) * 16  # one page past the table
    pool = prob.pool[0].to(DEV)
    before = pool.clone()
    w = fa.BatchDecodeWithPagedKVCacheWrapper(torch.empty(128 << 20, dtype=torch.uint8,
                                                          device=DEV), "HND")
    w.plan(_t(prob.kv_indptr), _t(prob.kv_indices), _t(prob.kv_last_page_len), 32, 4, 64, 16,
           q_data_type=torch.bfloat16)
    torch.cuda.synchronize()
    lir._lib.device_status()
    saved = fa._CHECK
    fa._CHECK = False
    try:
        w.run_with_append(prob.q.to(DEV), pool, prob.k_new.to(DEV), prob.v_new.to(DEV),
                          _t(positions))
        assert lir._lib.device_status() == lir._lib.PA_ERR_DEVICE_CHECK
    finally:
        fa._CHECK = saved
    # requests 0 and 2 were appended, request 1 left its pages untouched
    want = before.cpu()
    keep = [0, 2]
    paged_kv.append_paged_kv_cache(prob.k_new[keep], prob.v_new[keep], np.array(keep),
                                   prob.positions[keep], want, prob.kv_indices, prob.kv_indptr)
    assert torch.equal(pool.cpu(), want)


def test_fused_append_rejects_bad_rows(fi, workloads):
    prob = workloads.make_decode_problem(workloads.TINYLLAMA, 3, 10, 40, seed=6, num_layers=1)
    w = fi.BatchDecodeWithPagedKVCacheWrapper(torch.empty(128 << 20, dtype=torch.uint8,
                                                          device=DEV), "HND")
    w.plan(_t(prob.kv_indptr), _t(prob.kv_indices), _t(prob.kv_last_page_len), 32, 4, 64, 16,
           q_data_type=torch.bfloat16)
    pool = prob.pool[0].to(DEV)
    k = prob.k_new.to(DEV)
    with pytest.raises(ValueError):
        w.run_with_append(prob.q.to(DEV), pool, k[:2], k[:2], _t(prob.positions))
    with pytest.raises(ValueError):
        w.run_with_append(prob.q.to(DEV), pool, k.half(), k.half(), _t(prob.positions))
    with pytest.raises(ValueError):
        w.run_with_append(prob.q.to(DEV), pool, k, k, _t(prob.positions[:2]))


def test_full_size_config2_layer_fused(fi, workloads):
    """Configuration 2 size, one layer (B=256, L~U[1024,4096]) through the fused
    call the bench times: pool rows bit-exact against the two-call sequence,
    outputs bit-identical, oracle on a sample of requests."""
    prob = workloads.make_decode_problem(workloads.TINYLLAMA, 256, 1024, 4096, seed=0,
                                         device=DEV, num_layers=1)
    indptr, indices, last = prob.device_tables(DEV)
    pos = _t(prob.positions)
    w = fi.BatchDecodeWithPagedKVCacheWrapper(torch.empty(128 << 20, dtype=torch.uint8,
                                                          device=DEV), "HND")
    w.plan(indptr, indices, last, 32, 4, 64, 16, q_data_type=torch.bfloat16)
    pool_a = prob.pool[0].clone()
    fi.append_paged_kv_cache(prob.k_new, prob.v_new, _t(np.arange(256)), pos, pool_a, indices,
                             indptr, last, kv_layout="HND")
    out_a = w.run(prob.q, pool_a)
    pool_b = prob.pool[0]
    out_b = w.run_with_append(prob.q, pool_b, prob.k_new, prob.v_new, pos)
    assert torch.equal(pool_a, pool_b)
    assert torch.equal(out_a, out_b)
    sample = [0, 1, 77, 128, 200, 255]
    want, _ = attention.decode(prob.q.cpu(), pool_b.cpu(), prob.kv_indptr, prob.kv_indices,
                               prob.kv_last_page_len, requests=sample)
    mx, mean, ok = attention.compare(out_b.cpu()[sample], want[sample], MAX_ABS, MEAN_ABS)
    assert ok, f"max-abs {mx:.3e} mean-abs {mean:.3e}"


def test_full_size_config5_sampled(fi, workloads):
    """Configuration 5 at full size on one GPU: 512 Llama-3-8B requests with
    contexts ~ U[8192, 32768] (≈43 GB of K/V, every segment split and merged
    in the launch), the step's append fused in; oracle on a sample."""
    prob = workloads.make_decode_problem(workloads.LLAMA3_8B, 512, 8192, 32768, seed=0,
                                         device=DEV, num_layers=1)
    indptr, indices, last = prob.device_tables(DEV)
    w = fi.BatchDecodeWithPagedKVCacheWrapper(torch.empty(128 << 20, dtype=torch.uint8,
                                                          device=DEV), "HND")
    w.plan(indptr, indices, last, 32, 8, 128, 16, q_data_type=torch.bfloat16)
    out, lse = w.run_with_append(prob.q, prob.pool[0], prob.k_new, prob.v_new,
                                 _t(prob.positions), return_lse=True)
    assert torch.isfinite(out).all() and torch.isfinite(lse).all()
    sample = [0, 1, 255, 511]
    # the appended rows landed (bit-exact) in the sampled requests' last slots
    P = 16
    for b in sample:
        pos = int(prob.positions[b])
        page = int(prob.kv_indices[int(prob.kv_indptr[b]) + pos // P])
        assert torch.equal(prob.pool[0][page, 0, :, pos % P], prob.k_new[b])
        assert torch.equal(prob.pool[0][page, 1, :, pos % P], prob.v_new[b])
    want, want_lse = attention.decode(prob.q.cpu(), prob.pool[0], prob.kv_indptr,
                                      prob.kv_indices, prob.kv_last_page_len, requests=sample)
    mx, mean, ok = attention.compare(out.cpu()[sample], want[sample], MAX_ABS, MEAN_ABS)
    assert ok, f"max-abs {mx:.3e} mean-abs {mean:.3e}"
    assert torch.allclose(lse.cpu()[sample], want_lse[sample], atol=1e-3, rtol=1e-4)
