"""Batch indices / positions, KV append, RoPE and LSE merge on the GPU.

Integer and byte work is compared bit-exactly with the oracle; RoPE and the
merge (floating point) within stated tolerances.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_json
from oracle import paged_kv

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(a):
    return torch.as_tensor(np.asarray(a, dtype=np.int32)).to(DEV)


def test_batch_indices_positions_known_answers(fi):
    for ex in load_json("known_answers.json")["get_batch_indices_positions"]:
        bi, pos = fi.get_batch_indices_positions(_t(ex["append_indptr"]), _t(ex["seq_lens"]),
                                                 ex["nnz"])
        assert bi.cpu().tolist() == ex["batch_indices"]
        assert pos.cpu().tolist() == ex["positions"]


def test_batch_indices_positions_random_and_padding(fi):
    rng = np.random.default_rng(0)
    for B in (1, 7, 300):
        lens = rng.integers(0, 600, B)
        indptr = np.concatenate([[0], np.cumsum(lens)])
        seq = lens + rng.integers(0, 3000, B)
        nnz = int(indptr[-1]) + 5  # padded tail
        bi, pos = fi.get_batch_indices_positions(_t(indptr), _t(seq), nnz)
        wb, wp = paged_kv.batch_indices_positions(indptr, seq, nnz)
        assert np.array_equal(bi.cpu().numpy(), wb)
        assert np.array_equal(pos.cpu().numpy(), wp)


@pytest.mark.parametrize("layout", ["HND", "NHD"])
@pytest.mark.parametrize("hkv,d", [(4, 64), (8, 128)])
def test_append_bit_exact_chunked_prefill(fi, layout, hkv, d):
    """Ragged append of prefill chunks (positions over several pages)."""
    rng = np.random.default_rng(hkv + d)
    P, N = 16, 300
    chunk = np.array([37, 1, 512, 16])
    prefix = np.array([0, 15, 100, 32])
    seq = prefix + chunk
    npages = (seq + P - 1) // P
    indptr = np.concatenate([[0], np.cumsum(npages)]).astype(np.int32)
    indices = rng.permutation(N)[: indptr[-1]].astype(np.int32)
    last = (seq - (npages - 1) * P).astype(np.int32)
    shape = (N, 2, hkv, P, d) if layout == "HND" else (N, 2, P, hkv, d)
    pool = torch.randn(shape).to(torch.bfloat16)
    qkv = torch.randn(int(chunk.sum()), (32 + 2 * hkv) * d).to(torch.bfloat16)
    _, k, v = qkv.split([32 * d, hkv * d, hkv * d], dim=-1)
    k = k.view(-1, hkv, d)
    v = v.view(-1, hkv, d)
    append_indptr = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
    bi, pos = paged_kv.batch_indices_positions(append_indptr, seq)
    gpu_pool = pool.to(DEV)
    fi.append_paged_kv_cache(k.to(DEV), v.to(DEV), _t(bi), _t(pos), gpu_pool, _t(indices),
                             _t(indptr), _t(last), kv_layout=layout)
    paged_kv.append_paged_kv_cache(k, v, bi, pos, pool, indices, indptr, layout=layout)
    assert torch.equal(gpu_pool.cpu(), pool)


def test_append_flags_out_of_range_position(fi, lir):
    import importlib
    fa = importlib.import_module("llm-inference-runtime_b200.flashinfer_api")
    pool = torch.zeros(4, 2, 4, 16, 64, dtype=torch.bfloat16, device=DEV)
    k = torch.ones(1, 4, 64, dtype=torch.bfloat16, device=DEV)
    torch.cuda.synchronize()
    lir._lib.device_status()
    saved = fa._CHECK
    fa._CHECK = False
    try:
        # request 0 owns one page; position 20 needs a second one
        fi.append_paged_kv_cache(k, k, _t([0]), _t([20]), pool, _t([2]), _t([0, 1]), _t([5]),
                                 kv_layout="HND")
        assert lir._lib.device_status() == lir._lib.PA_ERR_DEVICE_CHECK
    finally:
        fa._CHECK = saved
    assert torch.count_nonzero(pool) == 0


@pytest.mark.parametrize("interleave", [False, True])
def test_rope_matches_float64_reference(fi, interleave):
    g = torch.Generator().manual_seed(3)
    nnz, hq, hkv, d = 40, 32, 4, 64
    qkv = torch.randn(nnz, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 32768, (nnz,), generator=g).to(torch.int32)
    ref_q = paged_kv.rope_reference(qkv[:, :hq * d].view(nnz, hq, d).float().numpy(),
                                    pos.numpy(), interleave=interleave, rope_theta=1e4)
    ref_k = paged_kv.rope_reference(qkv[:, hq * d:(hq + hkv) * d].view(nnz, hkv, d).float()
                                    .numpy(), pos.numpy(), interleave=interleave, rope_theta=1e4)
    gq = qkv.to(DEV)
    q, k, _ = gq.split([hq * d, hkv * d, hkv * d], dim=-1)
    fi.apply_rope_pos_ids_inplace(q.view(nnz, hq, d), k.view(nnz, hkv, d), pos.to(DEV),
                                  interleave=interleave)
    out = gq.cpu().float()
    got_q = out[:, :hq * d].view(nnz, hq, d).numpy()
    got_k = out[:, hq * d:(hq + hkv) * d].view(nnz, hkv, d).numpy()
    # bf16 output rounding: 2^-8 relative of |x| <= ~5
    assert np.abs(got_q - ref_q).max() < 4e-2
    assert np.abs(got_k - ref_k).max() < 4e-2
    assert np.abs(got_q - ref_q).mean() < 4e-3
    # v untouched
    assert torch.equal(out[:, (hq + hkv) * d:], qkv[:, (hq + hkv) * d:].float())


def test_merge_states_matches_float64(fi):
    g = torch.Generator().manual_seed(5)
    n, s, h, d = 9, 5, 8, 128
    v = torch.randn(n, s, h, d, generator=g).to(torch.bfloat16)
    lse = torch.randn(n, s, h, generator=g) * 4
    vm, sm = fi.merge_states(v.to(DEV), lse.to(DEV))
    wv, ws = paged_kv.merge_states(v.float().numpy(), lse.numpy())
    assert np.abs(vm.cpu().float().numpy() - wv).max() < 2e-2
    assert np.abs(sm.cpu().numpy() - ws).max() < 1e-4
    va, sa = fi.merge_state(v[:, 0].to(DEV), lse[:, 0].to(DEV), v[:, 1].to(DEV),
                            lse[:, 1].to(DEV))
    wv2, ws2 = paged_kv.merge_states(v[:, :2].float().numpy(), lse[:, :2].numpy())
    assert np.abs(va.cpu().float().numpy() - wv2).max() < 2e-2


def _rope_append_case(rng, layout, hkv, d, hq=32, dtype=torch.bfloat16):
    P, N = 16, 300
    chunk = np.array([37, 1, 200, 16, 5])
    prefix = np.array([0, 15, 100, 32, 4000])
    seq = prefix + chunk
    npages = (seq + P - 1) // P
    indptr = np.concatenate([[0], np.cumsum(npages)]).astype(np.int32)
    indices = rng.permutation(N)[: indptr[-1]].astype(np.int32)
    last = (seq - (npages - 1) * P).astype(np.int32)
    shape = (N, 2, hkv, P, d) if layout == "HND" else (N, 2, P, hkv, d)
    pool = torch.from_numpy(rng.standard_normal(shape, dtype=np.float32)).to(dtype)
    nnz = int(chunk.sum()) + 3  # three padding rows (batch index -1)
    qkv = torch.from_numpy(rng.standard_normal((nnz, (hq + 2 * hkv) * d),
                                               dtype=np.float32)).to(dtype)
    append_indptr = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
    bi, pos = paged_kv.batch_indices_positions(append_indptr, seq, nnz)
    return dict(pool=pool, qkv=qkv, bi=bi, pos=pos, indices=indices, indptr=indptr, last=last,
                hq=hq, nnz=nnz)


@pytest.mark.parametrize("layout", ["HND", "NHD"])
@pytest.mark.parametrize("hkv,d,rotary", [(4, 64, None), (8, 128, None), (8, 128, 64)])
@pytest.mark.parametrize("interleave", [False, True])
def test_rope_append_fused_equals_separate_calls(fi, layout, hkv, d, rotary, interleave):
    """The fused RoPE + append is bit-identical to RoPE followed by append,
    for q / k rotated in place (strided views of one fused QKV buffer) and
    for every pool byte; padding rows are rotated but not appended."""
    c = _rope_append_case(np.random.default_rng(hkv * d + (rotary or 0)), layout, hkv, d)
    hq, nnz = c["hq"], c["nnz"]
    runs = []
    for fused in (False, True):
        qkv = c["qkv"].to(DEV)
        pool = c["pool"].to(DEV)
        q, k, v = qkv.split([hq * d, hkv * d, hkv * d], dim=-1)
        q, k, v = q.view(nnz, hq, d), k.view(nnz, hkv, d), v.view(nnz, hkv, d)
        args = dict(batch_indices=_t(c["bi"]), positions=_t(c["pos"]), paged_kv_cache=pool,
                    kv_indices=_t(c["indices"]), kv_indptr=_t(c["indptr"]),
                    kv_last_page_len=_t(c["last"]), kv_layout=layout)
        if fused:
            fi.apply_rope_append(q, k, v, rotary_dim=rotary, interleave=interleave,
                                 rope_theta=5e5, **args)
        else:
            fi.apply_rope_pos_ids_inplace(q, k, _t(c["pos"]), rotary_dim=rotary,
                                          interleave=interleave, rope_theta=5e5)
            fi.append_paged_kv_cache(k, v, **args)
        runs.append((qkv.cpu(), pool.cpu()))
    assert torch.equal(runs[0][0], runs[1][0])
    assert torch.equal(runs[0][1], runs[1][1])
    # and the pool equals the oracle's append of the rotated rows
    qkv_rot = runs[1][0]
    _, k_rot, v_rot = qkv_rot.split([hq * d, hkv * d, hkv * d], dim=-1)
    want = c["pool"].clone()
    paged_kv.append_paged_kv_cache(k_rot.reshape(nnz, hkv, d), v_rot.reshape(nnz, hkv, d),
                                   c["bi"], c["pos"], want, c["indices"], c["indptr"],
                                   layout=layout)
    assert torch.equal(runs[1][1], want)


def test_rope_append_fused_fp16_and_unaligned_fallback(fi):
    """fp16, and a rotary_dim that is not a multiple of 16 (two-kernel path)."""
    rng = np.random.default_rng(11)
    for rotary in (None, 40):
        c = _rope_append_case(rng, "HND", 4, 64, dtype=torch.float16)
        hq, nnz, d, hkv = c["hq"], c["nnz"], 64, 4
        outs = []
        for fused in (False, True):
            qkv = c["qkv"].to(DEV)
            pool = c["pool"].to(DEV)
            q, k, v = qkv.split([hq * d, hkv * d, hkv * d], dim=-1)
            q, k, v = q.view(nnz, hq, d), k.view(nnz, hkv, d), v.view(nnz, hkv, d)
            args = dict(batch_indices=_t(c["bi"]), positions=_t(c["pos"]), paged_kv_cache=pool,
                        kv_indices=_t(c["indices"]), kv_indptr=_t(c["indptr"]),
                        kv_last_page_len=_t(c["last"]), kv_layout="HND")
            if fused:
                fi.apply_rope_append(q, k, v, rotary_dim=rotary, **args)
            else:
                fi.apply_rope_pos_ids_inplace(q, k, _t(c["pos"]), rotary_dim=rotary)
                fi.append_paged_kv_cache(k, v, **args)
            outs.append((qkv.cpu(), pool.cpu()))
        assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


def test_rope_append_flags_out_of_range_position(fi, lir):
    import importlib
    fa = importlib.import_module("llm-inference-runtime_b200.flashinfer_api")
    pool = torch.zeros(4, 2, 4, 16, 64, dtype=torch.bfloat16, device=DEV)
    q = torch.ones(1, 32, 64, dtype=torch.bfloat16, device=DEV)
    k = torch.ones(1, 4, 64, dtype=torch.bfloat16, device=DEV)
    torch.cuda.synchronize()
    lir._lib.device_status()
    saved = fa._CHECK
    fa._CHECK = False
    try:
        fi.apply_rope_append(q, k, k.clone(), _t([0]), _t([20]), pool, _t([2]), _t([0, 1]),
                             _t([5]), kv_layout="HND")
        assert lir._lib.device_status() == lir._lib.PA_ERR_DEVICE_CHECK
    finally:
        fa._CHECK = saved
    assert torch.count_nonzero(pool) == 0


@pytest.mark.parametrize("op", ["append", "rope_append", "qkv_rope_append"])
def test_append_flags_indptr_past_the_page_ids(fi, lir, op):
    """kv_indptr ranges must lie inside kv_indices: request 1 claims pages
    2..8 of a 3-entry index array, and a negative start is as bad. Those rows
    are skipped with a device check (no page id is read from outside the
    array); request 0's row lands in its page."""
    import importlib
    fa = importlib.import_module("llm-inference-runtime_b200.flashinfer_api")
    for indptr in ([0, 2, 9], [-1, 2, 3]):
        pool = torch.zeros(4, 2, 4, 16, 64, dtype=torch.bfloat16, device=DEV)
        q = torch.ones(2, 32, 64, dtype=torch.bfloat16, device=DEV)
        k = torch.ones(2, 4, 64, dtype=torch.bfloat16, device=DEV)
        torch.cuda.synchronize()
        lir._lib.device_status()
        saved = fa._CHECK
        fa._CHECK = False
        try:
            args = (_t([0, 1]), _t([3, 20]), pool, _t([1, 2, 3]), _t(indptr), _t([5, 5]))
            if op == "append":
                fi.append_paged_kv_cache(k, k, *args, kv_layout="HND")
            elif op == "rope_append":
                fi.apply_rope_append(q, k, k.clone(), *args, kv_layout="HND")
            else:  # the fused QKV projection's epilogue takes the same page-table checks
                fused = importlib.import_module("llm-inference-runtime_b200.fused")
                x = torch.full((2, 2048), 0.01, dtype=torch.bfloat16, device=DEV)
                w = torch.full(((32 + 2 * 4) * 64, 2048), 0.01, dtype=torch.bfloat16,
                               device=DEV)
                fused.qkv_rope_append(x, w, 32, args[0], args[1], pool, args[3], args[4],
                                      kv_layout="HND")
            assert lir._lib.device_status() == lir._lib.PA_ERR_DEVICE_CHECK
        finally:
            fa._CHECK = saved
        written = torch.nonzero(pool.abs().sum(dim=(1, 2, 4))).tolist()
        if indptr[0] == 0:  # request 0 is valid: its row goes to page 1, slot 3
            assert written == [[1, 3]]
        else:
            assert written == []
