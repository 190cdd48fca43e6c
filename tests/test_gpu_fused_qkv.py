"""Fused QKV projection -> RoPE -> KV append against an fp32 reference.

Floating point: the fused kernel rotates the fp32 accumulator, so it is
compared with fp32 math within bf16 output tolerance (max-abs 2e-2,
mean-abs 2e-3 for O(1) values), and with the unfused sequence (16-bit qkv,
then RoPE + append) within the same tolerance. Pool slots that no token
targets must be untouched, bit for bit.
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from oracle import paged_kv

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def fused():
    return importlib.import_module("llm-inference-runtime_b200.fused")


def _case(rng, m, hidden, hq, hkv, d, layout, dtype):
    P, N = 16, 400
    # tokens spread over a few requests with ragged positions, plus padding rows
    B = 5
    per = np.full(B, m // B)
    per[: m % B] += 1
    prefix = rng.integers(0, 300, B)
    seq = prefix + per
    npages = (seq + P - 1) // P
    indptr = np.concatenate([[0], np.cumsum(npages)]).astype(np.int32)
    indices = rng.permutation(N)[: indptr[-1]].astype(np.int32)
    append_indptr = np.concatenate([[0], np.cumsum(per)]).astype(np.int32)
    nnz = m + 2
    bi, pos = paged_kv.batch_indices_positions(append_indptr, seq, nnz)
    x = torch.from_numpy(rng.standard_normal((nnz, hidden), dtype=np.float32)).to(dtype)
    w = torch.from_numpy(rng.standard_normal(((hq + 2 * hkv) * d, hidden), dtype=np.float32)
                         / np.sqrt(hidden)).to(dtype)
    shape = (N, 2, hkv, P, d) if layout == "HND" else (N, 2, P, hkv, d)
    pool = torch.from_numpy(rng.standard_normal(shape, dtype=np.float32)).to(dtype)
    return dict(x=x, w=w, pool=pool, bi=bi, pos=pos, indices=indices, indptr=indptr, nnz=nnz)


def _t(a):
    return torch.as_tensor(np.asarray(a, dtype=np.int32)).to(DEV)


@pytest.mark.parametrize("geom", [(2048, 32, 4, 64), (4096, 32, 8, 128)])
@pytest.mark.parametrize("m", [37, 256, 1000])
@pytest.mark.parametrize("layout", ["HND", "NHD"])
def test_fused_qkv_matches_fp32_and_unfused(fused, fi, geom, m, layout):
    hidden, hq, hkv, d = geom
    rng = np.random.default_rng(hidden + m)
    c = _case(rng, m, hidden, hq, hkv, d, layout, torch.bfloat16)
    nnz = c["nnz"]
    theta = 5e5
    pool = c["pool"].to(DEV)
    q = fused.qkv_rope_append(c["x"].to(DEV), c["w"].to(DEV), hq, _t(c["bi"]), _t(c["pos"]), pool,
                              _t(c["indices"]), _t(c["indptr"]), kv_layout=layout,
                              rope_theta=theta)
    # fp32 reference
    qkv = (c["x"].double() @ c["w"].double().T).numpy()
    ref_q = paged_kv.rope_reference(qkv[:, :hq * d].reshape(nnz, hq, d), c["pos"],
                                    rope_theta=theta)
    ref_k = paged_kv.rope_reference(qkv[:, hq * d:(hq + hkv) * d].reshape(nnz, hkv, d),
                                    c["pos"], rope_theta=theta)
    ref_v = qkv[:, (hq + hkv) * d:].reshape(nnz, hkv, d)
    got_q = q.float().cpu().numpy()
    assert np.abs(got_q - ref_q).max() < 2e-2
    assert np.abs(got_q - ref_q).mean() < 2e-3
    want_pool = c["pool"].clone().float()
    paged_kv.append_paged_kv_cache(torch.from_numpy(ref_k).float(),
                                   torch.from_numpy(ref_v).float(), c["bi"], c["pos"], want_pool,
                                   c["indices"], c["indptr"], layout=layout)
    got_pool = pool.float().cpu()
    diff = (got_pool - want_pool).abs()
    assert diff.max() < 2e-2
    # untouched slots are bit-identical
    touched = torch.zeros_like(c["pool"], dtype=torch.bool)
    paged_kv.append_paged_kv_cache(torch.ones(nnz, hkv, d, dtype=torch.bool),
                                   torch.ones(nnz, hkv, d, dtype=torch.bool), c["bi"], c["pos"],
                                   touched, c["indices"], c["indptr"], layout=layout)
    assert torch.equal(pool.cpu()[~touched], c["pool"][~touched])
    # unfused sequence: 16-bit qkv, then RoPE + append
    pool2 = c["pool"].to(DEV)
    qkv16 = c["x"].to(DEV) @ c["w"].to(DEV).T
    q2, k2, v2 = qkv16.split([hq * d, hkv * d, hkv * d], dim=-1)
    q2, k2, v2 = q2.reshape(nnz, hq, d), k2.reshape(nnz, hkv, d), v2.reshape(nnz, hkv, d)
    fi.apply_rope_append(q2, k2, v2, _t(c["bi"]), _t(c["pos"]), pool2, _t(c["indices"]),
                         _t(c["indptr"]), None, kv_layout=layout, rope_theta=theta)
    # the unfused path rounds qkv to 16 bits before rotating: a few bf16 ulps
    # (2^-8 relative each) apart from the fused result
    def rel(a, b):
        return ((a.float() - b.float()).abs() / b.float().abs().clamp(min=1.0)).max().item()
    assert rel(q2, q) < 2 ** -6
    assert rel(pool2, pool) < 2 ** -6


def test_fused_qkv_fp16_and_partial_rotary(fused):
    hidden, hq, hkv, d = 2048, 32, 4, 64
    rng = np.random.default_rng(9)
    c = _case(rng, 100, hidden, hq, hkv, d, "HND", torch.float16)
    nnz = c["nnz"]
    pool = c["pool"].to(DEV)
    q = fused.qkv_rope_append(c["x"].to(DEV), c["w"].to(DEV), hq, _t(c["bi"]), _t(c["pos"]), pool,
                              _t(c["indices"]), _t(c["indptr"]), rotary_dim=32, interleave=True)
    qkv = (c["x"].double() @ c["w"].double().T).numpy()
    ref_q = paged_kv.rope_reference(qkv[:, :hq * d].reshape(nnz, hq, d), c["pos"],
                                    rotary_dim=32, interleave=True)
    got = q.float().cpu().numpy()
    assert np.abs(got - ref_q).max() < 1e-2
    assert np.abs(got - ref_q).mean() < 1e-3


def test_fused_qkv_rejects_unsupported(fused):
    w = torch.zeros(100, 2048, dtype=torch.bfloat16, device=DEV)
    assert not fused.supported(w, 32, 4, 64, torch.bfloat16)


@pytest.mark.parametrize("geom", [(2048, 32, 4, 64), (4096, 32, 8, 128)])
def test_fused_qkv_split_k_is_deterministic(fused, geom):
    # decode-sized batches split K over a cluster of CTAs; the partial tiles
    # are added in a fixed order, so repeated calls agree bit for bit
    hidden, hq, hkv, d = geom
    rng = np.random.default_rng(5)
    c = _case(rng, 37, hidden, hq, hkv, d, "HND", torch.bfloat16)
    outs = []
    for _ in range(3):
        pool = c["pool"].to(DEV)
        q = fused.qkv_rope_append(c["x"].to(DEV), c["w"].to(DEV), hq, _t(c["bi"]), _t(c["pos"]),
                                  pool, _t(c["indices"]), _t(c["indptr"]))
        outs.append((q.cpu(), pool.cpu()))
    for q, pool in outs[1:]:
        assert torch.equal(q, outs[0][0])
        assert torch.equal(pool, outs[0][1])
