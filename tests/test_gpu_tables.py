"""Device-side step tables vs the reference's Python table build.

The golden fixtures were captured by running the reference's StepExecutor
(tests/golden/step_tables.json); random cases are checked against the
oracle's restatement (oracle/tables.py). Integer work: bit-exact.
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from conftest import load_json
from oracle import tables as otab

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def tb():
    return importlib.import_module("llm-inference-runtime_b200.tables")


def _padded(tables, min_width=1):
    width = max([len(t) for t in tables] + [min_width])
    bt = np.full((len(tables), width + 3), -7, dtype=np.int32)  # padding never read
    for i, t in enumerate(tables):
        bt[i, :len(t)] = t
    return torch.from_numpy(bt).to(DEV), torch.tensor([len(t) for t in tables],
                                                      dtype=torch.int32, device=DEV)


def _i(x):
    return torch.tensor(np.asarray(x, dtype=np.int32), device=DEV)


def _decode(tb, seqs, P):
    bt, nb = _padded([t for _, t in seqs])
    out = tb.build_decode_tables(bt, nb, _i([g for g, _ in seqs]), P)
    c = out["counts"].cpu().tolist()
    assert c == [len(seqs), len(seqs), 0]
    n = int(out["kv_indptr"][-1])
    return {"kv_indptr": out["kv_indptr"].cpu().tolist(),
            "kv_indices": out["kv_indices"][:n].cpu().tolist(),
            "kv_last_page_len": out["kv_last_page_len"].cpu().tolist(),
            "batch_indices": out["batch_indices"].cpu().tolist(),
            "positions": out["positions"].cpu().tolist()}


def _prefill(tb, seqs, chunk_lens, P):
    bt, nb = _padded([t for _, _, t in seqs])
    rows_cap = int(sum(max(0, min(c, pl - cp)) for (pl, cp, _), c in zip(seqs, chunk_lens)))
    out = tb.build_prefill_tables(bt, nb, _i([s[0] for s in seqs]), _i([s[1] for s in seqs]),
                                  _i(chunk_lens), P, rows_capacity=rows_cap)
    na, rows, err = out["counts"].cpu().tolist()
    assert err == 0 and rows == rows_cap
    n = int(out["kv_indptr"][na])
    return {"active": out["active"][:na].cpu().tolist(),
            "qo_indptr": out["qo_indptr"][:na + 1].cpu().tolist(),
            "kv_indptr": out["kv_indptr"][:na + 1].cpu().tolist(),
            "kv_indices": out["kv_indices"][:n].cpu().tolist(),
            "kv_last_page_len": out["kv_last_page_len"][:na].cpu().tolist(),
            "seq_lens": out["seq_lens"][:na].cpu().tolist(),
            "positions": out["positions"][:rows].cpu().tolist(),
            "batch_indices": out["batch_indices"][:rows].cpu().tolist()}


def test_decode_tables_match_reference_capture(tb):
    g = load_json("step_tables.json")
    P = g["page_size"]
    for case in g["decode"]:
        got = _decode(tb, case["seqs"], P)
        cap = case["captured"]
        for key in ("kv_indptr", "kv_indices", "kv_last_page_len"):
            assert got[key] == cap["plan_decode"][key], key
        assert got["batch_indices"] == cap["batch_indices"]
        assert got["positions"] == cap["positions"]


def test_prefill_tables_match_reference_capture(tb):
    g = load_json("step_tables.json")
    P = g["page_size"]
    for case in g["prefill"]:
        got = _prefill(tb, case["seqs"], case["chunk_lens"], P)
        cap = case["captured"]
        for key in ("qo_indptr", "kv_indptr", "kv_indices", "kv_last_page_len"):
            assert got[key] == cap["plan_prefill"][key], key
        assert got["seq_lens"] == cap["bip"]["seq_lens"]
        assert got["qo_indptr"] == cap["bip"]["append_indptr"]
        flat_pos = [p for row in cap["position_ids"] for p in row]
        assert got["positions"] == flat_pos


def test_tables_random_vs_oracle(tb):
    rng = np.random.default_rng(0)
    P = 16
    for trial in range(6):
        B = int(rng.integers(1, 1500))
        # decode: some lengths multiple of P with the extra reserved page
        seqs = []
        for _ in range(B):
            L = int(rng.integers(1, 5000))
            pages = -(-L // P) + (1 if (L % P == 0 and rng.random() < 0.5) else 0)
            seqs.append((L, rng.integers(0, 1 << 20, pages).tolist()))
        assert _decode(tb, seqs, P) == otab.decode_tables(seqs, P)
        # prefill with some empty chunks (dropped) and chunks clipped to the prompt
        pseqs, chunks = [], []
        for _ in range(B):
            prompt = int(rng.integers(1, 3000))
            computed = int(rng.integers(0, prompt + 1))
            chunk = int(rng.integers(0, 700))
            table = rng.integers(0, 1 << 20, -(-prompt // P) + int(rng.integers(0, 3))).tolist()
            pseqs.append((prompt, computed, table))
            chunks.append(chunk)
        got = _prefill(tb, pseqs, chunks, P)
        want = otab.prefill_tables(pseqs, chunks, P)
        for key in ("active", "qo_indptr", "kv_indptr", "kv_indices", "kv_last_page_len",
                    "seq_lens", "positions"):
            assert got[key] == want[key], (trial, key)
        # batch index of every row is its output slot
        slots = np.repeat(np.arange(len(want["active"])), np.diff(want["qo_indptr"]))
        assert got["batch_indices"] == slots.tolist()


def test_tables_flag_short_block_table(tb, lir):
    torch.cuda.synchronize()
    lir._lib.device_status()
    bt, nb = _padded([[3, 4]])
    out = tb.build_decode_tables(bt, nb, _i([40]), 16)  # 40 tokens need 3 pages
    assert out["counts"].cpu().tolist() == [0, 0, 1]
    assert lir._lib.device_status() == lir._lib.PA_ERR_DEVICE_CHECK
    out = tb.build_decode_tables(bt, nb, _i([20]), 16, kv_indices_capacity=1)  # capacity
    assert out["counts"].cpu().tolist() == [0, 0, 1]
    assert lir._lib.device_status() == lir._lib.PA_ERR_DEVICE_CHECK


def test_decode_step_from_device_tables_captured_in_cuda_graph(tb, fi, workloads):
    """Table build + plan + decode captured once in a CUDA graph and replayed
    after the lengths change on the device: same output as eager calls."""
    geom = workloads.TINYLLAMA
    prob = workloads.make_decode_problem(geom, 24, 100, 900, seed=4, device=DEV, append=False)
    P = geom.page_size
    tables = [prob.kv_indices[prob.kv_indptr[b]:prob.kv_indptr[b + 1]].tolist()
              for b in range(prob.batch)]
    bt, nb = _padded(tables)
    lens = _i(prob.lengths)
    ws = torch.empty(64 << 20, dtype=torch.uint8, device=DEV)
    wrap = fi.BatchDecodeWithPagedKVCacheWrapper(ws, "HND")
    out = torch.empty_like(prob.q)

    def step():
        t = tb.build_decode_tables(bt, nb, lens, P, kv_indices_capacity=bt.numel())
        wrap.plan(t["kv_indptr"], t["kv_indices"], t["kv_last_page_len"], geom.num_qo_heads,
                  geom.num_kv_heads, geom.head_dim, P, q_data_type=prob.q.dtype)
        wrap.run(prob.q, prob.pool[0], out=out)

    step()
    torch.cuda.synchronize()
    eager = out.clone()
    import importlib as _il
    fa = _il.import_module("llm-inference-runtime_b200.flashinfer_api")
    saved = fa._CHECK
    fa._CHECK = False  # no host synchronisation inside the capture
    try:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()  # warm the allocator on the capture stream
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            step()
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
        # shorter contexts: new lengths on the device, same graph
        lens.copy_(torch.clamp(lens - 37, min=1))
        g.replay()
        torch.cuda.synchronize()
    finally:
        fa._CHECK = saved
    short = out.clone()
    step()  # eager with the new lengths
    torch.cuda.synchronize()
    assert torch.equal(short, out)
    assert not torch.equal(short, eager)


@pytest.mark.parametrize("layers", [1, 22])
def test_fork_pages_copies_every_layer_bit_exact(tb, layers):
    g = torch.Generator().manual_seed(layers)
    pool = torch.randn(layers, 64, 2, 4, 16, 64, generator=g).to(torch.bfloat16)
    src = torch.tensor([3, 9, 9, 40], dtype=torch.int32)  # a page may be forked twice
    dst = torch.tensor([10, 11, 50, 63], dtype=torch.int32)
    want = pool.clone()
    want[:, dst.long()] = pool[:, src.long()]
    gpu = pool.to(DEV)
    tb.fork_pages(gpu if layers > 1 else gpu[0], src.to(DEV), dst.to(DEV))
    assert torch.equal(gpu.cpu(), want)


def test_fork_pages_flags_out_of_range(tb, lir):
    torch.cuda.synchronize()
    lir._lib.device_status()
    pool = torch.zeros(2, 8, 2, 4, 16, 64, dtype=torch.bfloat16, device=DEV)
    tb.fork_pages(pool, _i([1]), _i([8]))
    assert lir._lib.device_status() == lir._lib.PA_ERR_DEVICE_CHECK
    assert torch.count_nonzero(pool) == 0
