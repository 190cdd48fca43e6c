"""Generates the golden fixtures that pin the CPU oracle to the reference.

Run in a container that has the reference checkout (its ``src/`` on the
import path) — NOT on the GPU box, and not by the tests:

    python tests/golden/make_golden.py /path/to/reference

It drives the reference's own code and records what it produces:

* bookkeeping_trace.json — a scripted + seeded-random sequence of
  BlockAllocator / RadixCache / match_prefix_for_new_run operations
  (src/engine/memory/*.py), with time.time replaced by a counter so the
  LRU order is deterministic. Includes the radix-shared-prefix scenario of
  configuration 4 (64 requests sharing a 2048-token prefix, then LRU
  eviction of 25 % of the unshared pages).
* step_tables.json — the CSR tables StepExecutor._run_prefill /
  _run_decode hand to plan_prefill / plan_decode /
  build_batch_indices_positions (src/engine/runtime/step_executor.py), with
  the model, sampler and tokenizer stubbed out. Includes the decode
  over-reservation case (get_len a multiple of the page size).
* attention_cases.npz — small paged-attention cases (inputs rounded to
  bf16) with outputs of transformers' eager_attention_forward + repeat_kv
  (the eager path the reference patches out) applied to the gathered pages.
* known_answers.json — the worked examples in FlashInfer 0.6.11's
  get_batch_indices_positions / append_paged_kv_cache docstrings
  (flashinfer/page.py), the reference's dependency for these calls.
"""

from __future__ import annotations

import itertools
import json
import math
import os
import random
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(ref_root: str):
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import engine.memory.radix_cache as rc_mod  # noqa: E402
    from engine.memory.allocator import BlockAllocator  # noqa: E402
    from engine.memory.prefix_match import match_prefix_for_new_run  # noqa: E402
    from engine.memory.radix_cache import RadixCache  # noqa: E402
    return rc_mod, BlockAllocator, RadixCache, match_prefix_for_new_run


class _Clock:
    def __init__(self):
        self.it = itertools.count()

    def __call__(self):
        return float(next(self.it))


def bookkeeping_trace(ref_root: str) -> dict:
    rc_mod, BlockAllocator, RadixCache, match_new = _import_reference(ref_root)
    clock = _Clock()
    rc_mod.time.time = clock  # radix_cache.py stamps nodes with time.time()
    P = 16
    out = {"page_size": P, "scenarios": []}

    def alloc(n):
        return BlockAllocator(num_blocks=n, block_size=P, num_layers=1, num_kv_heads=1,
                              head_dim=1, dtype=torch.float16, device="cpu")

    # ---- scenario A: configuration 4 (shared system prefix + eviction)
    clock.it = itertools.count()
    a = alloc(4096)
    cache = RadixCache(block_size=P, allocator=a)
    rng = random.Random(4)
    prefix = [rng.randrange(32000) for _ in range(2048)]
    ops = []
    tables = []
    for r in range(64):
        suffix_len = rng.randint(32, 256)
        toks = prefix + [rng.randrange(32000) for _ in range(suffix_len)]
        mt, mb = match_new(cache, a, toks)
        need = math.ceil(len(toks) / P) - len(mb)
        new = a.allocate(need)
        table = mb + new
        tables.append(table)
        ops.append({"op": "admit", "tokens_len": len(toks), "suffix_len": suffix_len,
                    "matched_tokens": len(mt), "matched_blocks": mb, "allocated": new})
        # the first request's prompt is inserted after its prefill
        if r == 0:
            ins = cache.insert(toks, table)
            ops.append({"op": "insert", "request": 0, "new": ins})
        # every request inserts its full prompt when its prefill completes
        else:
            ins = cache.insert(toks, table)
            ops.append({"op": "insert", "request": r, "new": ins})
    state_before = {"free_blocks": list(a.free_blocks), "ref_counts": list(a.ref_counts)}
    # requests finish: the sequence drops its own references
    for r, table in enumerate(tables):
        a.decref(table)
    unshared = sum(1 for b, c in enumerate(a.ref_counts) if c == 1)
    ev_n = unshared // 4
    evicted = cache.evict_lru(ev_n)
    ops.append({"op": "evict_lru", "num_blocks": ev_n, "evicted": evicted})
    out["scenarios"].append({
        "name": "config4_shared_prefix", "prefix": prefix, "ops": ops, "tables": tables,
        "state_before_finish": state_before,
        "final": {"free_blocks": list(a.free_blocks), "ref_counts": list(a.ref_counts)},
        "seed": 4,
    })

    # ---- scenario B: seeded random operation fuzz
    for seed in range(3):
        clock.it = itertools.count()
        rng = random.Random(100 + seed)
        a = alloc(96)
        cache = RadixCache(block_size=P, allocator=a)
        live = []  # (tokens, table)
        corpus = [[rng.randrange(50) for _ in range(rng.randint(1, 70))] for _ in range(6)]
        ops = []
        for step in range(160):
            kind = rng.choice(["admit", "admit", "finish", "evict", "decode_grow"])
            if kind == "admit":
                base = rng.choice(corpus)
                toks = base[:rng.randint(1, len(base))] + [rng.randrange(50)
                                                           for _ in range(rng.randint(0, 20))]
                mt, mb = match_new(cache, a, toks)
                need = math.ceil(len(toks) / P) - len(mb)
                ok = a.try_allocate(need, cache)
                rec = {"op": "admit", "tokens": toks, "matched_tokens": len(mt),
                       "matched_blocks": mb, "ok": ok}
                if ok:
                    new = a.allocate(need)
                    rec["allocated"] = new
                    table = mb + new
                    rec["inserted"] = cache.insert(toks, table)
                    live.append((toks, table))
                else:
                    a.decref(mb)
                ops.append(rec)
            elif kind == "finish" and live:
                i = rng.randrange(len(live))
                toks, table = live.pop(i)
                ins = cache.insert(toks, table)
                a.decref(table)
                ops.append({"op": "finish", "index": i, "inserted": ins})
            elif kind == "evict":
                n = rng.randint(1, 8)
                ops.append({"op": "evict_lru", "num_blocks": n, "evicted": cache.evict_lru(n)})
            elif kind == "decode_grow" and live:
                i = rng.randrange(len(live))
                toks, table = live[i]
                toks = toks + [rng.randrange(50)]
                need = math.ceil((len(toks) + 1) / P) - len(table)
                got = []
                if need > 0 and a.try_allocate(need, cache):
                    got = a.allocate(need)
                live[i] = (toks, table + got)
                ops.append({"op": "decode_grow", "index": i, "token": toks[-1],
                            "allocated": got})
            ops[-1]["free_blocks"] = list(a.free_blocks)
            ops[-1]["ref_counts"] = list(a.ref_counts)
        out["scenarios"].append({"name": f"fuzz_{seed}", "seed": 100 + seed, "corpus": corpus,
                                 "ops": ops})
    return out


def step_tables(ref_root: str) -> dict:
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import engine.runtime.step_executor as se  # noqa: E402
    from engine.memory.allocator import BlockAllocator  # noqa: E402
    from engine.request import InferenceRequest  # noqa: E402
    from engine.sequence import Sequence  # noqa: E402

    captured = {}

    def cap_plan_prefill(**kw):
        captured["plan_prefill"] = {k: (v.tolist() if isinstance(v, torch.Tensor) else v)
                                    for k, v in kw.items()}

    def cap_plan_decode(**kw):
        captured["plan_decode"] = {k: (v.tolist() if isinstance(v, torch.Tensor) else v)
                                   for k, v in kw.items()}

    def cap_bip(append_indptr, seq_lens):
        captured["bip"] = {"append_indptr": append_indptr.tolist(), "seq_lens": seq_lens.tolist()}

    se.plan_prefill = cap_plan_prefill
    se.plan_decode = cap_plan_decode
    se.build_batch_indices_positions = cap_bip

    class _Out:
        def __init__(self, n0, n1):
            self.logits = torch.zeros(n0, n1, 8)

    class _Model:
        device = torch.device("cpu")

        def __call__(self, input_ids, position_ids, use_cache):
            captured["input_ids"] = input_ids.tolist()
            captured["position_ids"] = position_ids.tolist()
            return _Out(*input_ids.shape)

    class _Tok:
        def decode(self, ids, skip_special_tokens=True):
            return "x" * len(ids)

    P = 16
    ex = se.StepExecutor(model=_Model(), tokenizer=_Tok(), block_size=P, max_chunk_size=512,
                         num_qo_heads=32, num_kv_heads=4, head_dim=64,
                         sampler=lambda logits, seqs: [7] * len(seqs))
    a = BlockAllocator(num_blocks=512, block_size=P, num_layers=1, num_kv_heads=1, head_dim=1,
                       dtype=torch.float16, device="cpu")
    rng = random.Random(7)
    a.free_blocks = rng.sample(range(512), 512)  # scrambled free order
    result = {"page_size": P, "prefill": [], "decode": []}

    def mk(prompt_len, computed, extra_blocks=0):
        req = InferenceRequest(request_id=f"r{rng.randrange(10**9)}", prompt="p")
        seq = Sequence(request=req, prompt_token_ids=[rng.randrange(32000)
                                                       for _ in range(prompt_len)],
                       eos_token_id=2)
        seq.computed_len = computed
        seq.block_table = a.allocate(math.ceil(prompt_len / P) + extra_blocks)
        return seq

    # prefill steps: chunked (computed > 0), exact page boundaries, a zero chunk
    for case in [
        [(37, 0, 37), (16, 0, 16), (100, 32, 48), (5, 0, 5)],
        [(600, 0, 512), (600, 512, 512), (33, 17, 16)],
        [(20, 20, 8), (64, 0, 64), (17, 16, 1)],
    ]:
        seqs = [mk(pl, comp) for pl, comp, _ in case]
        chunk = {id(s): c for s, (_, _, c) in zip(seqs, case)}
        captured.clear()
        pre = [(len(s.prompt_token_ids), s.computed_len, list(s.block_table)) for s in seqs]
        ex._run_prefill(seqs, chunk, se.StepResult(is_prefill=True))
        result["prefill"].append({"seqs": pre, "chunk_lens": [c for _, _, c in case],
                                  "captured": dict(captured)})

    # decode steps; tables carry the scheduler's ceil((get_len + 1) / P) reservation
    for lens in [[17, 32, 1, 16, 48, 100], [15, 16, 31, 64]]:
        seqs = []
        for L in lens:
            s = mk(L - 1, L - 1)
            s.generated_token_ids = [5]
            need = math.ceil((s.get_len + 1) / P) - len(s.block_table)
            if need > 0:
                s.block_table.extend(a.allocate(need))
            seqs.append(s)
        captured.clear()
        pre = [(s.get_len, list(s.block_table)) for s in seqs]
        ex._run_decode(seqs)
        cap = dict(captured)
        cap["batch_indices"] = se.FlashInferState.batch_indices.tolist()
        cap["positions"] = se.FlashInferState.positions.tolist()
        result["decode"].append({"seqs": pre, "captured": cap})
    return result


def _bf16_round(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def attention_cases() -> dict:
    from transformers.models.llama.modeling_llama import eager_attention_forward

    class _M:
        training = False

        def __init__(self, g):
            self.num_key_value_groups = g

    g = torch.Generator().manual_seed(1234)
    arrays = {}

    def tables(lengths, num_pages, perm_gen):
        perm = torch.randperm(num_pages, generator=perm_gen).tolist()
        indptr, indices, last = [0], [], []
        for L in lengths:
            n = math.ceil(L / 16)
            indices.extend(perm[:n])
            perm = perm[n:]
            indptr.append(len(indices))
            last.append(L - (n - 1) * 16 if n > 0 else 0)
        return indptr, indices, last

    def gather(pool, indptr, indices, last, b, layout):
        pages = indices[indptr[b]:indptr[b + 1]]
        blk = pool[pages]
        if layout == "HND":
            k = blk[:, 0].permute(1, 0, 2, 3).reshape(blk.shape[2], -1, blk.shape[4])
            v = blk[:, 1].permute(1, 0, 2, 3).reshape(blk.shape[2], -1, blk.shape[4])
        else:
            k = blk[:, 0].permute(2, 0, 1, 3).reshape(blk.shape[3], -1, blk.shape[4])
            v = blk[:, 1].permute(2, 0, 1, 3).reshape(blk.shape[3], -1, blk.shape[4])
        n = len(pages)
        L = (n - 1) * 16 + last[b]
        return k[:, :L], v[:, :L]

    cases = [
        # name, mode, Hq, Hkv, D, layout, kv lengths, qo lengths (prefill)
        ("decode_tinyllama", "decode", 32, 4, 64, "HND", [1, 15, 16, 33, 200], None),
        ("decode_llama3", "decode", 8, 2, 128, "HND", [17, 48, 5], None),
        ("decode_nhd", "decode", 8, 2, 64, "NHD", [9, 40], None),
        ("prefill_causal", "prefill", 4, 2, 64, "HND", [5, 23, 53], [5, 16, 20]),
        ("prefill_llama3", "prefill", 8, 2, 128, "HND", [40, 130], [40, 3]),
    ]
    index = []
    for name, mode, hq, hkv, d, layout, lens, qlens in cases:
        num_pages = sum(math.ceil(L / 16) for L in lens) + 3
        shape = ((num_pages, 2, hkv, 16, d) if layout == "HND" else (num_pages, 2, 16, hkv, d))
        pool = _bf16_round(torch.randn(shape, generator=g))
        indptr, indices, last = tables(lens, num_pages, g)
        rows = len(lens) if mode == "decode" else sum(qlens)
        q = _bf16_round(torch.randn((rows, hq, d), generator=g))
        out = torch.zeros((rows, hq, d))
        qo_indptr = [0]
        for b, L in enumerate(lens):
            k, v = gather(pool, indptr, indices, last, b, layout)
            if mode == "decode":
                qs, qe = b, b + 1
                mask = None
            else:
                qs, qe = qo_indptr[-1], qo_indptr[-1] + qlens[b]
                qo_indptr.append(qe)
                R = qe - qs
                qpos = torch.arange(R)[:, None] + (L - R)
                mask = torch.where(torch.arange(L)[None, :] > qpos,
                                   torch.finfo(torch.float32).min, 0.0)[None, None]
            query = q[qs:qe].permute(1, 0, 2)[None]  # [1, Hq, R, D]
            o, _ = eager_attention_forward(_M(hq // hkv), query, k[None], v[None], mask,
                                           scaling=d ** -0.5)
            out[qs:qe] = o[0]
        pre = f"{name}__"
        arrays[pre + "pool"] = pool.to(torch.bfloat16).view(torch.int16).numpy()
        arrays[pre + "q"] = q.to(torch.bfloat16).view(torch.int16).numpy()
        arrays[pre + "out"] = out.numpy()
        arrays[pre + "kv_indptr"] = np.array(indptr, dtype=np.int32)
        arrays[pre + "kv_indices"] = np.array(indices, dtype=np.int32)
        arrays[pre + "kv_last_page_len"] = np.array(last, dtype=np.int32)
        if mode == "prefill":
            arrays[pre + "qo_indptr"] = np.array(qo_indptr, dtype=np.int32)
        index.append({"name": name, "mode": mode, "num_qo_heads": hq, "num_kv_heads": hkv,
                      "head_dim": d, "layout": layout})
    arrays["index"] = np.frombuffer(json.dumps(index).encode(), dtype=np.uint8)
    return arrays


def known_answers() -> dict:
    """Worked examples from FlashInfer 0.6.11's docstrings (flashinfer/page.py)."""
    ex1 = {"append_indptr": [0, 1, 3, 6, 10], "seq_lens": [5, 5, 5, 5], "nnz": 10,
           "batch_indices": [0, 1, 1, 2, 2, 2, 3, 3, 3, 3],
           "positions": [4, 3, 4, 2, 3, 4, 1, 2, 3, 4]}
    lens = [45, 8, 25, 22]
    ex2 = {"append_indptr": [0, 45, 53, 78, 100], "kv_page_indptr": [0, 3, 4, 6, 8],
           "kv_last_page_len": [13, 8, 9, 6], "page_size": 16, "nnz": 100,
           "seq_lens": lens,
           "batch_indices": [b for b, L in enumerate(lens) for _ in range(L)],
           "positions": [p for L in lens for p in range(L)]}
    return {"get_batch_indices_positions": [ex1, ex2]}


def main(ref_root: str) -> None:
    with open(os.path.join(HERE, "bookkeeping_trace.json"), "w") as f:
        json.dump(bookkeeping_trace(ref_root), f)
    with open(os.path.join(HERE, "step_tables.json"), "w") as f:
        json.dump(step_tables(ref_root), f)
    np.savez_compressed(os.path.join(HERE, "attention_cases.npz"), **attention_cases())
    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump(known_answers(), f, indent=1)


if __name__ == "__main__":
    # usage: python tests/golden/make_golden.py <checkout of the reference project>
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py REFERENCE_CHECKOUT")
    main(sys.argv[1])
