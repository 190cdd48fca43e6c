"""End-to-end drop-in: a LLaMA model patched by this package's llama module.

Mirrors how the reference engine drives its patched model
(src/engine/runtime/step_executor.py:132-167, 204-245): CSR page tables from
the page allocator, build_batch_indices_positions, plan_prefill /
plan_decode, then the HF forward whose attention layers call RoPE, the KV
append and the paged prefill / decode kernels. The logits are compared with
the same weights running transformers' own eager attention.
"""

from __future__ import annotations

import copy
import importlib
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
P = 16


def _model():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=512, hidden_size=512, intermediate_size=1024,
                      num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                      max_position_embeddings=4096)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).to(torch.bfloat16).to(DEV).eval()


def _tables(lengths, pages_per_seq, page_ids):
    indptr = np.concatenate([[0], np.cumsum(pages_per_seq)]).astype(np.int32)
    indices = np.concatenate([page_ids[i] for i in range(len(lengths))]).astype(np.int32)
    last = np.array([L - (math.ceil(L / P) - 1) * P for L in lengths], dtype=np.int32)
    return indptr, indices, last


def _close(got, want):
    got, want = got.float(), want.float()
    rel = (got - want).abs().max() / want.abs().max()
    cos = torch.nn.functional.cosine_similarity(got.flatten(), want.flatten(), dim=0)
    return float(rel), float(cos)


@pytest.mark.parametrize("fused_qkv", [False, True])
def test_patched_model_prefill_then_decode_matches_hf_eager(fi, monkeypatch, fused_qkv):
    """fused_qkv: the projection + RoPE + append kernel instead of the
    projection followed by the RoPE + append kernel."""
    llama = importlib.import_module("llm-inference-runtime_b200.llama")
    monkeypatch.setattr(llama, "_FUSED_QKV", fused_qkv)
    ref = _model()
    ours = copy.deepcopy(ref)
    llama.patch_llama_model(ours)
    hd = 512 // 8
    num_pages = 64
    pool = torch.zeros((2, num_pages, 2, 2, P, hd), dtype=torch.bfloat16, device=DEV)
    llama.init_flashinfer_state(kv_pool=pool, page_size=P, device=DEV)

    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, 512, 37).tolist(), rng.integers(0, 512, 20).tolist()]
    perm = rng.permutation(num_pages)
    # pages reserved for prompt + 2 generated tokens, like the scheduler does
    need = [math.ceil((len(p) + 2) / P) for p in prompts]
    page_ids = [perm[:need[0]], perm[need[0]:need[0] + need[1]]]

    # ---- prefill (two chunks for request 0: 21 then 16 rows, as chunked prefill would)
    t = lambda a: torch.as_tensor(a).to(DEV)  # noqa: E731
    done = [0, 0]
    for chunk in ([21, 20], [16, 0]):
        active = [i for i in range(2) if chunk[i] > 0]
        new_lens = [done[i] + chunk[i] for i in active]
        qo = np.concatenate([[0], np.cumsum([chunk[i] for i in active])]).astype(np.int32)
        indptr, indices, last = _tables(new_lens, [math.ceil(L / P) for L in new_lens],
                                        [page_ids[i][:math.ceil(new_lens[k] / P)]
                                         for k, i in enumerate(active)])
        ids = [tok for i in active for tok in prompts[i][done[i]:done[i] + chunk[i]]]
        pos = [p for i in active for p in range(done[i], done[i] + chunk[i])]
        llama.build_batch_indices_positions(t(qo), t(np.array(new_lens, dtype=np.int32)),
                                            nnz=len(ids))
        llama.plan_prefill(qo_indptr=t(qo), kv_indptr=t(indptr), kv_indices=t(indices),
                           kv_last_page_len=t(last), num_qo_heads=8, num_kv_heads=2, head_dim=hd)
        with torch.no_grad():
            logits = ours(input_ids=t([ids]), position_ids=t([pos]), use_cache=False).logits[0]
        start = 0
        for k, i in enumerate(active):
            end = start + chunk[i]
            with torch.no_grad():
                want = ref(input_ids=t([prompts[i][:done[i] + chunk[i]]]),
                           use_cache=False).logits[0, done[i]:]
            rel, cos = _close(logits[start:end], want)
            assert rel < 0.05 and cos > 0.999, (i, rel, cos)
            start = end
        for i in active:
            done[i] += chunk[i]

    # ---- two decode steps for both requests
    seqs = [list(p) for p in prompts]
    for step in range(2):
        nxt = [int(rng.integers(0, 512)) for _ in seqs]
        for s, tok in zip(seqs, nxt):
            s.append(tok)
        lens = [len(s) for s in seqs]
        indptr, indices, last = _tables(lens, [math.ceil(L / P) for L in lens],
                                        [page_ids[i][:math.ceil(lens[i] / P)] for i in range(2)])
        llama.PagedAttnState.batch_indices = t(np.arange(2, dtype=np.int32))
        llama.PagedAttnState.positions = t(np.array([L - 1 for L in lens], dtype=np.int32))
        llama.plan_decode(kv_indptr=t(indptr), kv_indices=t(indices), kv_last_page_len=t(last),
                          num_qo_heads=8, num_kv_heads=2, head_dim=hd)
        with torch.no_grad():
            logits = ours(input_ids=t([[tok] for tok in nxt]),
                          position_ids=t([[L - 1] for L in lens]), use_cache=False).logits[:, -1]
        for i in range(2):
            with torch.no_grad():
                want = ref(input_ids=t([seqs[i]]), use_cache=False).logits[0, -1]
            rel, cos = _close(logits[i], want)
            assert rel < 0.05 and cos > 0.999, (step, i, rel, cos)


def test_patched_model_decode_step_replays_from_cuda_graph(fi):
    """The patched model's decode step (positions, device plan, forward) is
    captured once in a CUDA graph and replayed: bit-identical logits to the
    eager step, also after the step's device inputs change in place.
    transformers' "sdpa" setting keeps its mask builder off the host for a
    one-token query (the patched attention reads no mask)."""
    llama = importlib.import_module("llm-inference-runtime_b200.llama")
    model = _model()
    llama.patch_llama_model(model)
    model.config._attn_implementation = "sdpa"
    hd = 512 // 8
    num_pages = 64
    g = torch.Generator(device=DEV).manual_seed(3)
    pool = torch.randn((2, num_pages, 2, 2, P, hd), generator=g, device=DEV).to(torch.bfloat16)
    llama.init_flashinfer_state(kv_pool=pool, page_size=P, device=DEV)
    lens = [30, 45, 17]
    rng = np.random.default_rng(4)
    perm = rng.permutation(num_pages)
    npages = [math.ceil(L / P) for L in lens]
    page_ids = [perm[sum(npages[:i]):sum(npages[:i + 1])] for i in range(3)]
    indptr, indices, last = _tables(lens, npages, page_ids)
    t = lambda a: torch.as_tensor(a).to(DEV)  # noqa: E731
    indptr, indices, last = t(indptr), t(indices), t(last)
    seq = t(np.array(lens, dtype=np.int32))
    append_indptr = t(np.arange(4, dtype=np.int32))
    ids = t(rng.integers(0, 512, (3, 1)))

    def step():
        llama.build_batch_indices_positions(append_indptr, seq, nnz=3)
        llama.plan_decode(kv_indptr=indptr, kv_indices=indices, kv_last_page_len=last,
                          num_qo_heads=8, num_kv_heads=2, head_dim=hd)
        with torch.no_grad():
            return model(input_ids=ids, use_cache=False).logits[:, -1]

    lir = importlib.import_module("llm-inference-runtime_b200")
    eager = step().clone()
    saved = fi._CHECK
    fi._CHECK = False  # no host synchronisation inside the capture
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = step()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
        ids.copy_(t(rng.integers(0, 512, (3, 1))))  # new tokens, same buffers
        graph.replay()
        torch.cuda.synchronize()
        replayed = out.clone()
    finally:
        fi._CHECK = saved
    assert lir._lib.device_status() == lir._lib.PA_OK
    assert torch.equal(replayed, step())
    assert not torch.equal(replayed, eager)
