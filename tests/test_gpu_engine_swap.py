"""The reference engine's own calls, replayed against this package on a B200.

``tests/golden/engine_trace.json`` holds, in order, every call the
reference's unmodified step executor made into ``models.llama`` over four
serving steps (chunked prefill, prefill + decode in one step, two decodes;
recorded by ``tests/golden/make_engine_trace.py`` from
src/engine/runtime/step_executor.py:82-259), with positional and keyword
arguments exactly as the engine passes them — ``build_batch_indices_positions``
without a row count, direct ``FlashInferState.batch_indices / positions``
assignments on the decode path, the model calls' input_ids / position_ids.
Replayed against this package's ``llama`` module (the swap the integration
guide describes) on a bf16 model, every logits row must match transformers'
eager attention on the same weights (tolerance as the other patched-model
tests: max relative error 5 %, cosine similarity 0.999).

The second test captures the engine's prefill-step calls (positions without
a row count, device plan, one patched attention layer) in a CUDA graph: a
host synchronisation would fail the capture. The replayed outputs are
bit-identical to the eager ones.
"""

from __future__ import annotations

import copy
import importlib
import json
import os

import pytest
import torch

import engine_scenario as sc
from conftest import GOLDEN

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _trace():
    with open(os.path.join(GOLDEN, "engine_trace.json")) as f:
        return json.load(f)


def _close(got, want):
    rel = (got - want).abs().max() / want.abs().max()
    cos = torch.nn.functional.cosine_similarity(got.flatten(), want.flatten(), dim=0)
    return float(rel), float(cos)


@pytest.mark.parametrize("fused_qkv", [False, True])
def test_reference_engine_calls_replayed_match_hf_eager(fi, monkeypatch, fused_qkv):
    tr = _trace()
    llama = importlib.import_module("llm-inference-runtime_b200.llama")
    monkeypatch.setattr(llama, "_FUSED_QKV", fused_qkv)
    ref = sc.tiny_llama(DEV, torch.bfloat16)
    ours = copy.deepcopy(ref)
    llama.patch_llama_model(ours)
    g = tr["geometry"]
    pool = torch.zeros((g["layers"], g["num_pages"], 2, g["kv_heads"], g["page_size"],
                        g["hidden"] // g["heads"]), dtype=torch.bfloat16, device=DEV)
    llama.init_flashinfer_state(kv_pool=pool, page_size=g["page_size"], device=DEV)
    eager = sc.eager_logits(ref, tr["streams"])
    calls = iter(tr["rows"])
    for ev in tr["events"]:
        if "call" in ev:
            fn = getattr(llama, ev["call"])
            fn(*[sc.decode_value(a, DEV) for a in ev["args"]],
               **{k: sc.decode_value(v, DEV) for k, v in ev["kwargs"].items()})
        elif "set" in ev:
            setattr(llama.FlashInferState, ev["set"], sc.decode_value(ev["value"], DEV))
        else:
            kw = dict(ev["model"])
            kw["input_ids"] = torch.tensor(kw["input_ids"], dtype=torch.long, device=DEV)
            kw["position_ids"] = torch.tensor(kw["position_ids"], dtype=torch.long, device=DEV)
            with torch.no_grad():
                logits = ours(**kw).logits.float().cpu()
            rows = next(calls)
            flat = logits.reshape(-1, logits.shape[-1])
            assert flat.shape[0] == len(rows["rows"])
            for k, (i, pos) in enumerate(rows["rows"]):
                rel, cos = _close(flat[k], eager[i][pos])
                assert rel < 0.05 and cos > 0.999, (rows["mode"], i, pos, rel, cos)
    assert next(calls, None) is None
    lir = importlib.import_module("llm-inference-runtime_b200")
    assert lir._lib.device_status() == lir._lib.PA_OK


def test_engine_prefill_step_without_row_count_is_graph_capturable(fi):
    """build_batch_indices_positions(qo_indptr, seq_lens) as the engine calls
    it (step_executor.py:155, no row count), plan_prefill and one patched
    attention layer, captured in a CUDA graph and replayed."""
    tr = _trace()
    ev = [e for e in tr["events"] if "call" in e][:2]  # step 1: positions + prefill plan
    assert ev[0]["call"] == "build_batch_indices_positions" and not ev[0]["kwargs"]
    assert len(ev[0]["args"]) == 2 and ev[1]["call"] == "plan_prefill"
    llama = importlib.import_module("llm-inference-runtime_b200.llama")
    model = sc.tiny_llama(DEV, torch.bfloat16)
    llama.patch_llama_model(model)
    g = tr["geometry"]
    gen = torch.Generator(device=DEV).manual_seed(5)
    pool = torch.randn((g["layers"], g["num_pages"], 2, g["kv_heads"], g["page_size"],
                        g["hidden"] // g["heads"]), generator=gen,
                       device=DEV).to(torch.bfloat16)
    llama.init_flashinfer_state(kv_pool=pool, page_size=g["page_size"], device=DEV)
    args = [sc.decode_value(a, DEV) for a in ev[0]["args"]]
    plan_kw = {k: sc.decode_value(v, DEV) for k, v in ev[1]["kwargs"].items()}
    nnz = int(ev[0]["args"][0]["tensor"][-1])
    x = torch.randn((1, nnz, g["hidden"]), generator=gen, device=DEV).to(torch.bfloat16)
    attn = model.model.layers[0].self_attn

    def step():
        llama.build_batch_indices_positions(*args)
        llama.plan_prefill(**plan_kw)
        with torch.no_grad():
            return attn(x)[0]

    pool0 = pool.clone()
    eager = step().clone()
    eager_pool = pool.clone()
    saved = fi._CHECK
    fi._CHECK = False  # no host synchronisation inside the capture
    try:
        pool.copy_(pool0)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = step()
        pool.copy_(pool0)
        graph.replay()
        torch.cuda.synchronize()
    finally:
        fi._CHECK = saved
    assert torch.equal(out, eager)
    assert torch.equal(pool, eager_pool)  # the layer's KV append, replayed
    lir = importlib.import_module("llm-inference-runtime_b200")
    assert lir._lib.device_status() == lir._lib.PA_OK
