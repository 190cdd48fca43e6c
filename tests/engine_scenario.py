"""A short serving scenario driven through the reference's own step executor.

Test infrastructure shared by the engine-swap tests and by
``tests/golden/make_engine_trace.py``. It needs the reference checkout's
``src/`` on the import path (the engine's modules are imported from there,
unmodified): ``StepExecutor.run_step`` (src/engine/runtime/step_executor.py:
61-80) runs four steps over three requests —

1. chunked prefill of all three prompts (21, 20 and 32 of 37, 20, 50 tokens);
2. the rest of prompts 0 and 2 (16 and 18 tokens) with request 1's first
   decode in the same step (``_run_prefill`` then ``_run_decode``);
3. and 4. a decode of all three requests;

with block tables from the reference's ``BlockAllocator`` (scrambled free
list) and, before each decode, the scheduler's reservation of
``ceil((get_len + 1) / P)`` pages (src/engine/scheduling/
admission_controller.py:275). No decode length is a multiple of the page
size, so the reservation never hands the attention stale slots.

The engine imports its attention module by name (``from models.llama import
...``, step_executor.py:8-13): ``import_step_executor`` binds that name to
the module under test, which is exactly the swap a maintainer makes.
"""

from __future__ import annotations

import importlib
import importlib.util
import math
import os
import random
import sys
import types

import torch

P = 16
NUM_PAGES = 64
VOCAB = 512
HIDDEN, HEADS, KV_HEADS, LAYERS = 512, 8, 2, 2  # head_dim 64
HEAD_DIM = HIDDEN // HEADS
PROMPT_LENS = (37, 20, 50)
# per step: prefill chunk length per request, requests decoding
STEPS = [({0: 21, 1: 20, 2: 32}, []),
         ({0: 16, 2: 18}, [1]),
         ({}, [0, 1, 2]),
         ({}, [0, 1, 2])]
SEED = 11


def reference_src() -> str | None:
    """The reference checkout's src/ directory: $PA_REFERENCE_ROOT, else a
    ``reference`` directory beside this repository; None if absent."""
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    root = os.environ.get("PA_REFERENCE_ROOT") or os.path.join(os.path.dirname(here), "reference")
    src = os.path.join(root, "src")
    return src if os.path.isfile(os.path.join(src, "engine", "runtime", "step_executor.py")) \
        else None


def _ensure_path(ref_src: str) -> None:
    if ref_src not in sys.path:
        sys.path.insert(0, ref_src)


def import_step_executor(ref_src: str, llama_module):
    """The reference's step_executor module, freshly imported with
    ``models.llama`` bound to ``llama_module``."""
    _ensure_path(ref_src)
    saved = sys.modules.get("models.llama")
    sys.modules["models.llama"] = llama_module
    sys.modules.pop("engine.runtime.step_executor", None)
    try:
        return importlib.import_module("engine.runtime.step_executor")
    finally:
        if saved is None:
            sys.modules.pop("models.llama", None)
        else:
            sys.modules["models.llama"] = saved


def load_reference_llama(ref_src: str, flashinfer_obj):
    """The reference's unmodified src/models/llama.py, executed with its
    ``import flashinfer`` resolving to ``flashinfer_obj``."""
    _ensure_path(ref_src)
    path = os.path.join(ref_src, "models", "llama.py")
    spec = importlib.util.spec_from_file_location("reference_models_llama", path)
    mod = importlib.util.module_from_spec(spec)
    saved = sys.modules.get("flashinfer")
    sys.modules["flashinfer"] = flashinfer_obj
    try:
        spec.loader.exec_module(mod)
    finally:
        if saved is None:
            sys.modules.pop("flashinfer", None)
        else:
            sys.modules["flashinfer"] = saved
    return mod


class _Tokenizer:
    def decode(self, ids, skip_special_tokens=True):
        return "x" * len(ids)


def row_maps(prompt_lens=PROMPT_LENS, steps=STEPS):
    """(request, position) of every logits row, one list per model call, in
    call order (a step's prefill call precedes its decode call)."""
    computed = [0] * len(prompt_lens)
    generated = [0] * len(prompt_lens)
    maps = []
    for pre, dec in steps:
        if pre:
            rows = []
            for i, c in sorted(pre.items()):
                rows += [(i, p) for p in range(computed[i], computed[i] + c)]
                computed[i] += c
                if computed[i] == prompt_lens[i]:
                    generated[i] += 1  # the prefill's last row samples a token
            maps.append(("prefill", rows))
        if dec:
            maps.append(("decode", [(i, prompt_lens[i] + generated[i] - 1) for i in dec]))
            for i in dec:
                generated[i] += 1
    return maps


def run(se, model, device) -> dict:
    """Runs STEPS through ``se.StepExecutor`` with ``model`` (anything the
    executor can call with input_ids / position_ids / use_cache and read
    ``.device`` and ``.logits`` from). Returns the token streams and block
    tables of the three requests."""
    from engine.memory.allocator import BlockAllocator
    from engine.request import InferenceRequest
    from engine.sequence import Sequence

    rng = random.Random(SEED)
    alloc = BlockAllocator(num_blocks=NUM_PAGES, block_size=P, num_layers=1, num_kv_heads=1,
                           head_dim=1, dtype=torch.float16, device="cpu")
    alloc.free_blocks = rng.sample(range(NUM_PAGES), NUM_PAGES)
    seqs = []
    for i, n in enumerate(PROMPT_LENS):
        req = InferenceRequest(request_id=f"r{i}", prompt="p")
        s = Sequence(request=req, prompt_token_ids=[rng.randrange(VOCAB) for _ in range(n)],
                     eos_token_id=-1)
        s.block_table = alloc.allocate(math.ceil(n / P))
        seqs.append(s)
    sampled = iter([rng.randrange(VOCAB) for _ in range(64)])
    ex = se.StepExecutor(model=model, tokenizer=_Tokenizer(), block_size=P, max_chunk_size=512,
                         num_qo_heads=HEADS, num_kv_heads=KV_HEADS, head_dim=HEAD_DIM,
                         sampler=lambda logits, ss: [next(sampled) for _ in ss])
    for pre, dec in STEPS:
        for i in dec:
            need = math.ceil((seqs[i].get_len + 1) / P) - len(seqs[i].block_table)
            if need > 0:
                seqs[i].block_table.extend(alloc.allocate(need))
        ex.run_step([seqs[i] for i in sorted(pre)], {id(seqs[i]): c for i, c in pre.items()},
                    [seqs[i] for i in dec])
    return {"streams": [s.prompt_token_ids + s.generated_token_ids for s in seqs],
            "block_tables": [list(s.block_table) for s in seqs]}


class LogitsRecorder:
    """Wraps a model so each call's logits are kept (as float32 on the CPU)."""

    def __init__(self, model):
        self.model = model
        self.device = model.device
        self.logits = []

    def __call__(self, **kwargs):
        with torch.no_grad():
            out = self.model(**kwargs)
        self.logits.append(out.logits.float().cpu())
        return out


def tiny_llama(device, dtype):
    """Random-init LLaMA of the scenario's geometry (HF eager attention)."""
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=VOCAB, hidden_size=HIDDEN, intermediate_size=2 * HIDDEN,
                      num_hidden_layers=LAYERS, num_attention_heads=HEADS,
                      num_key_value_heads=KV_HEADS, max_position_embeddings=1024)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).to(dtype).to(device).eval()


def eager_logits(model, streams):
    """Per request: HF eager logits [len, vocab] over its whole token stream."""
    out = []
    for s in streams:
        ids = torch.tensor([s], dtype=torch.long, device=model.device)
        with torch.no_grad():
            out.append(model(input_ids=ids, use_cache=False).logits[0].float().cpu())
    return out


# ------------------------------------------------------------ call recording
def recording_llama_module(events: list):
    """A stand-in ``models.llama`` that records what the engine does with it:
    calls of build_batch_indices_positions / plan_prefill / plan_decode
    (positional and keyword arguments as given) and direct assignments to
    FlashInferState attributes (the decode path sets batch_indices and
    positions itself, step_executor.py:216-221)."""

    def enc(v):
        if isinstance(v, torch.Tensor):
            return {"tensor": v.tolist(), "dtype": str(v.dtype).replace("torch.", "")}
        return v

    def recorder(name):
        def fn(*args, **kwargs):
            events.append({"call": name, "args": [enc(a) for a in args],
                           "kwargs": {k: enc(v) for k, v in kwargs.items()}})
        return fn

    class _Meta(type):
        def __setattr__(cls, key, value):
            events.append({"set": key, "value": enc(value)})
            super().__setattr__(key, value)

    class FlashInferState(metaclass=_Meta):
        batch_indices = None
        positions = None

    mod = types.ModuleType("models.llama")
    mod.FlashInferState = FlashInferState
    for name in ("build_batch_indices_positions", "plan_prefill", "plan_decode"):
        setattr(mod, name, recorder(name))
    return mod


class RecordingModel:
    """Model stand-in for trace generation: records the call, returns zeros."""

    def __init__(self, events: list):
        self.events = events
        self.device = torch.device("cpu")

    def __call__(self, **kwargs):
        self.events.append({"model": {k: (v.tolist() if isinstance(v, torch.Tensor) else v)
                                      for k, v in kwargs.items()}})
        ids = kwargs["input_ids"]
        return types.SimpleNamespace(logits=torch.zeros(ids.shape[0], ids.shape[1], VOCAB))


def decode_value(v, device):
    """Inverse of the recorder's encoding: tensors come back on ``device``."""
    if isinstance(v, dict) and "tensor" in v:
        return torch.tensor(v["tensor"], dtype=getattr(torch, v["dtype"]), device=device)
    return v
