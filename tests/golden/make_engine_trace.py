"""Records what the reference's step executor hands its attention module.

Run where the reference checkout is present (not on the GPU box, not by the
tests' GPU half):

    python tests/golden/make_engine_trace.py [REFERENCE_CHECKOUT]

(default: $PA_REFERENCE_ROOT, else a ``reference`` directory beside this
repository). It imports the reference's unmodified
src/engine/runtime/step_executor.py with ``models.llama`` bound to a
recording stand-in, runs the scenario of ``tests/engine_scenario.py`` (four
steps: chunked prefill, prefill + decode in one step, two decodes) and
writes ``engine_trace.json``:

* ``events`` — in order, every call the executor made into ``models.llama``
  (build_batch_indices_positions, plan_prefill, plan_decode) with its
  positional and keyword arguments exactly as given, every assignment to a
  ``FlashInferState`` attribute, and every model call (input_ids,
  position_ids, use_cache);
* ``streams`` — each request's prompt + sampled tokens;
* ``rows`` — the (request, position) of every logits row of every model call.

The GPU test replays these events against this package's ``llama`` module
on a real model and compares the logits with transformers' eager attention.
"""

from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import engine_scenario as sc  # noqa: E402


def trace(ref_src: str) -> dict:
    events: list = []
    se = sc.import_step_executor(ref_src, sc.recording_llama_module(events))
    res = sc.run(se, sc.RecordingModel(events), "cpu")
    return {"geometry": {"page_size": sc.P, "num_pages": sc.NUM_PAGES, "vocab": sc.VOCAB,
                         "hidden": sc.HIDDEN, "heads": sc.HEADS, "kv_heads": sc.KV_HEADS,
                         "layers": sc.LAYERS},
            "events": events, "streams": res["streams"],
            "rows": [{"mode": m, "rows": r} for m, r in sc.row_maps()]}


def main() -> None:
    if len(sys.argv) > 1:
        os.environ["PA_REFERENCE_ROOT"] = sys.argv[1]
    ref_src = sc.reference_src()
    if ref_src is None:
        sys.exit("reference checkout not found (pass it as the first argument)")
    with open(os.path.join(HERE, "engine_trace.json"), "w") as f:
        json.dump(trace(ref_src), f)
    print("wrote engine_trace.json")


if __name__ == "__main__":
    main()
