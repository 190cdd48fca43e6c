"""Runs FlashInfer — the reference's actual GPU attention path — on the golden
attention cases and saves its outputs.

Run on a CUDA machine with flashinfer 0.6.11 installed (JIT-compiles its
kernels on first use); not run by the tests:

    python tests/golden/make_flashinfer_golden.py OUT.npz

The wrappers are built exactly as the reference builds them
(src/models/llama.py:49-67: 128 MiB workspace, default backend, the cases'
kv layout) and called as it calls them: plan via ``begin_forward`` with
``q_data_type`` = the cache dtype (llama.py:106-116, 138-147), decode via
``forward(q, cache)`` (llama.py:236), prefill via ``forward(q, cache,
causal=True)`` (llama.py:218-222). Inputs are the bf16 tensors stored in
attention_cases.npz; outputs are stored as float32. The committed copy
(flashinfer_outputs.npz) is compared with the CPU oracle by
tests/test_oracle_golden.py.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def main(out_path: str) -> None:
    import flashinfer

    z = np.load(os.path.join(HERE, "attention_cases.npz"))
    index = json.loads(bytes(z["index"]).decode())
    dev = torch.device("cuda:0")
    ws = torch.empty(128 * 1024 * 1024, dtype=torch.uint8, device=dev)
    res = {}
    for meta in index:
        pre = meta["name"] + "__"
        pool = torch.from_numpy(z[pre + "pool"]).view(torch.bfloat16).to(dev)
        q = torch.from_numpy(z[pre + "q"]).view(torch.bfloat16).to(dev)
        t = lambda k: torch.from_numpy(z[pre + k]).to(dev)  # noqa: E731
        hq, hkv, d = meta["num_qo_heads"], meta["num_kv_heads"], meta["head_dim"]
        if meta["mode"] == "decode":
            w = flashinfer.BatchDecodeWithPagedKVCacheWrapper(ws, meta["layout"])
            w.begin_forward(t("kv_indptr"), t("kv_indices"), t("kv_last_page_len"), hq, hkv, d,
                            16, q_data_type=torch.bfloat16)
            out = w.forward(q=q, paged_kv_cache=pool)
        else:
            w = flashinfer.BatchPrefillWithPagedKVCacheWrapper(ws, meta["layout"])
            w.begin_forward(t("qo_indptr"), t("kv_indptr"), t("kv_indices"),
                            t("kv_last_page_len"), hq, hkv, d, 16,
                            q_data_type=torch.bfloat16)
            out = w.forward(q=q, paged_kv_cache=pool, causal=True)
        res[pre + "out"] = out.float().cpu().numpy()
        print(meta["name"], "done", flush=True)
    res["flashinfer_version"] = np.frombuffer(flashinfer.__version__.encode(), dtype=np.uint8)
    res["device"] = np.frombuffer(torch.cuda.get_device_name(0).encode(), dtype=np.uint8)
    np.savez_compressed(out_path, **res)


if __name__ == "__main__":
    main(sys.argv[1])
