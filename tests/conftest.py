"""Shared test setup.

Markers: ``gpu`` tests need a CUDA device (a B200) and the built library;
everything else runs on the CPU. GPU tests fail (not skip) when CUDA is
unavailable, so a GPU run can never pass without the native path.
"""

from __future__ import annotations

import importlib
import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
if REPO not in sys.path:
    sys.path.insert(0, REPO)

os.environ.setdefault("PA_CHECK", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libpaged_attn.so")


def pytest_runtest_setup(item):
    if item.get_closest_marker("gpu") is not None:
        import torch
        if not torch.cuda.is_available():
            pytest.fail("GPU test run without a CUDA device")


@pytest.fixture(scope="session")
def lir():
    return importlib.import_module("llm-inference-runtime_b200")


@pytest.fixture(scope="session")
def fi(lir):
    lir.build.build()
    return importlib.import_module("llm-inference-runtime_b200.flashinfer_api")


@pytest.fixture(scope="session")
def workloads():
    return importlib.import_module("llm-inference-runtime_b200.workloads")


def load_json(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def load_attention_cases():
    """Golden attention cases: list of dicts with bf16 inputs decoded to torch."""
    import torch
    z = np.load(os.path.join(GOLDEN, "attention_cases.npz"))
    index = json.loads(bytes(z["index"]).decode())
    cases = []
    for meta in index:
        pre = meta["name"] + "__"
        case = dict(meta)
        for key in ("pool", "q"):
            case[key] = torch.from_numpy(z[pre + key]).view(torch.bfloat16)
        case["out"] = torch.from_numpy(z[pre + "out"])
        for key in ("kv_indptr", "kv_indices", "kv_last_page_len", "qo_indptr"):
            if pre + key in z.files:
                case[key] = z[pre + key]
        cases.append(case)
    return cases
