"""B200 (sm_100a) paged-attention backend for harsh-vsingh/LLM-Inference-Runtime.

Import it by path (the directory name is not a Python identifier):

    import importlib
    lir = importlib.import_module("llm-inference-runtime_b200")
    fi = lir.flashinfer_api      # FlashInfer-compatible operators
    llama = lir.llama            # drop-in for the reference's models/llama.py

Modules:
  _lib           ctypes binding of include/paged_attn.h (libpaged_attn.so)
  build          nvcc build of the library (sm_100a)
  flashinfer_api get_batch_indices_positions, append_paged_kv_cache,
                 apply_rope_pos_ids_inplace, apply_rope_append,
                 Batch{Prefill,Decode}...Wrapper,
                 merge_state(s)
  llama          init_flashinfer_state / plan_* / patched attention forward
  tables         device-side step tables (decode / prefill-chunk CSR build)
  workloads      seeded synthetic configurations (benchmarks and tests)
"""

from . import _lib, build  # noqa: F401

__all__ = ["_lib", "build", "flashinfer_api", "llama", "tables", "workloads"]


def __getattr__(name):
    if name in ("flashinfer_api", "llama", "workloads"):
        import importlib
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
