"""hachiue_b200 - B200 (sm_100a) backend for hachiue's attention hot path.

GQA decode attention over the KV cache (qwen3 / qwen35 full attention),
causal sliding-window attention (plamo3) and the Gated DeltaNet gated
delta-rule recurrence (qwen35), as hand-written CUDA kernels behind the C ABI
in include/hachiue_cuda.h.  ``CudaBackend`` is the Python host of that ABI and
mirrors the reference's attention-dispatch seam (src/engine.ts:1056-1075).
"""
from ._lib import (KV_BF16, KV_F16, KV_F32, KV_Q8_0, KV_Q8_0_WGSL, HachiueError, LIB_PATH, load)  # noqa: F401

__all__ = ["CudaBackend", "KVCache", "SHADERS", "HachiueError", "KV_F32", "KV_F16", "KV_BF16", "KV_Q8_0", "KV_Q8_0_WGSL",
           "LIB_PATH", "load"]


def __getattr__(name):
    # torch is imported lazily so that the C-ABI checks can run without it.
    if name in ("CudaBackend", "KVCache", "SHADERS", "f32_word"):
        from . import backend
        return getattr(backend, name)
    raise AttributeError(name)
