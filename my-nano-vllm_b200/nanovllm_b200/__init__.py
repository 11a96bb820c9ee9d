"""B200-native (sm_100a) FP8 PagedAttention hot path for nano-vLLM.

Public API (signatures of the reference's entry points, kept verbatim):

    from nanovllm_b200 import store_kvcache, fp8_decode_attention, fp8_prefill_attention
    from nanovllm_b200.patch import install      # bind them into nanovllm.layers.attention

All three call the C-ABI library ``libfp8attn.so`` (include/fp8attn.h).  The library is loaded
when one of them (or ``nanovllm_b200._lib``) is first imported, and that import raises if the
library is missing: there is no fallback.  The helper modules ``workloads`` and ``shard`` (seeded
benchmark inputs, head ranges) do not need the library, so the CPU-only reference leg of the
benchmark can use them without loading it.
"""
from __future__ import annotations

__all__ = ["store_kvcache", "fp8_decode_attention", "fp8_prefill_attention"]


def __getattr__(name):
    if name == "store_kvcache":
        from .attention import store_kvcache
        return store_kvcache
    if name in ("fp8_decode_attention", "fp8_prefill_attention"):
        from . import fp8_attention
        return getattr(fp8_attention, name)
    raise AttributeError(f"module 'nanovllm_b200' has no attribute {name!r}")
