"""B200-native (sm_100a) FP8 PagedAttention hot path for nano-vLLM.

Public API (signatures of the reference's entry points, kept verbatim):

    from nanovllm_b200 import store_kvcache, fp8_decode_attention, fp8_prefill_attention
    from nanovllm_b200.patch import install      # bind them into nanovllm.layers.attention

All three call the C-ABI library ``libfp8attn.so`` (include/fp8attn.h); importing this package
fails if the library is missing.
"""
from .attention import store_kvcache
from .fp8_attention import fp8_decode_attention, fp8_prefill_attention

__all__ = ["store_kvcache", "fp8_decode_attention", "fp8_prefill_attention"]
