"""Drop-in for the KV store of nanovllm/layers/attention.py.

``store_kvcache`` <- nanovllm/layers/attention.py:33-40 (same signature; the same assertions on
strides as :36-39).  Optional trailing ``k_scale`` / ``v_scale`` (fp32
``[num_blocks, block_size, KVH]``) receive the per-(token, kv-head) scales: 1.0 in the default
parity mode, amax/448 with ``scaled=True``.
"""
from __future__ import annotations

import torch

from . import _lib


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor,
                  k_scale: torch.Tensor | None = None, v_scale: torch.Tensor | None = None,
                  scaled: bool = False) -> None:
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == D and v_cache.stride(1) == D
    assert slot_mapping.numel() == N
    assert key.dtype == torch.bfloat16 and value.dtype == torch.bfloat16
    assert k_cache.dtype == torch.float8_e4m3fn and v_cache.dtype == torch.float8_e4m3fn
    assert k_cache.is_contiguous() and v_cache.is_contiguous()
    assert slot_mapping.dtype == torch.int32 and slot_mapping.is_contiguous()
    num_slots = k_cache.numel() // D
    ks = vs = 0
    if k_scale is not None or v_scale is not None:
        assert k_scale is not None and v_scale is not None
        for s in (k_scale, v_scale):
            assert s.dtype == torch.float32 and s.is_contiguous() and s.numel() == num_slots * num_heads
        ks, vs = k_scale.data_ptr(), v_scale.data_ptr()
    elif scaled:
        raise ValueError("scaled=True needs k_scale and v_scale")
    _lib.check(_lib.lib.fp8attn_store_kvcache(
        key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0), k_cache.data_ptr(),
        v_cache.data_ptr(), ks, vs, slot_mapping.data_ptr(), N, num_heads, head_dim, num_slots,
        1 if scaled else 0, torch.cuda.current_stream(key.device).cuda_stream))
