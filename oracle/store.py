"""Restatement of the reference KV store (test infrastructure only).

Follows nanovllm/layers/attention.py:11-40:
  * ``store_kvcache`` (:33-40) views each cache as ``[num_slots, KVH*D]`` (``stride(1) == D``,
    asserted at :38) and launches one program per token row;
  * the kernel (:22-31) loads ``slot = slot_mapping[idx]`` and returns when ``slot == -1`` (:24),
    otherwise stores row ``idx`` of key/value (row stride ``key.stride(0)``) into cache row
    ``slot`` with an implicit bf16 -> e4m3 cast.

The optional scale arrays are the store path's extension (the reference cache carries no scale):
parity mode writes 1.0, scaled mode writes amax/448 per (token, kv-head) row.
"""
from __future__ import annotations

import numpy as np

from . import e4m3


def store_kvcache(key_bits: np.ndarray, value_bits: np.ndarray, k_cache: np.ndarray,
                  v_cache: np.ndarray, slot_mapping: np.ndarray, k_scale: np.ndarray | None = None,
                  v_scale: np.ndarray | None = None, scaled: bool = False,
                  mode: int = e4m3.SATFINITE) -> None:
    """In-place store.  ``key_bits``/``value_bits``: uint16 bf16 patterns ``[N, KVH, D]``;
    ``k_cache``/``v_cache``: uint8 ``[num_blocks, BS, KVH, D]``; ``slot_mapping``: int ``[N]``;
    ``k_scale``/``v_scale``: float32 ``[num_blocks*BS, KVH]`` or None."""
    n, kvh, d = key_bits.shape
    slots = np.asarray(slot_mapping).astype(np.int64)
    assert slots.shape == (n,)
    keep = slots != -1
    rows = slots[keep]
    fk = k_cache.reshape(-1, kvh, d)
    fv = v_cache.reshape(-1, kvh, d)
    for src, dst, sc in ((key_bits, fk, k_scale), (value_bits, fv, v_scale)):
        x = np.ascontiguousarray(src[keep])
        if scaled:
            codes, scales = e4m3.quant_rows(x)
        else:
            codes = e4m3.from_bf16_bits(x, mode)
            scales = np.ones(x.shape[:2], dtype=np.float32)
        dst[rows] = codes
        if sc is not None:
            sc.reshape(-1, kvh)[rows] = scales
