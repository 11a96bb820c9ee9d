"""CPU restatement of the attention-input epilogue that fp8attn_qk_norm_rope_store fuses
(test infrastructure only).

The reference runs, for the q, k, v split of the QKV projection (nanovllm/models/qwen3.py:102-111):
  * RMSNorm.rms_forward (nanovllm/layers/layernorm.py:16-26) on q and k per head of 128 values,
    compiled by torch.compile: r = rsqrt(mean(x^2) + eps) in fp32 and out = bf16((x * r) * w) --
    the compiled function keeps x * r in fp32 before the weight multiply, so there is one bf16
    rounding (the eager function would round x * r to bf16 first);
  * RotaryEmbedding.forward (nanovllm/layers/rotary_embedding.py:37-47, apply_rotary_emb :6-14):
    cos, sin = the fp32 cache row of the token's position; y1 = x1 cos - x2 sin, y2 = x2 cos +
    x1 sin in fp32 over the two halves of the normalised bf16 head, then bf16; compiled, each line
    is one fused multiply-add of its first product and the rounded second;
  * store_kvcache (nanovllm/layers/attention.py:11-40): the rotated k and the raw v rows as e4m3
    at their slots (slot -1 skipped), via oracle.store.

Here the sum of squares is the correctly rounded fp32 value of the exact sum and the rsqrt is
correctly rounded; the GPU kernel (like the compiled reference) sums in a tree and uses the
hardware rsqrt, so a bf16 output can differ from this restatement by one step in rare rows.
"""
from __future__ import annotations

import numpy as np
import torch

from . import store as ostore


def _bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even) -> fp32."""
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def _f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """x: fp32 [..., 128] (bf16 values), w: fp32 [128] (bf16 values) -> fp32 of the bf16 result."""
    ss = _f32(np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True))
    var = _f32(ss / np.float32(128.0))
    r = _f32(1.0 / np.sqrt((var + np.float32(eps)).astype(np.float64)))
    return _bf16_round(_f32(_f32(x * r) * w))


def _fma32(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    # a*b of two fp32 values is exact in fp64; the fp64 sum is rounded once more to fp32
    return _f32(a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64))


def rope(n: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """n: fp32 [N, H, 128] (bf16 values); cos, sin: fp32 [N, 1, 64] -> fp32 of the bf16 result."""
    x1, x2 = n[..., :64], n[..., 64:]
    y1 = _fma32(x1, cos, -_f32(x2 * sin))
    y2 = _fma32(x2, cos, _f32(x1 * sin))
    return _bf16_round(np.concatenate([y1, y2], axis=-1))


def qk_norm_rope_store(qkv: torch.Tensor, positions: torch.Tensor, q_weight: torch.Tensor,
                       k_weight: torch.Tensor, eps: float, cos_sin: torch.Tensor, num_heads: int,
                       num_kv_heads: int, k_cache: np.ndarray | None = None,
                       v_cache: np.ndarray | None = None, slot_mapping: np.ndarray | None = None):
    """qkv: bf16 [N, (Hq + 2 KVH) * 128] (CPU); positions int64 [N]; weights bf16 [128]; cos_sin
    fp32 [max_position, (1,) 128].  Returns (q, k) as bf16 tensors [N, H, 128]; with caches (uint8
    numpy [num_blocks, block_size, KVH, 128]) the rotated k and raw v rows are stored into them."""
    n = qkv.shape[0]
    x = qkv.float().numpy().reshape(n, num_heads + 2 * num_kv_heads, 128)
    qw, kw = q_weight.float().numpy(), k_weight.float().numpy()
    cs = cos_sin.reshape(-1, 128).float().numpy()[positions.numpy()][:, None, :]
    cos, sin = cs[..., :64], cs[..., 64:]
    q = rope(rms_norm(x[:, :num_heads], qw, eps), cos, sin)
    k = rope(rms_norm(x[:, num_heads:num_heads + num_kv_heads], kw, eps), cos, sin)
    qb = torch.from_numpy(q).to(torch.bfloat16)
    kb = torch.from_numpy(k).to(torch.bfloat16)
    if k_cache is not None:
        vb = qkv[:, (num_heads + num_kv_heads) * 128:].reshape(n, num_kv_heads, 128)
        bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
        ostore.store_kvcache(bits(kb), bits(vb), k_cache, v_cache, np.asarray(slot_mapping))
    return qb, kb
