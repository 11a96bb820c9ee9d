"""Fused attention-input epilogue: q_norm / k_norm + rotary embedding + K/V store, one kernel.

``qk_norm_rope_store`` replaces, in one launch of ``fp8attn_qk_norm_rope_store``, the chain
Qwen3Attention.forward runs between its QKV projection and the attention kernels
(nanovllm/models/qwen3.py:102-111):

    q = q_norm(q); k = k_norm(k)                 RMSNorm       nanovllm/layers/layernorm.py:16-26
    q, k = rotary_emb(positions, q, k)           RoPE          nanovllm/layers/rotary_embedding.py:37-47
    store_kvcache(k, v, k_cache, v_cache, slots) (inside Attention.forward, attention.py:61-62)

``install(module)`` rebinds ``Qwen3Attention.forward`` of nanovllm.models.qwen3 to a forward that
does the same work through the fused kernel and then runs the attention dispatch of
Attention.forward without its (now done) store.  Everything else -- the projections, the
attention kernels the engine has bound, CUDA-graph capture -- is unchanged.
"""
from __future__ import annotations

import importlib

import torch

from . import _lib


def qk_norm_rope_store(qkv: torch.Tensor, positions: torch.Tensor, q_norm_weight: torch.Tensor,
                       k_norm_weight: torch.Tensor, eps: float, cos_sin_cache: torch.Tensor,
                       num_heads: int, num_kv_heads: int, k_cache: torch.Tensor | None,
                       v_cache: torch.Tensor | None, slot_mapping: torch.Tensor | None,
                       k_scale: torch.Tensor | None = None, v_scale: torch.Tensor | None = None,
                       scaled: bool = False, return_k: bool = False):
    """qkv: bf16 [N, (num_heads + 2 num_kv_heads) * 128] (rows may be strided); positions: int64
    [N]; weights: bf16 [128]; cos_sin_cache: fp32 [max_position, (1,) 128].  Returns (q, k):
    the normalised, rotated q [N, num_heads, 128] bf16 and, with ``return_k``, k the same way
    (else None).  The rotated K and the raw V rows go to the e4m3 caches at ``slot_mapping``
    (rows with slot -1 are skipped; no caches: nothing is stored)."""
    head_dim = 128
    n = qkv.shape[0]
    assert qkv.dtype == torch.bfloat16 and qkv.dim() == 2 and qkv.stride(-1) == 1
    assert qkv.shape[1] == (num_heads + 2 * num_kv_heads) * head_dim
    assert positions.dtype == torch.int64 and positions.is_contiguous() and positions.numel() == n
    for w in (q_norm_weight, k_norm_weight):
        assert w.dtype == torch.bfloat16 and w.is_contiguous() and w.numel() == head_dim
    cs = cos_sin_cache.reshape(-1, head_dim)
    assert cs.dtype == torch.float32 and cs.is_contiguous()
    q = torch.empty(n, num_heads, head_dim, dtype=torch.bfloat16, device=qkv.device)
    k = torch.empty(n, num_kv_heads, head_dim, dtype=torch.bfloat16, device=qkv.device) \
        if return_k else None
    if n == 0:
        return q, k
    if k_cache is not None and k_cache.numel() > 0:
        assert k_cache.dtype == torch.float8_e4m3fn and v_cache.dtype == torch.float8_e4m3fn
        assert k_cache.is_contiguous() and v_cache.is_contiguous()
        assert k_cache.shape[-2:] == (num_kv_heads, head_dim) and k_cache.shape == v_cache.shape
        assert slot_mapping.dtype == torch.int32 and slot_mapping.is_contiguous()
        assert slot_mapping.numel() == n
        num_slots = k_cache.numel() // (num_kv_heads * head_dim)
        kc, vc, sl = k_cache.data_ptr(), v_cache.data_ptr(), slot_mapping.data_ptr()
    else:  # no cache yet (the engine's warm-up run): nothing is stored
        num_slots = 0
        dummy = torch.full((n,), -1, dtype=torch.int32, device=qkv.device)
        kc, vc, sl = q.data_ptr(), q.data_ptr(), dummy.data_ptr()
    ks = vs = 0
    if k_scale is not None or v_scale is not None:
        assert k_scale is not None and v_scale is not None
        for s in (k_scale, v_scale):
            assert s.dtype == torch.float32 and s.is_contiguous() and s.numel() == num_slots * num_kv_heads
        ks, vs = k_scale.data_ptr(), v_scale.data_ptr()
    elif scaled:
        raise ValueError("scaled=True needs k_scale and v_scale")
    _lib.check(_lib.lib.fp8attn_qk_norm_rope_store(
        qkv.data_ptr(), qkv.stride(0), positions.data_ptr(), q_norm_weight.data_ptr(),
        k_norm_weight.data_ptr(), float(eps), cs.data_ptr(), cs.shape[0], q.data_ptr(),
        k.data_ptr() if k is not None else 0, kc, vc, ks, vs, sl, n, num_heads, num_kv_heads,
        head_dim, num_slots, 1 if scaled else 0, torch.cuda.current_stream(qkv.device).cuda_stream))
    return q, k


def _attention_after_store(attn, q, k, v):
    """Attention.forward (nanovllm/layers/attention.py:58-96) from the point after its K/V
    store: the same split of the batch at ``split_pt`` and the same calls of its decode and
    prefill paths (which use whatever kernels nanovllm.layers.attention has bound)."""
    from nanovllm.utils.context import get_context
    context = get_context()
    split_pt = context.split_pt
    block_tables = context.block_tables
    if block_tables is not None:
        d_block_tables = block_tables[:split_pt]
        p_block_tables = block_tables[split_pt:]
        if d_block_tables.numel() == 0:
            d_block_tables = None
        if p_block_tables.numel() == 0:
            p_block_tables = None
    else:
        d_block_tables = p_block_tables = None
    q_d, q_p = q[:split_pt], q[split_pt:]
    if p_block_tables is not None:
        k_p, v_p = attn.k_cache, attn.v_cache
    elif k is not None:
        k_p, v_p = k[split_pt:], v[split_pt:]
    else:  # no prefill rows: the prefill path is not taken
        k_p = v_p = None
    outs = []
    if len(q_d) > 0:
        outs.append(attn._decode_attention(q_d, attn.k_cache, attn.v_cache, d_block_tables,
                                           context.context_lens))
    if len(q_p) > 0:
        outs.append(attn._prefill_attention(q_p, k_p, v_p, max_seqlen_q=context.max_seqlen_q,
                                            cu_seqlens_q=context.cu_seqlens_q,
                                            max_seqlen_k=context.max_seqlen_k,
                                            cu_seqlens_k=context.cu_seqlens_k,
                                            block_tables=p_block_tables))
    return torch.cat(outs, 0)


def install(module=None):
    """Rebind Qwen3Attention.forward (nanovllm/models/qwen3.py:95-112) of the given module (default
    nanovllm.models.qwen3) to the fused epilogue; returns the previous forward for ``uninstall``.
    Layers the kernel does not cover (a q/k bias instead of the norms, head_dim other than 128,
    non-bf16 norm weights, a cache that is not e4m3) keep the original forward."""
    if module is None:
        module = importlib.import_module("nanovllm.models.qwen3")
    cls = module.Qwen3Attention
    original = cls.forward

    def forward(self, positions, hidden_states):
        attn = self.attn
        has_cache = attn.k_cache.numel() > 0
        if (self.qkv_bias or self.head_dim != 128 or self.q_norm.weight.dtype != torch.bfloat16
                or (has_cache and attn.k_cache.dtype != torch.float8_e4m3fn)):
            return original(self, positions, hidden_states)
        from nanovllm.utils.context import get_context
        context = get_context()
        qkv = self.qkv_proj(hidden_states)
        # the bf16 k is needed only by the prefill path that reads k and v directly (no tables)
        need_k = not has_cache or context.block_tables is None
        q, k = qk_norm_rope_store(
            qkv, positions, self.q_norm.weight, self.k_norm.weight, self.q_norm.eps,
            self.rotary_emb.cos_sin_cache, self.num_heads, self.num_kv_heads,
            attn.k_cache if has_cache else None, attn.v_cache if has_cache else None,
            context.slot_mapping if has_cache else None, return_k=need_k)
        v = qkv[:, self.q_size + self.kv_size:].view(-1, self.num_kv_heads, self.head_dim)
        o = _attention_after_store(attn, q, k, v)
        return self.o_proj(o.flatten(1, -1))

    cls.forward = forward
    return original


def uninstall(original, module=None):
    if module is None:
        module = importlib.import_module("nanovllm.models.qwen3")
    module.Qwen3Attention.forward = original
