"""Drop-in for nanovllm/kernels/fp8_attention.py: same entry points, same argument meaning.

``fp8_decode_attention``  <- nanovllm/kernels/fp8_attention.py:173-207
``fp8_prefill_attention`` <- nanovllm/kernels/fp8_attention.py:314-353

Both allocate their output with ``torch.empty_like(q)`` on the current stream (as the reference
does), launch on ``torch.cuda.current_stream()`` and never synchronise or read device memory on
the host, so they can be captured into CUDA graphs (ModelRunner.capture_cudagraph).  Optional
trailing ``k_scale`` / ``v_scale`` (fp32 ``[num_blocks, block_size, KVH]``) enable the scaled
cache format; ``None`` is the reference's unit-scale cache.
"""
from __future__ import annotations

import torch

from . import _lib

_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-initialised scratch for the current stream of ``device`` (grown on demand).  The
    kernels leave its counters at zero after every call, so it is reused without clearing."""
    stream = torch.cuda.current_stream(device)
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           stream.cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def device_error(device: torch.device | None = None) -> int:
    """Largest device-side error word over the workspaces of ``device`` (0 = none).  Reads device
    memory: for tests and diagnostics only."""
    worst = 0
    for (dev, _), ws in _WORKSPACES.items():
        if device is None or dev == torch.device(device).index:
            worst = max(worst, int(ws[:4].view(torch.int32).item()))
    return worst


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check_cache(k_cache: torch.Tensor, v_cache: torch.Tensor):
    assert k_cache.dtype == torch.float8_e4m3fn and v_cache.dtype == torch.float8_e4m3fn
    assert k_cache.shape == v_cache.shape and k_cache.dim() == 4
    assert k_cache.is_contiguous() and v_cache.is_contiguous()


def _check_scales(k_scale, v_scale, rows: int, kvh: int):
    if k_scale is None and v_scale is None:
        return 0, 0
    assert k_scale is not None and v_scale is not None, "give both k_scale and v_scale"
    for s in (k_scale, v_scale):
        assert s.dtype == torch.float32 and s.is_contiguous() and s.numel() == rows * kvh
    return k_scale.data_ptr(), v_scale.data_ptr()


def fp8_decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                         block_tables: torch.Tensor, context_lens: torch.Tensor,
                         softmax_scale: float, k_scale: torch.Tensor | None = None,
                         v_scale: torch.Tensor | None = None) -> torch.Tensor:
    """
    Args:
        q: [batch_size, num_heads, head_dim] bf16
        k_cache: [num_blocks, block_size, num_kv_heads, head_dim] float8_e4m3fn
        v_cache: same
        block_tables: [batch_size, max_num_blocks] int32 (-1 padded)
        context_lens: [batch_size] int32
        softmax_scale: attention scaling factor (1/sqrt(head_dim))
    Returns:
        [batch_size, num_heads, head_dim] attention output (bf16)
    """
    num_heads = q.shape[1]
    num_blocks, block_size, num_kv_heads, head_dim = k_cache.shape
    batch_size, max_num_blocks = block_tables.shape
    _check_cache(k_cache, v_cache)
    assert q.dtype == torch.bfloat16 and q.stride(-1) == 1 and q.stride(1) == head_dim
    assert block_tables.dtype == torch.int32 and block_tables.stride(-1) == 1
    assert context_lens.dtype == torch.int32 and context_lens.is_contiguous()
    assert context_lens.numel() >= batch_size and q.shape[0] == batch_size
    out = torch.empty_like(q) if q.is_contiguous() else torch.empty(
        q.shape, dtype=q.dtype, device=q.device)
    if batch_size == 0:
        return out
    ks, vs = _check_scales(k_scale, v_scale, num_blocks * block_size, num_kv_heads)
    nbytes = _lib.lib.fp8attn_workspace_bytes(batch_size, num_heads, num_kv_heads, 1)
    ws = workspace(q.device, nbytes)
    _lib.check(_lib.lib.fp8attn_decode(
        out.data_ptr(), q.data_ptr(), q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(), ks, vs,
        block_tables.data_ptr(), block_tables.stride(0), max_num_blocks, context_lens.data_ptr(),
        batch_size, num_heads, num_kv_heads, head_dim, num_blocks, block_size,
        float(softmax_scale), ws.data_ptr(), ws.numel(), _stream(q.device)))
    return out


def fp8_prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                          block_tables: torch.Tensor | None, cu_seqlens_q: torch.Tensor,
                          cu_seqlens_k: torch.Tensor, max_seqlen_q: int, max_seqlen_k: int,
                          softmax_scale: float, k_scale: torch.Tensor | None = None,
                          v_scale: torch.Tensor | None = None) -> torch.Tensor:
    """Varlen causal attention over ``cu_seqlens``; k/v are the paged caches when
    ``block_tables`` is given, else contiguous ``[Tk, num_kv_heads, head_dim]`` e4m3 tensors."""
    num_tokens, num_heads, head_dim = q.shape
    num_seqs = cu_seqlens_q.shape[0] - 1
    assert q.dtype == torch.bfloat16 and q.stride(-1) == 1 and q.stride(1) == head_dim
    assert cu_seqlens_q.dtype == torch.int32 and cu_seqlens_k.dtype == torch.int32
    assert cu_seqlens_q.is_contiguous() and cu_seqlens_k.is_contiguous()
    out = torch.empty_like(q) if q.is_contiguous() else torch.empty(
        q.shape, dtype=q.dtype, device=q.device)
    if num_tokens == 0 or num_seqs <= 0:
        return out
    if block_tables is not None:
        _check_cache(k, v)
        num_blocks, block_size, num_kv_heads, _ = k.shape
        assert block_tables.dtype == torch.int32 and block_tables.stride(-1) == 1
        assert block_tables.shape[0] >= num_seqs
        bt_ptr, bt_stride, max_num_blocks = (block_tables.data_ptr(), block_tables.stride(0),
                                             block_tables.shape[1])
        kv_row_stride = num_kv_heads * head_dim
        n_rows = num_blocks
        ks, vs = _check_scales(k_scale, v_scale, num_blocks * block_size, num_kv_heads)
    else:
        assert k.dtype == torch.float8_e4m3fn and v.dtype == torch.float8_e4m3fn
        assert k.stride(-1) == 1 and k.stride(1) == head_dim and k.stride() == v.stride()
        num_kv_heads = k.shape[1]
        block_size, bt_ptr, bt_stride, max_num_blocks = 1, 0, 0, 0
        kv_row_stride = k.stride(0)
        n_rows = k.shape[0]
        ks, vs = _check_scales(k_scale, v_scale, n_rows, num_kv_heads)
    nbytes = _lib.lib.fp8attn_workspace_bytes(num_seqs, num_heads, num_kv_heads,
                                              int(max_seqlen_q))
    ws = workspace(q.device, nbytes)
    _lib.check(_lib.lib.fp8attn_prefill(
        out.data_ptr(), q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), kv_row_stride,
        ks, vs, bt_ptr, bt_stride, max_num_blocks, cu_seqlens_q.data_ptr(),
        cu_seqlens_k.data_ptr(), num_seqs, int(max_seqlen_q), int(max_seqlen_k), num_heads,
        num_kv_heads, head_dim, n_rows, block_size, float(softmax_scale), ws.data_ptr(),
        ws.numel(), _stream(q.device)))
    return out
