"""Drop-in for nanovllm/kernels/fp8_linear.py: the FP8 block-scaled linear layer.

``fp8_block_linear(x, weight, weight_scale)`` <- nanovllm/kernels/fp8_linear.py:93-139 (called by
LinearBase.apply_linear, nanovllm/layers/linear.py:58): y = x . weight^T with an e4m3 weight in
128 x 128 blocks (bf16 ``weight_scale`` [N / 128, K / 128]) and the activation quantised per
token and 128-column group on the fly.  Its two stages are also exposed:

``fp8_dyn_quant(x)``  <- fp8_dyn_quant_kernel (:11-31): (xq e4m3 [M, K], x_scale bf16 [M, K/128])
``fp8_block_gemm(xq, x_scale, weight, weight_scale)`` <- fp8_block_gemm_kernel (:34-71)

All launch on ``torch.cuda.current_stream()``, allocate their outputs with ``torch.empty`` and
never synchronise, so they can be captured into CUDA graphs.  Activations and outputs are bf16
(the reference also accepts fp16; that is rejected here).
"""
from __future__ import annotations

import torch

from . import _lib
from .fp8_attention import _stream, workspace

BLOCK_SIZE = 128


def _check_weight(weight: torch.Tensor, weight_scale: torch.Tensor, K: int) -> int:
    assert weight.dtype == torch.float8_e4m3fn and weight.dim() == 2 and weight.is_contiguous()
    assert weight_scale.dtype == torch.bfloat16 and weight_scale.is_contiguous()
    N = weight.shape[0]
    assert weight.shape[1] == K
    assert tuple(weight_scale.shape) == (N // BLOCK_SIZE, K // BLOCK_SIZE)
    assert N % BLOCK_SIZE == 0 and K % BLOCK_SIZE == 0
    return N


def fp8_dyn_quant(x: torch.Tensor):
    """x: bf16 [M, K] (K a multiple of 128, unit column stride).  Returns (xq, x_scale)."""
    assert x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(-1) == 1
    M, K = x.shape
    xq = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x.device)
    xs = torch.empty((M, K // BLOCK_SIZE), dtype=torch.bfloat16, device=x.device)
    _lib.check(_lib.lib.fp8attn_fp8_dyn_quant(x.data_ptr(), x.stride(0), xq.data_ptr(), K,
                                              xs.data_ptr(), M, K, _stream(x.device)))
    return xq, xs


def fp8_block_gemm(xq: torch.Tensor, x_scale: torch.Tensor, weight: torch.Tensor,
                   weight_scale: torch.Tensor) -> torch.Tensor:
    """xq: e4m3 [M, K]; x_scale: bf16 [M, K / 128] contiguous.  Returns bf16 [M, N]."""
    assert xq.dtype == torch.float8_e4m3fn and xq.dim() == 2 and xq.stride(-1) == 1
    M, K = xq.shape
    N = _check_weight(weight, weight_scale, K)
    assert x_scale.dtype == torch.bfloat16 and x_scale.is_contiguous()
    assert tuple(x_scale.shape) == (M, K // BLOCK_SIZE)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=xq.device)
    if M == 0:
        return out
    nbytes = _lib.lib.fp8attn_fp8_gemm_workspace_bytes(M, N, K)
    ws = workspace(xq.device, nbytes)
    _lib.check(_lib.lib.fp8attn_fp8_block_gemm(
        xq.data_ptr(), xq.stride(0), x_scale.data_ptr(), weight.data_ptr(), weight_scale.data_ptr(),
        out.data_ptr(), N, M, N, K, ws.data_ptr(), ws.numel(), _stream(xq.device)))
    return out


def fp8_block_linear(x: torch.Tensor, weight: torch.Tensor,
                     weight_scale: torch.Tensor) -> torch.Tensor:
    """x: bf16 [M, K]; weight: e4m3 [N, K]; weight_scale: bf16 [N / 128, K / 128].
    Returns bf16 [M, N] = x . weight^T (quantise, then the block-scaled GEMM)."""
    assert x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(-1) == 1
    M, K = x.shape
    N = _check_weight(weight, weight_scale, K)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    if M == 0:
        return out
    nbytes = _lib.lib.fp8attn_fp8_linear_workspace_bytes(M, N, K)
    ws = workspace(x.device, nbytes)
    _lib.check(_lib.lib.fp8attn_fp8_block_linear(
        x.data_ptr(), x.stride(0), weight.data_ptr(), weight_scale.data_ptr(), out.data_ptr(), N,
        M, N, K, ws.data_ptr(), ws.numel(), _stream(x.device)))
    return out
