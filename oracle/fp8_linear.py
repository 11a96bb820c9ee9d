"""CPU restatement of the FP8 block-scaled linear layer (test infrastructure only).

The reference (nanovllm/kernels/fp8_linear.py) computes y = x . w^T for an e4m3 weight w [N, K]
stored in 128 x 128 blocks with one bf16 scale each (w_scale [N / 128, K / 128]):

  * fp8_dyn_quant_kernel (:11-31), per token m and 128-column group g:
        s = max|x[m, g]| / 448 in fp32, s = 1 when that is 0;
        xq[m, g] = e4m3(clamp(x[m, g] / s, -448, 448))   (fp32 quotient, round to nearest even);
        x_scale[m, g] = bf16(s)                           (the quotient used the fp32 s);
  * fp8_block_gemm_kernel (:34-71), per output (m, n), over the groups g in order:
        partial = fp32 dot of xq[m, g] and w[n, g]        (tl.dot, fp32 accumulation);
        acc += partial * (fp32(x_scale[m, g]) * fp32(w_scale[n / 128, g]))   (fused multiply-add);
        y[m, n] = bf16(acc).

Here each group's dot is exact (e4m3 products summed in fp64 -- 128 of them span fewer than 53
bits -- then rounded once to fp32) and the update is one fp32 fused multiply-add computed in fp64.
The quotient x / s is the IEEE fp32 quotient: the reference's Triton build divides with the GPU's
approximate fp32 division (within 2 ulp), so an element whose quotient lies within a few ulp of
a rounding midpoint of e4m3 can round the other way there; ``near_midpoint`` marks those.
"""
from __future__ import annotations

import numpy as np
import torch

from . import e4m3

FP8_MAX = 448.0
BLOCK = 128


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16)
    return t.view(torch.int16).numpy().view(np.uint16)


def _quotients(x_bits: np.ndarray):
    """fp32 group scales [M, K/128] and fp32 quotients x / s [M, K]."""
    x = bf16_bits_to_f32(x_bits)
    M, K = x.shape
    g = x.reshape(M, K // BLOCK, BLOCK)
    amax = np.abs(g).max(axis=2) if M else np.zeros((0, K // BLOCK), np.float32)
    s = (amax / np.float32(FP8_MAX)).astype(np.float32)
    s = np.where(s > 0, s, np.float32(1.0)).astype(np.float32)
    q = (g / s[:, :, None]).astype(np.float32).reshape(M, K)
    return s, q


def dyn_quant(x_bits: np.ndarray):
    """x_bits: bf16 bits [M, K].  Returns (xq e4m3 codes uint8 [M, K], x_scale bf16 bits
    [M, K / 128])."""
    s, q = _quotients(x_bits)
    q = np.clip(q, -FP8_MAX, FP8_MAX).astype(np.float32)
    codes = torch.from_numpy(q).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return codes, f32_to_bf16_bits(s)


def _e4m3_midpoints() -> np.ndarray:
    vals = np.unique(np.abs(e4m3.to_f32(np.arange(256, dtype=np.uint8)).astype(np.float64)))
    vals = vals[np.isfinite(vals)]
    vals = vals[vals <= FP8_MAX]
    return (vals[1:] + vals[:-1]) / 2


_MIDS = None


def near_midpoint(x_bits: np.ndarray, ulps: int = 4) -> np.ndarray:
    """Boolean [M, K]: the fp32 quotient x / s lies within ``ulps`` fp32 ulp of a rounding
    midpoint of e4m3 (an element where an approximate division may round the other way)."""
    global _MIDS
    if _MIDS is None:
        _MIDS = _e4m3_midpoints()
    _, q = _quotients(x_bits)
    a = np.abs(q.astype(np.float64))
    i = np.clip(np.searchsorted(_MIDS, a), 1, len(_MIDS) - 1)
    d = np.minimum(np.abs(a - _MIDS[i - 1]), np.abs(a - _MIDS[i]))
    ulp = np.spacing(np.abs(q).astype(np.float32)).astype(np.float64)
    return d <= ulps * ulp


def block_gemm_f32(xq: np.ndarray, xs_bits: np.ndarray, w: np.ndarray,
                   ws_bits: np.ndarray) -> np.ndarray:
    """fp32 accumulators [M, N] before the output rounding (xq, w: e4m3 codes; scales: bf16
    bits)."""
    M, K = xq.shape
    N = w.shape[0]
    kc = K // BLOCK
    xf = e4m3.to_f32(np.ascontiguousarray(xq)).astype(np.float64).reshape(M, K)
    wf = e4m3.to_f32(np.ascontiguousarray(w)).astype(np.float64).reshape(N, K)
    xs = bf16_bits_to_f32(xs_bits).reshape(M, kc)
    wsc = bf16_bits_to_f32(ws_bits).reshape(N // BLOCK, kc)
    acc = np.zeros((M, N), np.float32)
    for g in range(kc):
        cols = slice(g * BLOCK, (g + 1) * BLOCK)
        partial = (xf[:, cols] @ wf[:, cols].T).astype(np.float32)
        scale = (xs[:, g][:, None] * np.repeat(wsc[:, g], BLOCK)[None, :]).astype(np.float32)
        acc = (partial.astype(np.float64) * scale.astype(np.float64)
               + acc.astype(np.float64)).astype(np.float32)
    return acc


def block_gemm(xq: np.ndarray, xs_bits: np.ndarray, w: np.ndarray,
               ws_bits: np.ndarray) -> np.ndarray:
    """y bf16 bits [M, N] of fp8_block_gemm_kernel."""
    return f32_to_bf16_bits(block_gemm_f32(xq, xs_bits, w, ws_bits))


def block_linear(x_bits: np.ndarray, w: np.ndarray, ws_bits: np.ndarray) -> np.ndarray:
    """y bf16 bits [M, N] of fp8_block_linear: quantise x, then the block-scaled GEMM."""
    xq, xs = dyn_quant(x_bits)
    return block_gemm(xq, xs, w, ws_bits)


def rank_slices(x_bits: np.ndarray, w: np.ndarray, ws_bits: np.ndarray, rank: int, world: int):
    """Rank ``rank``'s share of a row-parallel layer, as RowParallelLinear keeps it
    (nanovllm/layers/linear.py:215-232): columns [r K/world, (r+1) K/world) of the activation and
    the weight, and the matching block columns of the weight scale (dim 1)."""
    k = x_bits.shape[1]
    kl = k // world
    return (np.ascontiguousarray(x_bits[:, rank * kl:(rank + 1) * kl]),
            np.ascontiguousarray(w[:, rank * kl:(rank + 1) * kl]),
            np.ascontiguousarray(ws_bits[:, rank * kl // BLOCK:(rank + 1) * kl // BLOCK]))


def row_parallel_linear(x_bits: np.ndarray, w: np.ndarray, ws_bits: np.ndarray,
                        world: int) -> np.ndarray:
    """RowParallelLinear.forward over ``world`` ranks (nanovllm/layers/linear.py:235-239): each
    rank's fp8_block_linear of its slice (bf16), then the all-reduce: the ranks' bf16 values added
    in rank order in fp32 and rounded to bf16 (for two ranks this is what NCCL's sum gives; with
    more, NCCL's order and intermediate rounding may differ by a bf16 step)."""
    acc = None
    for r in range(world):
        part = bf16_bits_to_f32(block_linear(*rank_slices(x_bits, w, ws_bits, r, world)))
        acc = part if acc is None else (acc + part).astype(np.float32)
    return f32_to_bf16_bits(acc)
