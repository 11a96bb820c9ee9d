"""Shared helpers for the test-suite: fixture decoding and tolerance checks."""
from __future__ import annotations

import numpy as np
import torch

# Attention tolerance (bf16 output vs an fp32-accumulated reference):
# max |err| <= ATOL + RTOL * |ref| elementwise.
ATOL = 2e-2
RTOL = 1e-2


def bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def u8(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint8))


def fp8(a: np.ndarray) -> torch.Tensor:
    return u8(a).view(torch.float8_e4m3fn)


def assert_close(out: torch.Tensor, ref: torch.Tensor, atol: float = ATOL, rtol: float = RTOL,
                 what: str = ""):
    o = out.detach().float().cpu()
    r = ref.detach().float().cpu()
    assert o.shape == r.shape, (o.shape, r.shape)
    assert torch.isfinite(o).all(), f"{what}: non-finite output"
    err = (o - r).abs()
    bound = atol + rtol * r.abs()
    bad = err > bound
    if bad.any():
        idx = bad.nonzero()[0].tolist()
        raise AssertionError(
            f"{what}: {int(bad.sum())} elements out of tolerance; max abs err {err.max():.3e}; "
            f"first at {idx}: out={o[tuple(idx)]:.5f} ref={r[tuple(idx)]:.5f}")
    return float(err.max())
