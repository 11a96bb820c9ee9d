"""ctypes binding of the C E4M3 oracle (``oracle/e4m3.c``).  Test infrastructure only.

The shared object is built by ``oracle/Makefile`` into ``oracle/_build/`` (``build()`` runs make
when it is missing).  All functions take and return numpy arrays.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libe4m3_oracle.so")
_lib = None

SATFINITE = 0  # hardware cvt.rn.satfinite semantics (finite overflow -> +-448)
TORCH = 1      # torch .to(float8_e4m3fn) semantics (|x| > 464 -> NaN)


def build() -> str:
    """Compile the C oracle if needed and return the path of the shared object."""
    src = os.path.join(_HERE, "e4m3.c")
    if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE])
    return _SO


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(build())
        p = ctypes.c_void_p
        lib.e4m3_from_bf16_vec.argtypes = [p, p, ctypes.c_int64, ctypes.c_int]
        lib.e4m3_to_f32_vec.argtypes = [p, p, ctypes.c_int64]
        lib.e4m3_quant_rows_bf16.argtypes = [p, p, p, ctypes.c_int64, ctypes.c_int]
        _lib = lib
    return _lib


def from_bf16_bits(bits: np.ndarray, mode: int = SATFINITE) -> np.ndarray:
    """bf16 bit patterns (uint16, any shape) -> e4m3 bytes (uint8, same shape)."""
    src = np.ascontiguousarray(bits, dtype=np.uint16)
    out = np.empty(src.shape, dtype=np.uint8)
    _load().e4m3_from_bf16_vec(src.ctypes.data, out.ctypes.data, src.size, mode)
    return out


def to_f32(codes: np.ndarray) -> np.ndarray:
    """e4m3 bytes (uint8, any shape) -> float32 values (NaN codes -> NaN)."""
    src = np.ascontiguousarray(codes, dtype=np.uint8)
    out = np.empty(src.shape, dtype=np.float32)
    _load().e4m3_to_f32_vec(src.ctypes.data, out.ctypes.data, src.size)
    return out


def quant_rows(bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Scaled quantiser over the last axis: returns (bytes, fp32 scale per row)."""
    src = np.ascontiguousarray(bits, dtype=np.uint16)
    d = src.shape[-1]
    rows = src.size // d
    out = np.empty(src.shape, dtype=np.uint8)
    scales = np.empty(src.shape[:-1], dtype=np.float32)
    _load().e4m3_quant_rows_bf16(src.ctypes.data, out.ctypes.data, scales.ctypes.data, rows, d)
    return out, scales
