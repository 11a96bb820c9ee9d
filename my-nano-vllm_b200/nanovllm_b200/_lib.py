"""ctypes binding of ``libfp8attn.so`` (declared in include/fp8attn.h).

The library is the only implementation: if it is missing or fails to load, importing this
module raises -- there is no CPU or Triton fallback.
"""
from __future__ import annotations

import ctypes
import os
import re

from .build import LIB_PATH, INCLUDE

OK, EINVAL, EWORKSPACE, ECUDA = 0, 1, 2, 3
WS_ERROR_OFFSET = 0
NOALLOC_SCRATCH_BYTES = 32 << 20  # FP8ATTN_NOALLOC_SCRATCH_BYTES


class Fp8AttnError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"fp8attn error {code}: {msg}")
        self.code = code


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python my-nano-vllm_b200/nanovllm_b200/build.py` "
            "(there is no fallback implementation)")
    lib = ctypes.CDLL(LIB_PATH)
    i32, i64, f32, vp = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p
    lib.fp8attn_version.restype = i32
    lib.fp8attn_version.argtypes = []
    lib.fp8attn_last_error.restype = ctypes.c_char_p
    lib.fp8attn_last_error.argtypes = []
    lib.fp8attn_set_decode_min_chunk.restype = i32
    lib.fp8attn_set_decode_min_chunk.argtypes = [i32]
    lib.fp8attn_store_kvcache.restype = i32
    lib.fp8attn_store_kvcache.argtypes = [vp, i64, vp, i64, vp, vp, vp, vp, vp, i64, i32, i32,
                                          i64, i32, vp]
    lib.fp8attn_decode_ctas.restype = i32
    lib.fp8attn_decode_ctas.argtypes = [i32, i32, i32, i32]
    lib.fp8attn_workspace_bytes.restype = i64
    lib.fp8attn_workspace_bytes.argtypes = [i32, i32, i32, i32]
    lib.fp8attn_decode.restype = i32
    lib.fp8attn_decode.argtypes = [vp, vp, i64, vp, vp, vp, vp, vp, i64, i32, vp, i32, i32, i32,
                                   i32, i64, i32, f32, vp, i64, vp]
    lib.fp8attn_decode_noalloc.restype = i32
    lib.fp8attn_decode_noalloc.argtypes = [vp, vp, i64, vp, vp, vp, vp, vp, i64, i32, vp, i32, i32,
                                           i32, i32, i64, i32, f32, vp]
    lib.fp8attn_read_error.restype = i32
    lib.fp8attn_read_error.argtypes = [vp, vp, i32, vp]
    lib.fp8attn_noalloc_read_error.restype = i32
    lib.fp8attn_noalloc_read_error.argtypes = [vp, i32, vp]
    lib.fp8attn_fp8_gemm_workspace_bytes.restype = i64
    lib.fp8attn_fp8_gemm_workspace_bytes.argtypes = [i64, i32, i32]
    lib.fp8attn_fp8_linear_workspace_bytes.restype = i64
    lib.fp8attn_fp8_linear_workspace_bytes.argtypes = [i64, i32, i32]
    lib.fp8attn_fp8_dyn_quant.restype = i32
    lib.fp8attn_fp8_dyn_quant.argtypes = [vp, i64, vp, i64, vp, i64, i32, vp]
    lib.fp8attn_fp8_block_gemm.restype = i32
    lib.fp8attn_fp8_block_gemm.argtypes = [vp, i64, vp, vp, vp, vp, i64, i64, i32, i32, vp, i64, vp]
    lib.fp8attn_tp_linear_layout.restype = i64
    lib.fp8attn_tp_linear_layout.argtypes = [i64, i32, i32, vp, vp]
    lib.fp8attn_fp8_tp_linear_workspace_bytes.restype = i64
    lib.fp8attn_fp8_tp_linear_workspace_bytes.argtypes = [i64, i32]
    lib.fp8attn_fp8_tp_linear.restype = i32
    lib.fp8attn_fp8_tp_linear.argtypes = [vp, i64, vp, vp, vp, i32, i32, ctypes.c_uint64, i64,
                                          i64, i32, i32, vp, i64, vp]
    lib.fp8attn_fp8_block_linear.restype = i32
    lib.fp8attn_fp8_block_linear.argtypes = [vp, i64, vp, vp, vp, i64, i64, i32, i32, vp, i64, vp]
    lib.fp8attn_diag_wait_timeout.restype = i32
    lib.fp8attn_diag_wait_timeout.argtypes = [vp, i64, i32, vp]
    lib.fp8attn_diag_exp2.restype = i32
    lib.fp8attn_diag_exp2.argtypes = [vp, vp, vp, i64, vp]
    lib.fp8attn_qk_norm_rope_store.restype = i32
    lib.fp8attn_qk_norm_rope_store.argtypes = [vp, i64, vp, vp, vp, f32, vp, i64, vp, vp, vp, vp,
                                               vp, vp, vp, i64, i32, i32, i32, i64, i32, vp]
    lib.fp8attn_prefill.restype = i32
    lib.fp8attn_prefill.argtypes = [vp, vp, i64, vp, vp, i64, vp, vp, vp, i64, i32, vp, vp, i32,
                                    i32, i32, i32, i32, i32, i64, i32, f32, vp, i64, vp]
    return lib


lib = _load()


def check(rc: int) -> None:
    if rc != OK:
        raise Fp8AttnError(rc, lib.fp8attn_last_error().decode(errors="replace"))


def header_symbols() -> list[str]:
    """Names of the functions declared in include/fp8attn.h."""
    with open(os.path.join(INCLUDE, "fp8attn.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"FP8ATTN_API\s+[\w\s\*]+?\b(fp8attn_\w+)\s*\(", text)))
