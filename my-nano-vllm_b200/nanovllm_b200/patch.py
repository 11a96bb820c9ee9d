"""Bind the B200 entry points into nano-vLLM in place of its Triton kernels.

``Attention.forward`` (nanovllm/layers/attention.py:58-96) calls the module-level names
``store_kvcache`` (:62), ``fp8_decode_attention`` (:100, imported at :7) and
``fp8_prefill_attention`` (:117, imported at :7).  Rebinding those three globals of that module
is the whole integration: the engine, scheduler, block manager and graph capture stay untouched.
"""
from __future__ import annotations

import importlib

from . import attention as _attention
from . import fp8_attention as _fp8

NAMES = ("store_kvcache", "fp8_decode_attention", "fp8_prefill_attention")


def install(module=None):
    """Patch ``nanovllm.layers.attention`` (or the given module object); returns the previous
    bindings so ``uninstall`` can restore them."""
    if module is None:
        module = importlib.import_module("nanovllm.layers.attention")
    previous = {n: getattr(module, n) for n in NAMES}
    module.store_kvcache = _attention.store_kvcache
    module.fp8_decode_attention = _fp8.fp8_decode_attention
    module.fp8_prefill_attention = _fp8.fp8_prefill_attention
    return previous


def uninstall(previous, module=None):
    if module is None:
        module = importlib.import_module("nanovllm.layers.attention")
    for n, f in previous.items():
        setattr(module, n, f)
