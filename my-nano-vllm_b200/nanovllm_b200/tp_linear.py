"""Row-parallel FP8 linear layer with its tensor-parallel all-reduce in one kernel.

The reference's ``RowParallelLinear.forward`` (nanovllm/layers/linear.py:235-239) computes
``y = fp8_block_linear(x, weight, weight_scale)`` on each rank's K slice and then
``dist.all_reduce(y)`` through NCCL.  ``fp8_row_parallel_linear`` does both in one launch of
``fp8attn_fp8_tp_linear``: each rank's bf16 result tile is written over NVLink into the tile
owner's receive buffer, the owner adds the ranks' tiles in rank order and writes the sum into
every rank's output buffer.  The buffers are torch symmetric memory (``TpLinearBuffers``), mapped
into every rank's address space.

``install(module)`` rebinds ``RowParallelLinear.forward`` (o_proj and down_proj of Qwen3) for
block-quantised layers without bias when the tensor-parallel size is above 1.  Calls made while a
CUDA graph is being captured keep the original forward: the kernel takes the call's stamp (epoch)
as an argument, which a replayed graph would repeat.
"""
from __future__ import annotations

import ctypes
import importlib

import torch
import torch.distributed as dist

from . import _lib
from .fp8_attention import _stream, workspace


class TpLinearBuffers:
    """Symmetric buffers for calls with up to ``max_tokens`` rows and ``out_features`` outputs.
    Construction is collective over ``group`` (every rank constructs it, in the same order)."""

    def __init__(self, max_tokens: int, out_features: int, group=None, device=None):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.max_tokens, self.out_features = int(max_tokens), int(out_features)
        out_off, recv_off = ctypes.c_int64(), ctypes.c_int64()
        total = _lib.lib.fp8attn_tp_linear_layout(self.max_tokens, self.out_features, self.world,
                                                  ctypes.byref(out_off), ctypes.byref(recv_off))
        if total < 0:
            raise ValueError(f"no layout for max_tokens={max_tokens}, out_features="
                             f"{out_features}, world={self.world}")
        device = torch.device("cuda") if device is None else torch.device(device)
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if hasattr(symm_mem, "enable_symm_mem_for_group"):  # needed by older torch releases
            try:
                symm_mem.enable_symm_mem_for_group(self.group.group_name)
            except Exception:
                pass
        self.buf = symm_mem.empty(total, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, self.group)
        self.ptrs = (ctypes.c_void_p * self.world)(*[int(p) for p in self.handle.buffer_ptrs])
        self.out_offset = out_off.value
        self.epoch = 0
        # every rank's stamps must be zero before any peer's first call writes into them
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    def output(self, m: int) -> torch.Tensor:
        n = self.out_features
        return self.buf[self.out_offset:self.out_offset + m * n * 2].view(torch.bfloat16).view(m, n)


def fp8_row_parallel_linear(x: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
                            bufs: TpLinearBuffers) -> torch.Tensor:
    """x: bf16 [M, K] (this rank's K slice); weight: e4m3 [N, K]; weight_scale: bf16
    [N / 128, K / 128].  Returns the all-reduced bf16 [M, N] -- a view into ``bufs``, valid until
    this rank's next call on them.  Every rank must call with the same M, in the same order."""
    assert x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(-1) == 1
    m, k = x.shape
    n = weight.shape[0]
    assert weight.dtype == torch.float8_e4m3fn and weight.is_contiguous() and weight.shape[1] == k
    assert weight_scale.dtype == torch.bfloat16 and weight_scale.is_contiguous()
    assert tuple(weight_scale.shape) == (n // 128, k // 128)
    assert n == bufs.out_features and m <= bufs.max_tokens
    bufs.epoch += 1
    if m == 0:
        return bufs.output(0)
    ws = workspace(x.device, _lib.lib.fp8attn_fp8_tp_linear_workspace_bytes(m, k))
    _lib.check(_lib.lib.fp8attn_fp8_tp_linear(
        x.data_ptr(), x.stride(0), weight.data_ptr(), weight_scale.data_ptr(), bufs.ptrs,
        bufs.rank, bufs.world, bufs.epoch, bufs.max_tokens, m, n, k, ws.data_ptr(), ws.numel(),
        _stream(x.device)))
    return bufs.output(m)


_BUFFERS: dict[tuple[int, int], TpLinearBuffers] = {}


def install(module=None, max_tokens: int = 16384):
    """Rebind RowParallelLinear.forward of the given module (default nanovllm.layers.linear) to
    the fused kernel; returns the previous forward.  Layers that are not block-quantised, have a
    bias, run with tp_size 1, get more than ``max_tokens`` rows or are called during CUDA-graph
    capture keep the original forward.  The result is copied out of the symmetric buffer, so it
    stays valid like the original's."""
    mod = module if module is not None else importlib.import_module("nanovllm.layers.linear")
    cls = mod.RowParallelLinear
    orig = cls.forward

    def forward(self, x):
        if (not self.quantized or self.tp_size == 1 or self.bias is not None
                or x.shape[0] > max_tokens or torch.cuda.is_current_stream_capturing()):
            return orig(self, x)
        key = (x.device.index, self.weight.shape[0])
        bufs = _BUFFERS.get(key)
        if bufs is None:
            bufs = _BUFFERS[key] = TpLinearBuffers(max_tokens, self.weight.shape[0],
                                                   device=x.device)
        return fp8_row_parallel_linear(x, self.weight, self.weight_scale, bufs).clone()

    cls.forward = forward
    return orig
