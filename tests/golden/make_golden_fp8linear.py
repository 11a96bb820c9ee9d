"""Generate tests/golden/fp8_linear.npz from the reference's own FP8 block-scaled linear layer.

Run on a machine with a CUDA GPU and the reference installed under baseline/_ref (it is NOT
needed at test time):

    python tests/golden/make_golden_fp8linear.py OUT_DIR

For a few seeded shapes (M tokens, K input and N output features) it runs the reference's
fp8_dyn_quant_kernel and fp8_block_linear (nanovllm/kernels/fp8_linear.py:11-31, :93-139) on bf16
activations, e4m3 weights and bf16 block scales, and writes inputs and outputs (the quantised
activation bytes and scales, and y) to OUT_DIR/fp8_linear.npz as arrays named ``<field>_<i>``.
Case 0's first 128-column group of token 0 is all zero (the scale-1 branch), and token 1 holds one
large value (a group whose other elements quantise to small codes).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

SHAPES = [(3, 256, 384), (70, 384, 256), (129, 128, 512)]  # (M, K, N)


def main(out_dir: str) -> None:
    sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
    import torch
    from nanovllm.kernels.fp8_linear import fp8_block_linear, fp8_dyn_quant_kernel

    bits16 = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    bits8 = lambda t: t.detach().cpu().contiguous().view(torch.uint8).numpy()
    arrays = {}
    for i, (m, k, n) in enumerate(SHAPES):
        g = torch.Generator().manual_seed(20261202 + i)
        x = (torch.randn(m, k, generator=g) * 2).to(torch.bfloat16)
        if i == 0:
            x[0, :128] = 0
            x[1, 5] = 3000
        w = (torch.randn(n, k, generator=g) * 0.5).to(torch.float8_e4m3fn)
        ws = (torch.rand(n // 128, k // 128, generator=g) * 0.02 + 0.001).to(torch.bfloat16)
        xd, wd, wsd = x.cuda(), w.cuda(), ws.cuda()
        xq = torch.empty(m, k, dtype=torch.float8_e4m3fn, device="cuda")
        xs = torch.empty(m, k // 128, dtype=torch.bfloat16, device="cuda")
        fp8_dyn_quant_kernel[(m, k // 128)](xd, xq, xs, k // 128, xd.stride(0), xq.stride(0),
                                            BLOCK_K=128, num_warps=4)
        y = fp8_block_linear(xd, wd, wsd)
        torch.cuda.synchronize()
        arrays.update({f"x_{i}": bits16(x), f"w_{i}": bits8(w), f"ws_{i}": bits16(ws),
                       f"xq_{i}": bits8(xq), f"xs_{i}": bits16(xs), f"y_{i}": bits16(y)})
    arrays["shapes"] = np.array(SHAPES, dtype=np.int64)
    np.savez_compressed(os.path.join(out_dir, "fp8_linear.npz"), **arrays)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
