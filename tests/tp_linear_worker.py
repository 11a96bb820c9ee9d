"""One rank of the row-parallel FP8 linear test (tests/test_tp_linear_gpu.py).  Run as a script, one
process per GPU, with RANK, WORLD_SIZE, MASTER_ADDR and MASTER_PORT set:

    python tests/tp_linear_worker.py OUT_DIR

For seeded shapes (the same inputs on every rank) the rank takes its K slice of the activation,
the weight and the weight scales, as RowParallelLinear's loaders do
(nanovllm/layers/linear.py:215-232), and computes the all-reduced output three ways:
``fp8_row_parallel_linear`` (one kernel), this library's ``fp8_block_linear`` followed by
``dist.all_reduce`` (NCCL), and, when the reference is installed under baseline/_ref, the
reference's own Triton ``fp8_block_linear`` followed by ``dist.all_reduce`` -- the reference's
``RowParallelLinear.forward``.  Outputs (bf16 bits) go to OUT_DIR/rank<r>.npz.
"""
from __future__ import annotations

import datetime
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

# (M tokens, K in_features in all, N out_features, seed): partial token tiles, one token, a
# smaller M after a larger one (the stamps of the larger call's extra tiles stay behind)
CASES = [(256, 4096, 1024, 1), (37, 4096, 1024, 2), (1, 2048, 1024, 3), (1000, 8192, 1024, 4),
         (300, 2048, 1024, 5), (37, 4096, 1024, 6)]
MAX_TOKENS = 1024


def main(out_dir: str) -> None:
    sys.path.insert(0, os.path.join(ROOT, "my-nano-vllm_b200"))
    import torch
    import torch.distributed as dist
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    from nanovllm_b200.fp8_attention import device_error
    from nanovllm_b200.fp8_linear import fp8_block_linear
    from nanovllm_b200.tp_linear import TpLinearBuffers, fp8_row_parallel_linear
    ref_linear = None
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if os.path.isdir(os.path.join(ref_dir, "nanovllm")):
        sys.path.insert(0, ref_dir)
        from nanovllm.kernels.fp8_linear import fp8_block_linear as ref_linear
    bits = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    bufs = TpLinearBuffers(MAX_TOKENS, 1024, device=dev)
    res = {}
    for i, (m, k, n, seed) in enumerate(CASES):
        g = torch.Generator().manual_seed(seed)
        x = (torch.randn(m, k, generator=g) * 2).to(torch.bfloat16)
        w = (torch.randn(n, k, generator=g) * 0.5).to(torch.float8_e4m3fn)
        ws = (torch.rand(n // 128, k // 128, generator=g) * 0.02 + 0.001).to(torch.bfloat16)
        kl = k // world
        xd = x.to(dev)[:, rank * kl:(rank + 1) * kl]          # strided rows, as a view would be
        wd = w[:, rank * kl:(rank + 1) * kl].contiguous().to(dev)
        wsd = ws[:, rank * kl // 128:(rank + 1) * kl // 128].contiguous().to(dev)
        fused = fp8_row_parallel_linear(xd, wd, wsd, bufs).clone()
        base = fp8_block_linear(xd, wd, wsd)
        dist.all_reduce(base)
        res[f"fused_{i}"] = bits(fused)
        res[f"nccl_{i}"] = bits(base)
        if ref_linear is not None:
            r = ref_linear(xd, wd, wsd)
            dist.all_reduce(r)
            res[f"ref_{i}"] = bits(r)
        if i == 0:
            res["x_0"], res["w_0"], res["ws_0"] = bits(x), w.view(torch.uint8).numpy(), bits(ws)
    torch.cuda.synchronize()
    res["device_error"] = np.array(device_error(dev))
    res["epoch"] = np.array(bufs.epoch)
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
