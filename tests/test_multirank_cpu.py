"""KV-head-group sharding (two gloo ranks on CPU): each rank computes attention for its own kv
heads with no collective in the path; gathering the per-rank outputs along the head axis gives
the unsharded result exactly (heads never interact)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nanovllm_b200 import shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed):
    from nanovllm_b200 import workloads
    return workloads.decode_case(5, 16, 4, 1, 300, seed=seed, block_size=32, pool_factor=1.3)


def _rank_main(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import attention as oatt
        c = _case(11)
        kvh = c.k_cache.shape[2]
        q = shard.shard_q(c.q, kvh, rank, world).contiguous()
        kc = shard.shard_cache(c.k_cache.view(torch.uint8), rank, world)
        vc = shard.shard_cache(c.v_cache.view(torch.uint8), rank, world)
        out = oatt.decode(q, kc, vc, c.block_tables, c.context_lens, c.scale)
        # the gather is the test's, standing in for the engine's o_proj all-reduce
        parts = [torch.empty_like(out.float()) for _ in range(world)]
        dist.all_gather(parts, out.float())
        if rank == 0:
            results.put(torch.cat(parts, dim=1))
    finally:
        dist.destroy_process_group()


def test_kv_head_shards_reassemble_the_unsharded_output():
    from oracle import attention as oatt
    world = 2
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = results.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    c = _case(11)
    ref = oatt.decode(c.q, c.k_cache.view(torch.uint8), c.v_cache.view(torch.uint8),
                      c.block_tables, c.context_lens, c.scale).float()
    assert torch.equal(got, ref)


def test_head_ranges():
    assert shard.kv_head_range(8, 3, 4) == (6, 8)
    assert shard.q_head_range(64, 8, 1, 8) == (8, 16)
    assert shard.q_head_range(32, 8, 0, 2) == (0, 16)
    with pytest.raises(ValueError):
        shard.kv_head_range(8, 0, 3)
    with pytest.raises(ValueError):
        shard.kv_head_range(8, 2, 2)


def test_config5_shards_are_slices_of_the_unsharded_batch():
    """Every rank's config-5 inputs are the matching slices of the one-GPU batch: same block
    tables and lengths, its own q heads and kv heads (generated per kv head)."""
    from nanovllm_b200 import workloads
    full = workloads.config5("cpu", gpus=1, rank=0, batch=1)
    for world in (2, 4, 8):
        for rank in (0, world - 1):
            part = workloads.config5("cpu", gpus=world, rank=rank, batch=1)
            k0, k1 = shard.kv_head_range(8, rank, world)
            h0, h1 = shard.q_head_range(64, 8, rank, world)
            assert torch.equal(part.block_tables, full.block_tables)
            assert torch.equal(part.context_lens, full.context_lens)
            assert torch.equal(part.q, full.q[:, h0:h1])
            assert torch.equal(part.k_cache.view(torch.uint8),
                               full.k_cache.view(torch.uint8)[:, :, k0:k1])
            assert torch.equal(part.v_cache.view(torch.uint8),
                               full.v_cache.view(torch.uint8)[:, :, k0:k1])


def _tp_linear_rank(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import fp8_linear as ofl
        x, w, ws = _tp_linear_inputs()
        part = ofl.block_linear(*ofl.rank_slices(x, w, ws, rank, world))  # this rank's bf16 y_r
        y = torch.from_numpy(ofl.bf16_bits_to_f32(part).copy())
        dist.all_reduce(y)                                                 # linear.py:238
        if rank == 0:
            results.put(ofl.f32_to_bf16_bits(y.numpy()))
    finally:
        dist.destroy_process_group()


def _tp_linear_inputs():
    import numpy as np
    g = torch.Generator().manual_seed(23)
    x = (torch.randn(9, 512, generator=g) * 2).to(torch.bfloat16)
    w = (torch.randn(256, 512, generator=g) * 0.5).to(torch.float8_e4m3fn)
    ws = (torch.rand(2, 4, generator=g) * 0.02 + 0.001).to(torch.bfloat16)
    return (x.view(torch.int16).numpy().view(np.uint16), w.view(torch.uint8).numpy(),
            ws.view(torch.int16).numpy().view(np.uint16))


def test_row_parallel_linear_shards_and_all_reduce():
    """RowParallelLinear over two gloo ranks (nanovllm/layers/linear.py:215-239): each rank keeps
    its K slice of x, w and the scale's block columns, computes its bf16 partial, and the sum over
    ranks equals the restatement the fused kernel follows (oracle.fp8_linear.row_parallel_linear)
    exactly, and the unsharded layer within the rounding of the partials."""
    import numpy as np
    from oracle import fp8_linear as ofl
    world = 2
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_linear_rank, args=(r, world, port, results))
             for r in range(world)]
    for p in procs:
        p.start()
    got = results.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, w, ws = _tp_linear_inputs()
    assert np.array_equal(got, ofl.row_parallel_linear(x, w, ws, world))
    full = ofl.bf16_bits_to_f32(ofl.block_linear(x, w, ws)).astype(np.float64)
    err = np.abs(ofl.bf16_bits_to_f32(got) - full)
    assert bool((err <= 2.0 ** -6 * np.abs(full) + 2e-3 * np.abs(full).max()).all()), err.max()
