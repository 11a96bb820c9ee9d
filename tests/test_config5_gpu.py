"""Config 5 (Qwen3-32B heads 64 q / 8 kv, 32768-token contexts) split by kv-head group at every
shard geometry the benchmark runs (KVH/Hq per GPU = 8/64, 4/32, 2/16, 1/8 at 1/2/4/8 GPUs), on a
few sequences of the full context length: each rank's output against the fp32 oracle, and the
ranks' outputs against the matching head slices of the unsharded call (the heads never interact,
so a shard must give its slice of the one-GPU result, within the tolerance)."""
import pytest
import torch

from helpers import assert_close
from oracle import attention as oatt

pytestmark = pytest.mark.gpu

BATCH = 3


def _run(c):
    from nanovllm_b200 import fp8_decode_attention
    from nanovllm_b200.fp8_attention import device_error
    out = fp8_decode_attention(c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale)
    torch.cuda.synchronize()
    assert device_error() == 0
    return out


@pytest.fixture(scope="module")
def unsharded():
    from nanovllm_b200 import workloads
    c = workloads.config5("cuda", gpus=1, rank=0, batch=BATCH)
    out = _run(c).cpu()
    ref = oatt.decode(c.q.cpu(), c.k_cache.cpu(), c.v_cache.cpu(), c.block_tables.cpu(),
                      c.context_lens.cpu(), c.scale)
    assert_close(out, ref, what="config5 unsharded")
    return out


@pytest.mark.parametrize("gpus", [2, 4, 8])
def test_config5_shards_match_oracle_and_unsharded_slices(gpus, unsharded):
    from nanovllm_b200 import workloads
    for rank in sorted({0, gpus - 1}):
        c = workloads.config5("cuda", gpus=gpus, rank=rank, batch=BATCH)
        assert c.k_cache.shape[2] == 8 // gpus and c.q.shape[1] == 64 // gpus
        out = _run(c).cpu()
        ref = oatt.decode(c.q.cpu(), c.k_cache.cpu(), c.v_cache.cpu(), c.block_tables.cpu(),
                          c.context_lens.cpu(), c.scale)
        assert_close(out, ref, what=f"config5 rank {rank}/{gpus}")
        h0, h1 = c.meta["q_heads"]
        assert_close(out, unsharded[:, h0:h1], what=f"config5 rank {rank}/{gpus} vs unsharded")
        del c
        torch.cuda.empty_cache()


def test_config5_shard_inputs_are_slices_of_the_unsharded_batch():
    from nanovllm_b200 import workloads
    full = workloads.config5("cuda", gpus=1, rank=0, batch=1)
    part = workloads.config5("cuda", gpus=4, rank=2, batch=1)
    assert torch.equal(part.block_tables, full.block_tables)
    assert torch.equal(part.q, full.q[:, 32:48])
    assert torch.equal(part.k_cache.view(torch.uint8), full.k_cache.view(torch.uint8)[:, :, 4:6])
    assert torch.equal(part.v_cache.view(torch.uint8), full.v_cache.view(torch.uint8)[:, :, 4:6])
