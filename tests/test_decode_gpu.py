"""Decode engine parity: reference golden outputs, the fp32 oracle on the benchmark configs and on
edge cases (ragged lengths, zero lengths, -1 padding, block sizes 16..512, GQA 1..16, split-KV
chunking, a 128k-token sequence), scaled caches, and CUDA-graph capture."""
import pytest
import torch

from helpers import ATOL, RTOL, assert_close, bf16, fp8
from oracle import attention as oatt

pytestmark = pytest.mark.gpu


def _lib():
    from nanovllm_b200 import _lib
    return _lib.lib


def _decode(case_or_args, **kw):
    from nanovllm_b200 import fp8_decode_attention
    out = fp8_decode_attention(*case_or_args, **kw)
    torch.cuda.synchronize()
    return out


def _no_device_error():
    from nanovllm_b200.fp8_attention import device_error
    assert device_error() == 0


@pytest.mark.parametrize("name", ["decode_bs32", "decode_bs256", "decode_bs16_g8"])
def test_decode_matches_reference_golden(golden, name):
    g = golden(name)
    args = (bf16(g["q"]).cuda(), fp8(g["k_cache"]).cuda(), fp8(g["v_cache"]).cuda(),
            torch.from_numpy(g["block_tables"]).cuda(), torch.from_numpy(g["context_lens"]).cuda(),
            float(g["scale"]))
    out = _decode(args)
    assert_close(out, bf16(g["out"]), what=name)
    _no_device_error()


def _oracle_case(c, **kw):
    return oatt.decode(c.q.cpu(), c.k_cache.cpu(), c.v_cache.cpu(), c.block_tables.cpu(),
                       c.context_lens.cpu(), c.scale, **kw)


def test_decode_config1():
    from nanovllm_b200 import workloads
    c = workloads.config1("cuda")
    out = _decode((c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale))
    assert_close(out, _oracle_case(c), what="config1")
    _no_device_error()


@pytest.mark.parametrize("min_chunk", [128, 512])
@pytest.mark.parametrize("bs,hq,kvh", [(16, 4, 4), (32, 8, 2), (64, 16, 1), (256, 32, 8),
                                       (48, 8, 8), (80, 32, 2), (256, 64, 8),
                                       (64, 12, 4), (128, 48, 8),  # GQA 3 and 6
                                       (512, 32, 8)])
def test_decode_edge_cases(bs, hq, kvh, min_chunk):
    from nanovllm_b200 import workloads
    lens = [0, 1, bs - 1, bs, bs + 1, 63, 64, 65, 3 * bs + 17, 700, -5, 1000]
    c = workloads.decode_case(len(lens), hq, kvh, 0, 0, seed=bs + hq, device="cuda",
                              block_size=bs, pool_factor=1.3, lens=lens, extra_cols=2)
    prev = _lib().fp8attn_set_decode_min_chunk(min_chunk)
    try:
        out = _decode((c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale))
    finally:
        _lib().fp8attn_set_decode_min_chunk(prev)
    ref = _oracle_case(c)
    assert_close(out, ref, what=f"bs{bs} hq{hq} kvh{kvh}")
    assert torch.all(out[0] == 0) and torch.all(out[10] == 0)   # empty contexts give zeros
    _no_device_error()


@pytest.mark.parametrize("min_chunk", [128, 32768])
def test_decode_score_spikes(min_chunk):
    """Keys planted to match chosen query heads late in long contexts: their scores jump far
    above everything before (the reference moves inside an item, or between the chunks the
    combine merges), against the fp32 oracle."""
    from nanovllm_b200 import workloads
    lens = [20000, 9000, 4000, 300, 16000, 2500]
    c = workloads.decode_case(len(lens), 32, 8, 0, 0, seed=21, device="cuda", block_size=256,
                              pool_factor=1.1, lens=lens)
    bt = c.block_tables.cpu()
    g = 32 // 8
    plants = [(0, 5, [100, 9000, 19999], [0.6, 1.2, 2.5]), (1, 31, [8999], [3.0]),
              (2, 0, [10, 3000], [1.0, 2.0]), (4, 17, [2000, 8000, 15000], [0.8, 1.6, 2.4])]
    for b, h, positions, gains in plants:
        qrow = c.q[b, h].float()
        for pos, gain in zip(positions, gains):
            c.k_cache[int(bt[b, pos // 256]), pos % 256, h // g] = (gain * qrow).to(torch.float8_e4m3fn)
    prev = _lib().fp8attn_set_decode_min_chunk(min_chunk)
    try:
        out = _decode((c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale))
    finally:
        _lib().fp8attn_set_decode_min_chunk(prev)
    assert_close(out, _oracle_case(c), what=f"score spikes, min chunk {min_chunk}")
    _no_device_error()


def test_decode_single_long_sequence_many_chunks():
    """A 128k-token sequence next to a short one: each of its (sequence, kv head) pairs splits
    into hundreds of chunks, the producer refreshes its block-table window many times, and the
    combine merges the chunks over more than one round of its staged weights."""
    from nanovllm_b200 import workloads
    c = workloads.decode_case(2, 32, 8, 0, 0, seed=33, device="cuda", block_size=256,
                              lens=[131072, 37])
    out = _decode((c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale))
    assert_close(out, _oracle_case(c), what="128k-token sequence")
    _no_device_error()


@pytest.mark.parametrize("bs,hq,kvh", [(2048, 32, 8), (601, 64, 8)])
def test_decode_large_batches(bs, hq, kvh):
    """Batches past 511 sequences run the sampled plan (ranges of ceil(B / 256) sequences):
    2048 sequences (the most one call takes; ranges of 8, the last one without any work) and 601
    (ranges of 3, the last one partial); lengths 0..300 with zeros and negatives among them."""
    from nanovllm_b200 import workloads
    gen = torch.Generator().manual_seed(44 + bs)
    lens = torch.randint(0, 301, (bs,), generator=gen)
    lens[torch.randint(0, bs, (bs // 7,), generator=gen)] = 0
    lens[torch.randint(0, bs, (20,), generator=gen)] = -3
    lens[-8:] = 0
    c = workloads.decode_case(bs, hq, kvh, 0, 0, seed=44, device="cuda", block_size=64,
                              lens=lens.tolist(), extra_cols=1)
    out = _decode((c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale))
    assert_close(out, _oracle_case(c), what=f"{bs} sequences")
    assert torch.all(out[lens.cuda() <= 0] == 0)
    _no_device_error()


def test_decode_ctas_per_sm_at_every_batch_size():
    """The persistent grid keeps its CTAs on every SM from 1 to 2048 sequences, for each engine
    variant: two per SM for the single-plane engines (decode GQA 4 and 8) -- the in-kernel plan
    switches to per-range arrays before its shared memory would push the second CTA off -- and
    one per SM for the wide spec-verify engines (4 and 5 query rows of GQA 4: 16 and 20 rows)."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for bs in [1, 256, 511, 512, 1000, 1919, 1920, 2048]:
        for hq, kvh, mq, per_sm in [(32, 8, 1, 2), (64, 8, 1, 2), (32, 8, 4, 1), (32, 8, 5, 1)]:
            assert _lib().fp8attn_decode_ctas(bs, hq, kvh, mq) == per_sm * sms, (bs, hq, kvh, mq)


def test_decode_nan_bytes_beyond_context_are_ignored():
    # slots past each context hold NaN codes (0x7F): they must not leak into the output
    from nanovllm_b200 import workloads
    lens = [5, 70, 300]
    c = workloads.decode_case(3, 8, 2, 0, 0, seed=9, device="cuda", block_size=64,
                              lens=lens, pool_factor=1.0)
    kc = c.k_cache.view(torch.uint8)
    vc = c.v_cache.view(torch.uint8)
    for b, n in enumerate(lens):
        for j in range(n, ((n + 63) // 64) * 64):
            blk = int(c.block_tables[b, j // 64])
            kc[blk, j % 64] = 0x7F
            vc[blk, j % 64] = 0x7F
    out = _decode((c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale))
    assert torch.isfinite(out.float()).all()
    assert_close(out, _oracle_case(c), what="nan-padding")


def test_decode_scaled_cache():
    from nanovllm_b200 import workloads
    c = workloads.decode_case(6, 16, 4, 1, 900, seed=11, device="cuda", block_size=128)
    nb, bs, kvh, _ = c.k_cache.shape
    gen = torch.Generator().manual_seed(5)
    ks = (torch.rand(nb, bs, kvh, generator=gen) * 0.05 + 0.001).cuda()
    vs = (torch.rand(nb, bs, kvh, generator=gen) * 0.05 + 0.001).cuda()
    out = _decode((c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale),
                  k_scale=ks, v_scale=vs)
    ref = _oracle_case(c, k_scale=ks.cpu(), v_scale=vs.cpu())
    assert_close(out, ref, what="scaled")


def test_decode_config2_full_size_sampled():
    # full config-2 launch; the oracle checks a deterministic sample of sequences
    from nanovllm_b200 import workloads
    c = workloads.config2("cuda")
    out = _decode((c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale))
    idx = list(range(0, 256, 17)) + [255]
    sub = workloads.DecodeCase(c.q[idx], c.k_cache, c.v_cache, c.block_tables[idx],
                               c.context_lens[idx])
    assert_close(out[idx], _oracle_case(sub), what="config2 sample")
    _no_device_error()


def test_decode_cuda_graph_replay():
    """Captured once, replayed with new lengths / tables: matches eager (graph capture path of
    ModelRunner.capture_cudagraph, nanovllm/engine/model_runner.py:294-329)."""
    from nanovllm_b200 import fp8_decode_attention, workloads
    c = workloads.decode_case(16, 32, 8, 1, 2000, seed=3, device="cuda", block_size=256,
                              extra_cols=3)
    static_q = c.q.clone()
    static_bt = c.block_tables.clone()
    static_ctx = torch.zeros_like(c.context_lens)
    fp8_decode_attention(static_q, c.k_cache, c.v_cache, static_bt, static_ctx, c.scale)  # warmup
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        static_out = fp8_decode_attention(static_q, c.k_cache, c.v_cache, static_bt, static_ctx,
                                          c.scale)
    for trial in range(3):
        gen = torch.Generator().manual_seed(trial)
        ctx = torch.randint(0, 2000, (16,), generator=gen, dtype=torch.int32)
        ctx[trial] = 0
        static_ctx.copy_(ctx.cuda())
        static_q.copy_(torch.randn(16, 32, 128, generator=gen).to(torch.bfloat16).cuda())
        g.replay()
        torch.cuda.synchronize()
        eager = fp8_decode_attention(static_q, c.k_cache, c.v_cache, static_bt, static_ctx, c.scale)
        torch.cuda.synchronize()
        assert torch.equal(static_out, eager)
    _no_device_error()
