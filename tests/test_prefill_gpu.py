"""Prefill entry point parity: reference golden outputs (paged and contiguous layouts, long and
speculative-verify sized query sequences), the fp32 oracle on benchmark configs 3 and 4 at full
size, and edge cases (query tiles straddling 128 rows, nk < nq, empty sequences, block sizes
16..512, GQA 1..8, NaN bytes outside the context, scaled caches)."""
import pytest
import torch

from helpers import assert_close, bf16, fp8
from oracle import attention as oatt

pytestmark = pytest.mark.gpu


def _prefill(q, k, v, bt, cq, ck, mq, mk, scale, **kw):
    from nanovllm_b200 import fp8_prefill_attention
    out = fp8_prefill_attention(q, k, v, block_tables=bt, cu_seqlens_q=cq, cu_seqlens_k=ck,
                                max_seqlen_q=mq, max_seqlen_k=mk, softmax_scale=scale, **kw)
    torch.cuda.synchronize()
    return out


def _no_device_error():
    from nanovllm_b200.fp8_attention import device_error
    assert device_error() == 0


def _oracle(c, rows=None, **kw):
    return oatt.prefill(c.q.cpu(), c.k.cpu(), c.v.cpu(),
                        None if c.block_tables is None else c.block_tables.cpu(),
                        c.cu_seqlens_q.cpu(), c.cu_seqlens_k.cpu(), c.scale, **kw)


@pytest.mark.parametrize("name", ["prefill_paged", "prefill_paged_small", "prefill_paged_bs256",
                                  "prefill_contig"])
def test_prefill_matches_reference_golden(golden, name):
    g = golden(name)
    cq, ck = torch.from_numpy(g["cu_seqlens_q"]), torch.from_numpy(g["cu_seqlens_k"])
    bt = torch.from_numpy(g["block_tables"]).cuda() if "block_tables" in g else None
    nq = (cq[1:] - cq[:-1]).max().item()
    nk = (ck[1:] - ck[:-1]).max().item()
    out = _prefill(bf16(g["q"]).cuda(), fp8(g["k"]).cuda(), fp8(g["v"]).cuda(), bt, cq.cuda(),
                   ck.cuda(), nq, nk, float(g["scale"]))
    assert_close(out, bf16(g["out"]), what=name)
    _no_device_error()


def _store_new_rows(c):
    from nanovllm_b200 import store_kvcache
    store_kvcache(c.new_k, c.new_v, c.k, c.v, c.slot_mapping)
    torch.cuda.synchronize()


def test_prefill_config3_full_size():
    from nanovllm_b200 import workloads
    c = workloads.config3("cuda")
    _store_new_rows(c)
    out = _prefill(c.q, c.k, c.v, c.block_tables, c.cu_seqlens_q, c.cu_seqlens_k, c.max_seqlen_q,
                   c.max_seqlen_k, c.scale)
    assert_close(out, _oracle(c), what="config3")
    _no_device_error()


def test_prefill_config4_mixed_spec_and_fresh():
    from nanovllm_b200 import workloads
    c = workloads.config4("cuda")
    _store_new_rows(c)
    out = _prefill(c.q, c.k, c.v, c.block_tables, c.cu_seqlens_q, c.cu_seqlens_k, c.max_seqlen_q,
                   c.max_seqlen_k, c.scale)
    # the oracle on a sample: 24 spec-verify sequences and both fresh 512-token chunks
    cq = c.cu_seqlens_q.cpu()
    pick = list(range(0, 192, 8)) + [192, 193]
    rows = torch.cat([torch.arange(int(cq[s]), int(cq[s + 1])) for s in pick])
    from nanovllm_b200.workloads import PrefillCase
    ck = c.cu_seqlens_k.cpu()
    nqs = [int(cq[s + 1] - cq[s]) for s in pick]
    nks = [int(ck[s + 1] - ck[s]) for s in pick]
    sub = PrefillCase(q=c.q[rows.cuda()], k=c.k, v=c.v, block_tables=c.block_tables[pick],
                      cu_seqlens_q=torch.tensor([0] + torch.tensor(nqs).cumsum(0).tolist(), dtype=torch.int32),
                      cu_seqlens_k=torch.tensor([0] + torch.tensor(nks).cumsum(0).tolist(), dtype=torch.int32),
                      max_seqlen_q=max(nqs), max_seqlen_k=max(nks))
    assert_close(out[rows.cuda()], _oracle(sub), what="config4 sample")
    _no_device_error()


def test_prefill_long_context_with_score_spikes():
    """Long cached contexts where chosen query rows meet a matching key late in the context: their
    scores jump far above everything before (a reference move well after the first tiles, several
    times per row, in both column halves of a row), against the fp32 oracle."""
    from nanovllm_b200 import workloads
    nqs, pre, bs = [300, 700, 129], [12000, 5000, 0], 256
    c = workloads.prefill_case(nqs, pre, 8, 2, seed=11, device="cuda", block_size=bs,
                               pool_factor=1.1)
    _store_new_rows(c)
    bt = c.block_tables.cpu()
    cq = c.cu_seqlens_q.cpu()
    g = 8 // 2
    plants = [(0, 299, 1, [700, 6000, 9000, 11500], [0.5, 1.0, 1.5, 2.0]),   # last row, head 1
              (0, 150, 4, [3000, 11999], [1.0, 3.0]),                         # mid row, head 4
              (1, 699, 6, [100, 2500, 4999], [0.7, 1.4, 2.5])]                # seq 1, head 6
    for s, row, h, positions, gains in plants:
        qrow = c.q[int(cq[s]) + row, h].float()
        for pos, gain in zip(positions, gains):
            blk, off = int(bt[s, pos // bs]), pos % bs
            c.k[blk, off, h // g] = (gain * qrow).to(torch.float8_e4m3fn)
    out = _prefill(c.q, c.k, c.v, c.block_tables, c.cu_seqlens_q, c.cu_seqlens_k, c.max_seqlen_q,
                   c.max_seqlen_k, c.scale)
    assert_close(out, _oracle(c), what="long context with score spikes")
    _no_device_error()


def test_prefill_many_spec_verify_sequences():
    """700 sequences, mostly speculative-verify sized (1..5 query rows, served by the decode
    engine in spec mode) with some longer chunks among them (served by the prefill kernel): the
    spec-mode plan then spans several sequences per range, some of them not routed to it."""
    from nanovllm_b200 import workloads
    gen = torch.Generator().manual_seed(45)
    nqs = torch.randint(1, 6, (700,), generator=gen)
    nqs[torch.randint(0, 700, (12,), generator=gen)] = 40
    nqs[[3, 350, 699]] = 200
    pre = torch.randint(0, 401, (700,), generator=gen)
    pre[torch.randint(0, 700, (60,), generator=gen)] = 0
    c = workloads.prefill_case(nqs.tolist(), pre.tolist(), 32, 8, seed=45, device="cuda",
                               block_size=128)
    _store_new_rows(c)
    out = _prefill(c.q, c.k, c.v, c.block_tables, c.cu_seqlens_q, c.cu_seqlens_k, c.max_seqlen_q,
                   c.max_seqlen_k, c.scale)
    assert_close(out, _oracle(c), what="700 spec-verify sequences")
    _no_device_error()


@pytest.mark.parametrize("nseq,max_nq", [(700, 2), (2048, 5)])
def test_prefill_spec_verify_large_batches(nseq, max_nq):
    """Spec-verify batches whose decode-engine plan is sampled: 700 sequences of up to 2 query
    rows (GQA 4: the 8-row engine, ranges of 3 sequences) and 2048 of up to 5 (the 24-row
    engine, ranges of 8), with empty query sequences and empty prefixes among them."""
    from nanovllm_b200 import workloads
    gen = torch.Generator().manual_seed(46 + nseq)
    nqs = torch.randint(1, max_nq + 1, (nseq,), generator=gen)
    nqs[torch.randint(0, nseq, (nseq // 10,), generator=gen)] = 0
    pre = torch.randint(0, 201, (nseq,), generator=gen)
    pre[torch.randint(0, nseq, (nseq // 10,), generator=gen)] = 0
    c = workloads.prefill_case(nqs.tolist(), pre.tolist(), 32, 8, seed=46, device="cuda",
                               block_size=64)
    _store_new_rows(c)
    out = _prefill(c.q, c.k, c.v, c.block_tables, c.cu_seqlens_q, c.cu_seqlens_k, c.max_seqlen_q,
                   c.max_seqlen_k, c.scale)
    assert_close(out, _oracle(c), what=f"{nseq} spec-verify sequences")
    _no_device_error()


@pytest.mark.parametrize("bs", [16, 32, 64, 256, 512])
@pytest.mark.parametrize("hq,kvh", [(4, 4), (8, 2), (16, 2), (12, 4), (24, 4)])  # + GQA 3, 6
def test_prefill_paged_edge_cases(bs, hq, kvh):
    from nanovllm_b200 import workloads
    nqs = [127, 128, 129, 1, 300, 0, 40, 9]
    pre = [0, 3, 200, 77, 1000, 5, 0, 130]
    c = workloads.prefill_case(nqs, pre, hq, kvh, seed=bs + hq, device="cuda", block_size=bs,
                               pool_factor=1.2)
    _store_new_rows(c)
    out = _prefill(c.q, c.k, c.v, c.block_tables, c.cu_seqlens_q, c.cu_seqlens_k, c.max_seqlen_q,
                   c.max_seqlen_k, c.scale)
    assert_close(out, _oracle(c), what=f"paged bs{bs} hq{hq} kvh{kvh}")
    _no_device_error()


@pytest.mark.parametrize("hq,kvh", [(4, 4), (8, 1)])
def test_prefill_contiguous_edge_cases(hq, kvh):
    from nanovllm_b200 import workloads
    nqs = [130, 1, 64, 257, 3]
    pre = [0, 10, 100, 0, 2]
    c = workloads.prefill_case(nqs, pre, hq, kvh, seed=7 + hq, device="cuda", paged=False)
    out = _prefill(c.q, c.k, c.v, None, c.cu_seqlens_q, c.cu_seqlens_k, c.max_seqlen_q,
                   c.max_seqlen_k, c.scale)
    assert_close(out, _oracle(c), what=f"contig hq{hq} kvh{kvh}")
    _no_device_error()


def test_prefill_rows_without_keys_and_nan_padding():
    # nk < nq: the first rows see no key and give 0 (reference :311); cache bytes outside every
    # sequence are NaN codes that must not leak
    from nanovllm_b200 import workloads
    from nanovllm_b200.workloads import PrefillCase
    c = workloads.prefill_case([200, 150], [60, 0], 8, 2, seed=21, device="cuda", block_size=64,
                               pool_factor=1.0)
    _store_new_rows(c)
    kc, vc = c.k.view(torch.uint8), c.v.view(torch.uint8)
    ck = c.cu_seqlens_k.cpu()
    for s in range(2):
        n = int(ck[s + 1] - ck[s])
        for j in range(n, ((n + 63) // 64) * 64):
            blk = int(c.block_tables[s, j // 64])
            kc[blk, j % 64] = 0x7F
            vc[blk, j % 64] = 0x7F
    # shrink sequence 1's keys below its queries: rows 0..39 then see nothing
    ck2 = ck.clone()
    ck2[2] = ck2[1] + 110
    c2 = PrefillCase(q=c.q, k=c.k, v=c.v, block_tables=c.block_tables, cu_seqlens_q=c.cu_seqlens_q,
                     cu_seqlens_k=ck2.cuda(), max_seqlen_q=200, max_seqlen_k=260)
    out = _prefill(c2.q, c2.k, c2.v, c2.block_tables, c2.cu_seqlens_q, c2.cu_seqlens_k, 200, 260,
                   c2.scale)
    assert torch.isfinite(out.float()).all()
    ref = _oracle(c2)
    assert_close(out, ref, what="nk<nq + nan padding")
    assert torch.all(out[200:240] == 0)
    _no_device_error()


def test_prefill_scaled_cache():
    from nanovllm_b200 import workloads
    c = workloads.prefill_case([150, 20, 4], [100, 300, 50], 8, 2, seed=31, device="cuda",
                               block_size=128)
    nb, bs, kvh, _ = c.k.shape
    gen = torch.Generator().manual_seed(8)
    ks = (torch.rand(nb, bs, kvh, generator=gen) * 0.05 + 0.001).cuda()
    vs = (torch.rand(nb, bs, kvh, generator=gen) * 0.05 + 0.001).cuda()
    out = _prefill(c.q, c.k, c.v, c.block_tables, c.cu_seqlens_q, c.cu_seqlens_k, c.max_seqlen_q,
                   c.max_seqlen_k, c.scale, k_scale=ks, v_scale=vs)
    assert_close(out, _oracle(c, k_scale=ks.cpu(), v_scale=vs.cpu()), what="prefill scaled")
    _no_device_error()


def test_prefill_mixed_batch_cuda_graph_replay():
    """A mixed call (speculative-verify rows and chunked-prefill chunks in one paged prefill)
    captured once in a CUDA graph and replayed on other batches of the same sequence count and
    token count: the launches depend on neither the lengths nor max_seqlen_q beyond the cap the
    caller passes (the prefill grid follows the sequence count and the cap, and its CTAs find
    their work on the device; the split-KV engine's width follows min(cap, spec limit)), so one
    graph serves every such batch."""
    from nanovllm_b200 import fp8_prefill_attention, store_kvcache, workloads
    cap = 512
    batches = [([5, 5, 300, 5, 200, 5], [900, 1700, 0, 2500, 300, 3000]),
               ([5, 310, 5, 5, 5, 190], [2100, 600, 4000, 10, 700, 0]),
               ([260, 5, 5, 250, 0, 0], [0, 300, 800, 1200, 50, 0])]
    cases = [workloads.prefill_case(nqs, pre, 32, 8, seed=61 + i, device="cuda", block_size=256,
                                    pool_factor=1.2) for i, (nqs, pre) in enumerate(batches)]
    width = max(c.block_tables.shape[1] for c in cases)
    pool = max(c.k.shape[0] for c in cases)
    static = {}
    for c in cases:  # same cache pool, table width and buffers for every batch
        bt = torch.full((6, width), -1, dtype=torch.int32, device="cuda")
        bt[:, :c.block_tables.shape[1]] = c.block_tables
        c.block_tables = bt
        k = torch.zeros(pool, 256, 8, 128, dtype=torch.uint8, device="cuda").view(torch.float8_e4m3fn)
        v = torch.zeros_like(k)
        k[:c.k.shape[0]] = c.k
        v[:c.v.shape[0]] = c.v
        c.k, c.v = k, v
        store_kvcache(c.new_k, c.new_v, c.k, c.v, c.slot_mapping)
    assert len({c.q.shape[0] for c in cases}) == 1
    for name in ("q", "k", "v", "block_tables", "cu_seqlens_q", "cu_seqlens_k"):
        static[name] = getattr(cases[0], name).clone()

    def call():
        return fp8_prefill_attention(static["q"], static["k"], static["v"],
                                     block_tables=static["block_tables"],
                                     cu_seqlens_q=static["cu_seqlens_q"],
                                     cu_seqlens_k=static["cu_seqlens_k"], max_seqlen_q=cap,
                                     max_seqlen_k=8192, softmax_scale=cases[0].scale)

    call()  # the workspace of this shape exists before capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = call()
    for c in cases:
        for name in static:
            static[name].copy_(getattr(c, name))
        graph.replay()
        torch.cuda.synchronize()
        assert_close(out, _oracle(c), what="mixed batch, graph replay")
    _no_device_error()
