"""Seeded synthetic inputs for the five benchmark configurations (and smaller test cases).

All K/V values are N(0,1) bf16 quantised to e4m3 (torch's round-to-nearest-even cast, identical
to the store kernel's for |x| <= 464, which N(0,1) never exceeds); q is N(0,1) bf16; the softmax
scale is 1/sqrt(128).  Physical blocks are a random permutation of the pool (``torch.randperm``
on a seeded generator) and table rows are padded with -1, as ModelRunner.prepare_block_tables
does (nanovllm/engine/model_runner.py:133-142).  Random draws happen on the CPU generator, so a
given seed gives the same inputs on every machine; large tensors are generated on the target
device in chunks.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

HEAD_DIM = 128
SCALE = HEAD_DIM ** -0.5


def _normal_e4m3(shape, gen_seed: int, device) -> torch.Tensor:
    """N(0,1) -> bf16 -> e4m3, generated in chunks directly on ``device``."""
    out = torch.empty(shape, dtype=torch.float8_e4m3fn, device=device)
    flat = out.view(-1)
    g = torch.Generator(device=device).manual_seed(gen_seed)
    chunk = 1 << 26
    for i in range(0, flat.numel(), chunk):
        n = min(chunk, flat.numel() - i)
        x = torch.randn(n, generator=g, device=device, dtype=torch.float32)
        flat[i:i + n] = x.to(torch.bfloat16).to(torch.float8_e4m3fn)
    return out


def _tables(lens, block_size, pool_factor, gen, extra_cols=0):
    nblk = [(max(n, 0) + block_size - 1) // block_size for n in lens]
    total = sum(nblk)
    pool = max(int(math.ceil(total * pool_factor)), total, 1)
    perm = torch.randperm(pool, generator=gen)
    width = max(max(nblk) if nblk else 0, 1) + extra_cols
    rows = torch.full((len(lens), width), -1, dtype=torch.int32)
    k = 0
    for i, nb in enumerate(nblk):
        rows[i, :nb] = perm[k:k + nb].to(torch.int32)
        k += nb
    return rows, pool


@dataclass
class DecodeCase:
    q: torch.Tensor
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    block_tables: torch.Tensor
    context_lens: torch.Tensor
    scale: float = SCALE
    meta: dict = field(default_factory=dict)

    def kv_bytes(self) -> int:
        """Algorithmic bytes of one decode call: every visible K and V byte once, plus q, out,
        the block tables and the lengths."""
        kvh = self.k_cache.shape[2]
        ctx = int(self.context_lens.clamp(min=0).sum())
        b, hq, d = self.q.shape
        return ctx * kvh * d * 2 + 2 * b * hq * d * 2 + 4 * self.block_tables.numel() + 4 * b


def decode_case(batch, num_heads, num_kv_heads, ctx_lo, ctx_hi, seed, device="cpu",
                block_size=256, pool_factor=1.0, lens=None, extra_cols=0) -> DecodeCase:
    gen = torch.Generator().manual_seed(seed)
    if lens is None:
        lens = torch.randint(ctx_lo, ctx_hi + 1, (batch,), generator=gen).tolist()
    tables, pool = _tables(lens, block_size, pool_factor, gen, extra_cols)
    q = torch.randn(batch, num_heads, HEAD_DIM, generator=gen).to(torch.bfloat16)
    shape = (pool, block_size, num_kv_heads, HEAD_DIM)
    kc = _normal_e4m3(shape, seed * 7 + 1, device)
    vc = _normal_e4m3(shape, seed * 7 + 2, device)
    return DecodeCase(q.to(device), kc, vc, tables.to(device),
                      torch.tensor(lens, dtype=torch.int32).to(device),
                      meta=dict(batch=batch, num_heads=num_heads, num_kv_heads=num_kv_heads,
                                block_size=block_size, pool_blocks=pool, seed=seed))


# BASELINE.json configs (decode geometry)
def config1(device="cpu"):
    """CPU-runnable reference case: Qwen3-0.6B heads, 8 sequences, ctx U[64, 1024]."""
    return decode_case(8, 16, 8, 64, 1024, seed=0, device=device)


def config2(device="cpu"):
    """Large-batch decode: Qwen3-8B heads, 256 sequences, ctx U[512, 4096], pool 1.25x."""
    return decode_case(256, 32, 8, 512, 4096, seed=1, device=device, pool_factor=1.25)


def _normal_e4m3_heads(pool, block_size, kv_heads, seed, device) -> torch.Tensor:
    """Paged cache [pool, block_size, len(kv_heads), 128] whose head slice i holds the N(0,1)
    e4m3 values of global kv head kv_heads[i], drawn from its own seeded generator: a rank's
    shard of the cache is then the same bytes as the matching slice of the unsharded cache."""
    out = torch.empty((pool, block_size, len(kv_heads), HEAD_DIM), dtype=torch.float8_e4m3fn,
                      device=device)
    for i, h in enumerate(kv_heads):
        out[:, :, i].copy_(_normal_e4m3((pool, block_size, HEAD_DIM), seed * 1000 + h, device))
    return out


def sharded_decode_case(batch, num_heads, num_kv_heads, lens, seed, device="cpu", gpus=1, rank=0,
                        block_size=256, pool_factor=1.0) -> DecodeCase:
    """Rank ``rank`` of ``gpus``'s part of one decode batch split by kv-head group (the reference's
    tensor-parallel head split, nanovllm/engine/model_runner.py:111, nanovllm/models/qwen3.py:53-59):
    kv heads [r*KVH/g, (r+1)*KVH/g) and their q heads.  Lengths and block tables are the same on
    every rank; q and the caches are the matching slices of the unsharded batch (every kv head's
    bytes come from its own generator), so the ranks' outputs concatenated along the head axis are
    the unsharded problem's."""
    from .shard import kv_head_range, q_head_range
    gen = torch.Generator().manual_seed(seed)
    tables, pool = _tables(lens, block_size, pool_factor, gen)
    q = torch.randn(batch, num_heads, HEAD_DIM, generator=gen).to(torch.bfloat16)
    k0, k1 = kv_head_range(num_kv_heads, rank, gpus)
    h0, h1 = q_head_range(num_heads, num_kv_heads, rank, gpus)
    heads = list(range(k0, k1))
    kc = _normal_e4m3_heads(pool, block_size, heads, seed * 7 + 1, device)
    vc = _normal_e4m3_heads(pool, block_size, heads, seed * 7 + 2, device)
    return DecodeCase(q[:, h0:h1].contiguous().to(device), kc, vc, tables.to(device),
                      torch.tensor(lens, dtype=torch.int32).to(device),
                      meta=dict(batch=batch, num_heads=h1 - h0, num_kv_heads=k1 - k0,
                                block_size=block_size, pool_blocks=pool, seed=seed, gpus=gpus,
                                rank=rank, kv_heads=(k0, k1), q_heads=(h0, h1)))


def config5(device="cpu", gpus=1, rank=0, batch=64):
    """Long-context decode, Qwen3-32B heads (64 q / 8 kv), 64 sequences at 32768 (128 blocks of
    256 each), KV heads split across ``gpus`` ranks: rank r holds kv heads [r*8/g, (r+1)*8/g) and
    their q heads.  A smaller ``batch`` gives the same geometry over fewer sequences (tests and
    profile captures), with a pool of just their blocks."""
    return sharded_decode_case(batch, 64, 8, [32768] * batch, seed=4, device=device, gpus=gpus,
                               rank=rank)


@dataclass
class PrefillCase:
    q: torch.Tensor
    k: torch.Tensor            # paged cache (prefix + new rows stored) or contiguous rows
    v: torch.Tensor
    block_tables: torch.Tensor | None
    cu_seqlens_q: torch.Tensor
    cu_seqlens_k: torch.Tensor
    max_seqlen_q: int
    max_seqlen_k: int
    scale: float = SCALE
    new_k: torch.Tensor | None = None   # bf16 rows stored through slot_mapping before attention
    new_v: torch.Tensor | None = None
    slot_mapping: torch.Tensor | None = None
    meta: dict = field(default_factory=dict)

    def causal_flops(self) -> int:
        """4 * D * Hq * sum over query rows of the keys they attend (causal-useful only)."""
        hq = self.q.shape[1]
        tot = 0
        cq = self.cu_seqlens_q.tolist()
        ck = self.cu_seqlens_k.tolist()
        for s in range(len(cq) - 1):
            nq, nk = cq[s + 1] - cq[s], ck[s + 1] - ck[s]
            p = nk - nq
            tot += sum(max(0, min(nk, p + i + 1)) for i in range(nq))
        return 4 * HEAD_DIM * hq * tot


def prefill_case(nqs, prefixes, num_heads, num_kv_heads, seed, device="cpu", block_size=256,
                 paged=True, pool_factor=1.0) -> PrefillCase:
    """Chunked prefill: sequence s has ``prefixes[s]`` cached key positions and ``nqs[s]`` new
    rows.  Paged: the cache holds the prefix; the new rows' K/V come as bf16 with a slot mapping
    (the caller stores them, as Attention.forward does).  Contiguous: K/V rows are e4m3 tensors
    holding prefix + new rows per sequence."""
    gen = torch.Generator().manual_seed(seed)
    nks = [p + n for p, n in zip(prefixes, nqs)]
    tq = sum(nqs)
    q = torch.randn(tq, num_heads, HEAD_DIM, generator=gen).to(torch.bfloat16)
    cu_q = torch.tensor([0] + list(torch.tensor(nqs).cumsum(0).tolist()), dtype=torch.int32)
    cu_k = torch.tensor([0] + list(torch.tensor(nks).cumsum(0).tolist()), dtype=torch.int32)
    case = dict(q=q.to(device), cu_seqlens_q=cu_q.to(device), cu_seqlens_k=cu_k.to(device),
                max_seqlen_q=max(nqs), max_seqlen_k=max(nks))
    if paged:
        tables, pool = _tables(nks, block_size, pool_factor, gen)
        shape = (pool, block_size, num_kv_heads, HEAD_DIM)
        kc = _normal_e4m3(shape, seed * 7 + 1, device)
        vc = _normal_e4m3(shape, seed * 7 + 2, device)
        new_k = torch.randn(tq, num_kv_heads, HEAD_DIM, generator=gen).to(torch.bfloat16)
        new_v = torch.randn(tq, num_kv_heads, HEAD_DIM, generator=gen).to(torch.bfloat16)
        slots = []
        for s, (p, n) in enumerate(zip(prefixes, nqs)):
            for j in range(p, p + n):
                slots.append(int(tables[s, j // block_size]) * block_size + j % block_size)
        case.update(k=kc, v=vc, block_tables=tables.to(device), new_k=new_k.to(device),
                    new_v=new_v.to(device),
                    slot_mapping=torch.tensor(slots, dtype=torch.int32).to(device))
    else:
        tk = sum(nks)
        kk = _normal_e4m3((tk, num_kv_heads, HEAD_DIM), seed * 7 + 1, device)
        vv = _normal_e4m3((tk, num_kv_heads, HEAD_DIM), seed * 7 + 2, device)
        case.update(k=kk, v=vv, block_tables=None)
    return PrefillCase(**case, meta=dict(nqs=list(nqs), prefixes=list(prefixes),
                                         num_heads=num_heads, num_kv_heads=num_kv_heads,
                                         block_size=block_size, seed=seed))


def config3(device="cpu"):
    """Chunked prefill: Qwen3-8B heads, 16 sequences, new chunks U[128, 512], cached prefixes
    U[0, 3584]."""
    gen = torch.Generator().manual_seed(2)
    nqs = torch.randint(128, 513, (16,), generator=gen).tolist()
    pre = torch.randint(0, 3585, (16,), generator=gen).tolist()
    return prefill_case(nqs, pre, 32, 8, seed=2, device=device)


def config4(device="cpu"):
    """Mixed batch: 192 spec-verify sequences (1 + 4 rows, cached context U[1024, 8187]) plus two
    fresh 512-token prefill chunks, all through one prefill call (split_pt = 0)."""
    gen = torch.Generator().manual_seed(3)
    ctx = torch.randint(1024, 8188, (192,), generator=gen).tolist()
    nqs = [5] * 192 + [512, 512]
    pre = ctx + [0, 0]
    return prefill_case(nqs, pre, 32, 8, seed=3, device=device)
