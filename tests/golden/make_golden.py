"""Generate the golden fixtures in this directory from the reference's own kernels.

Run in a container that has the reference checkout (it is NOT needed at test time):

    TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/reference

It imports ``store_kvcache`` (nanovllm/layers/attention.py:33-40), ``fp8_decode_attention``
(nanovllm/kernels/fp8_attention.py:173-207) and ``fp8_prefill_attention``
(nanovllm/kernels/fp8_attention.py:314-353) from the reference and runs them with Triton's CPU
interpreter on seeded inputs, then writes one ``.npz`` per case.

Notes on what the interpreter can and cannot pin:
  * Attention outputs: the interpreter widens e4m3 exactly and computes in fp32 (numpy dot in
    place of the GPU's TF32 ``tl.dot``), so its outputs pin the algorithm (masking, block
    indexing, GQA mapping, the fp16 -> bf16 output path).
  * Store: the interpreter's bf16 -> e4m3 store does not round to nearest-even, so store
    fixtures use values that are exactly representable in e4m3; they pin slot placement, the
    ``slot == -1`` skip and strided rows, not rounding.  Rounding is pinned separately against
    torch's cast over all bf16 values.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _bits(t):
    import torch
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _codes(t):
    import torch
    return t.contiguous().view(torch.uint8).numpy()


def _cache_from_normal(gen, nb, bs, kvh, d):
    import torch
    x = torch.randn(nb, bs, kvh, d, generator=gen).to(torch.bfloat16)
    return x.to(torch.float8_e4m3fn)


def _paged_tables(gen, lens, bs, extra_cols, spare_blocks):
    """Random physical block permutation; rows padded with -1 (model_runner.py:133-142)."""
    import torch
    nblk = [(n + bs - 1) // bs for n in lens]
    total = sum(nblk) + spare_blocks
    perm = torch.randperm(total, generator=gen).tolist()
    width = max(nblk) + extra_cols
    rows, k = [], 0
    for nbk in nblk:
        rows.append(perm[k:k + nbk] + [-1] * (width - nbk))
        k += nbk
    return torch.tensor(rows, dtype=torch.int32), total


def gen_store(ref, gen):
    import torch
    kvh, d, bs, nb = 2, 128, 16, 8
    hq = 4
    n = 40
    # exactly-representable values: random finite e4m3 codes widened to bf16
    codes = torch.randint(0, 256, (n, hq + 2 * kvh, d), generator=gen, dtype=torch.int32)
    codes = torch.where((codes & 0x7F) == 0x7F, codes - 1, codes).to(torch.uint8)
    qkv = codes.view(torch.float8_e4m3fn).to(torch.bfloat16)     # [n, Hq+2KVH, D]
    key = qkv[:, hq:hq + kvh].contiguous()                        # fresh contiguous tensor
    value = qkv[:, hq + kvh:]                                     # strided view (row stride (Hq+2KVH)*D)
    slots = torch.randperm(nb * bs, generator=gen)[:n].to(torch.int32)
    slots[torch.tensor([3, 11, 12, 39])] = -1
    k_cache = torch.full((nb, bs, kvh, d), 0x55, dtype=torch.uint8).view(torch.float8_e4m3fn)
    v_cache = torch.full((nb, bs, kvh, d), 0x55, dtype=torch.uint8).view(torch.float8_e4m3fn)
    ref.store_kvcache(key, value, k_cache, v_cache, slots)
    return dict(qkv=_bits(qkv), hq=hq, kvh=kvh, slots=slots.numpy(), init=0x55,
                k_cache=_codes(k_cache), v_cache=_codes(v_cache))


def gen_decode(ref, gen, b_lens, hq, kvh, bs, extra_cols=1, spare=3):
    import torch
    d = 128
    tables, nb = _paged_tables(gen, b_lens, bs, extra_cols, spare)
    kc = _cache_from_normal(gen, nb, bs, kvh, d)
    vc = _cache_from_normal(gen, nb, bs, kvh, d)
    q = torch.randn(len(b_lens), hq, d, generator=gen).to(torch.bfloat16)
    ctx = torch.tensor(b_lens, dtype=torch.int32)
    out = ref.fp8_decode_attention(q, kc, vc, tables, ctx, d ** -0.5)
    return dict(q=_bits(q), k_cache=_codes(kc), v_cache=_codes(vc), block_tables=tables.numpy(),
                context_lens=ctx.numpy(), scale=np.float64(d ** -0.5), out=_bits(out))


def gen_prefill(ref, gen, nqs, nks, hq, kvh, bs=None, extra_cols=1, spare=2):
    import torch
    d = 128
    tq = sum(nqs)
    q = torch.randn(tq, hq, d, generator=gen).to(torch.bfloat16)
    cu_q = torch.tensor(np.concatenate([[0], np.cumsum(nqs)]), dtype=torch.int32)
    cu_k = torch.tensor(np.concatenate([[0], np.cumsum(nks)]), dtype=torch.int32)
    if bs is None:
        tk = sum(nks)
        k = _cache_from_normal(gen, tk, 1, kvh, d).reshape(tk, kvh, d)
        v = _cache_from_normal(gen, tk, 1, kvh, d).reshape(tk, kvh, d)
        tables = None
    else:
        tables, nb = _paged_tables(gen, nks, bs, extra_cols, spare)
        k = _cache_from_normal(gen, nb, bs, kvh, d)
        v = _cache_from_normal(gen, nb, bs, kvh, d)
    out = ref.fp8_prefill_attention(q, k, v, block_tables=tables, cu_seqlens_q=cu_q,
                                    cu_seqlens_k=cu_k, max_seqlen_q=max(nqs),
                                    max_seqlen_k=max(nks), softmax_scale=d ** -0.5)
    res = dict(q=_bits(q), k=_codes(k), v=_codes(v), cu_seqlens_q=cu_q.numpy(),
               cu_seqlens_k=cu_k.numpy(), scale=np.float64(d ** -0.5), out=_bits(out))
    if tables is not None:
        res["block_tables"] = tables.numpy()
    return res


def main(ref_root: str):
    assert os.environ.get("TRITON_INTERPRET") == "1", "run with TRITON_INTERPRET=1"
    sys.path.insert(0, ref_root)
    import torch
    from nanovllm.layers import attention as ref_attn
    from nanovllm.kernels import fp8_attention as ref_k

    class Ref:
        store_kvcache = staticmethod(ref_attn.store_kvcache)
        fp8_decode_attention = staticmethod(ref_k.fp8_decode_attention)
        fp8_prefill_attention = staticmethod(ref_k.fp8_prefill_attention)

    cases = {
        "store_placement": lambda g: gen_store(Ref, g),
        # decode: block size 32 with ragged lengths, a zero-length row and -1 padding
        "decode_bs32": lambda g: gen_decode(Ref, g, [1, 31, 32, 33, 150, 0], 8, 2, 32),
        # decode: the engine's block size 256, GQA 4:1, lengths straddling blocks
        "decode_bs256": lambda g: gen_decode(Ref, g, [256, 257, 700], 4, 1, 256),
        # decode: block size 16, GQA 8:1 (the 32B geometry's ratio)
        "decode_bs16_g8": lambda g: gen_decode(Ref, g, [5, 16, 17, 90], 8, 1, 16),
        # paged prefill (chunked: cached prefix + new rows), BLOCK_M = 32 path
        "prefill_paged": lambda g: gen_prefill(Ref, g, [1, 17, 40], [1, 22, 110], 4, 2, bs=32),
        # paged prefill with <= 16 query rows (BLOCK_M = 16 path), spec-verify-like shapes
        "prefill_paged_small": lambda g: gen_prefill(Ref, g, [5, 5, 3, 1], [300, 64, 5, 40], 4, 1,
                                                     bs=32),
        # paged prefill at block size 256 with a zero-length query sequence in the middle
        "prefill_paged_bs256": lambda g: gen_prefill(Ref, g, [70, 0, 33], [330, 7, 33], 8, 2,
                                                     bs=256),
        # contiguous layout (block_tables=None): fresh, with a prefix, and nk < nq
        "prefill_contig": lambda g: gen_prefill(Ref, g, [5, 20, 33, 4], [5, 23, 33, 2], 4, 2),
    }
    for i, (name, fn) in enumerate(cases.items()):
        gen = torch.Generator().manual_seed(1000 + i)
        data = fn(gen)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **data)
        print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
