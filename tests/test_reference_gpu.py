"""Parity against the reference's own GPU kernels, run on the same B200 from its unmodified install
under baseline/_ref (the Triton kernels of nanovllm/layers/attention.py:11-40 and
nanovllm/kernels/fp8_attention.py:88-353, through their stock entry points).

* Store: the bytes the reference's store_kvcache_kernel writes for every bf16 bit pattern (finite,
  beyond e4m3's range, +-inf, NaN), through strided value rows and slot -1 rows, must equal ours
  byte for byte; where the input is NaN any NaN code (0x7F / 0xFF) is accepted from either side.
* Decode and prefill (paged, contiguous, and a mixed spec-verify batch): our outputs against the
  reference kernels' outputs within the attention tolerance (the reference's prefill runs its
  fp32 tl.dot as TF32 on the GPU, so it is itself within a few 1e-3 of the fp32 oracle).
"""
import os
import sys

import numpy as np
import pytest
import torch

from helpers import assert_close, bf16

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "nanovllm")):
        pytest.skip("the reference is not installed under baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    from nanovllm.kernels import fp8_attention as rk
    from nanovllm.layers import attention as ra
    return {"store": ra.store_kvcache, "decode": rk.fp8_decode_attention,
            "prefill": rk.fp8_prefill_attention}


def _all_bf16_rows(kvh, shift):
    allbits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    per_row = kvh * 128
    n = (allbits.size + per_row - 1) // per_row
    pad = np.zeros(n * per_row, dtype=np.uint16)
    pad[:allbits.size] = np.roll(allbits, shift)
    return n, pad.reshape(n, kvh, 128)


@pytest.mark.parametrize("kvh", [1, 8])
def test_store_bytes_equal_reference_store_on_every_bf16_pattern(ref, kvh):
    from nanovllm_b200 import store_kvcache
    n, kbits = _all_bf16_rows(kvh, 0)
    _, vbits = _all_bf16_rows(kvh, 12345)
    hq = 2 * kvh
    qkv = torch.zeros(n, hq + 2 * kvh, 128, dtype=torch.bfloat16)
    qkv[:, hq:hq + kvh] = bf16(kbits)
    qkv[:, hq + kvh:] = bf16(vbits)
    qkv = qkv.cuda()
    key = qkv[:, hq:hq + kvh].contiguous()
    value = qkv[:, hq + kvh:]                     # strided rows, as the engine passes them
    bs = 16
    nb = (n + bs - 1) // bs + 2
    gen = torch.Generator().manual_seed(kvh)
    slots = torch.randperm(nb * bs, generator=gen)[:n].to(torch.int32)
    slots[::11] = -1
    slots = slots.cuda()
    caches = []
    for fn in (ref["store"], store_kvcache):
        kc = torch.full((nb, bs, kvh, 128), 0x55, dtype=torch.uint8, device="cuda")
        vc = torch.full((nb, bs, kvh, 128), 0x55, dtype=torch.uint8, device="cuda")
        fn(key, value, kc.view(torch.float8_e4m3fn), vc.view(torch.float8_e4m3fn), slots)
        torch.cuda.synchronize()
        caches.append((kc.cpu().numpy(), vc.cpu().numpy()))
    for (a, b), src in zip(zip(caches[0], caches[1]), (kbits, vbits)):
        # NaN inputs (exponent all ones, mantissa non-zero) may come out as either NaN code
        nan_in = np.zeros_like(a, dtype=bool)
        s = slots.cpu().numpy()
        flat_a = a.reshape(-1, kvh, 128)
        isnan = ((src & 0x7F80) == 0x7F80) & ((src & 0x7F) != 0)
        nan_in.reshape(-1, kvh, 128)[s[s >= 0]] = isnan[s >= 0]
        same = a == b
        both_nan = ((a & 0x7F) == 0x7F) & ((b & 0x7F) == 0x7F)
        bad = ~same & ~(nan_in & both_nan)
        assert not bad.any(), (int(bad.sum()), flat_a.reshape(-1)[np.flatnonzero(bad)[:8]],
                               b.reshape(-1)[np.flatnonzero(bad)[:8]])
        # |x| >= 448 (rounding to 448 or beyond e4m3's range) and +-inf both give +-448 (0x7E / 0xFE)
        big = ((src & 0x7FFF) >= 0x43E0) & ((src & 0x7FFF) <= 0x7F80)   # |x| >= 448, inf
        sel = np.zeros_like(a, dtype=bool)
        sel.reshape(-1, kvh, 128)[s[s >= 0]] = big[s >= 0]
        assert np.all((a[sel] & 0x7F) == 0x7E)


def test_decode_config1_against_reference_gpu(ref):
    from nanovllm_b200 import fp8_decode_attention, workloads
    c = workloads.config1("cuda")
    args = (c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale)
    r = ref["decode"](*args)
    o = fp8_decode_attention(*args)
    torch.cuda.synchronize()
    assert_close(o, r, what="config1 decode vs reference GPU")


def test_decode_sampled_config5_against_reference_gpu(ref):
    from nanovllm_b200 import fp8_decode_attention, workloads
    c = workloads.config5("cuda", gpus=8, rank=5, batch=2)
    args = (c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale)
    r = ref["decode"](*args)
    o = fp8_decode_attention(*args)
    torch.cuda.synchronize()
    assert_close(o, r, what="config5 shard decode vs reference GPU")


def _prefill_both(ref, c):
    from nanovllm_b200 import fp8_prefill_attention
    kw = dict(block_tables=c.block_tables, cu_seqlens_q=c.cu_seqlens_q,
              cu_seqlens_k=c.cu_seqlens_k, max_seqlen_q=c.max_seqlen_q,
              max_seqlen_k=c.max_seqlen_k, softmax_scale=c.scale)
    r = ref["prefill"](c.q, c.k, c.v, **kw)
    o = fp8_prefill_attention(c.q, c.k, c.v, **kw)
    torch.cuda.synchronize()
    return o, r


def test_prefill_paged_reduced_config3_against_reference_gpu(ref):
    from nanovllm_b200 import store_kvcache, workloads
    gen = torch.Generator().manual_seed(2)
    nqs = torch.randint(128, 513, (4,), generator=gen).tolist()
    pre = torch.randint(0, 3585, (4,), generator=gen).tolist()
    c = workloads.prefill_case(nqs, pre, 32, 8, seed=52, device="cuda")
    store_kvcache(c.new_k, c.new_v, c.k, c.v, c.slot_mapping)
    o, r = _prefill_both(ref, c)
    assert_close(o, r, what="reduced config3 vs reference GPU")


def test_prefill_contiguous_against_reference_gpu(ref):
    from nanovllm_b200 import workloads
    c = workloads.prefill_case([300, 17, 130], [0, 0, 0], 32, 8, seed=53, device="cuda",
                               paged=False)
    o, r = _prefill_both(ref, c)
    assert_close(o, r, what="contiguous prefill vs reference GPU")


def test_mixed_spec_batch_against_reference_gpu(ref):
    from nanovllm_b200 import store_kvcache, workloads
    gen = torch.Generator().manual_seed(3)
    ctx = torch.randint(1024, 4000, (6,), generator=gen).tolist()
    c = workloads.prefill_case([5] * 6 + [300], ctx + [0], 32, 8, seed=54, device="cuda")
    store_kvcache(c.new_k, c.new_v, c.k, c.v, c.slot_mapping)
    o, r = _prefill_both(ref, c)
    assert_close(o, r, what="mixed spec-verify batch vs reference GPU")
