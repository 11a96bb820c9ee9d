"""Store kernel parity: cache bytes, scales and slot placement bit-exact against the oracle."""
import numpy as np
import pytest
import torch

from helpers import bf16, bits
from oracle import e4m3
from oracle import store as ostore

pytestmark = pytest.mark.gpu


def _run(key, value, nb, bs, kvh, slots, scaled=False, with_scales=False, init=0x55):
    from nanovllm_b200 import store_kvcache
    dev = "cuda"
    kc = torch.full((nb, bs, kvh, 128), init, dtype=torch.uint8, device=dev).view(torch.float8_e4m3fn)
    vc = torch.full((nb, bs, kvh, 128), init, dtype=torch.uint8, device=dev).view(torch.float8_e4m3fn)
    ks = vs = None
    if with_scales:
        ks = torch.full((nb, bs, kvh), -7.0, dtype=torch.float32, device=dev)
        vs = torch.full((nb, bs, kvh), -7.0, dtype=torch.float32, device=dev)
    store_kvcache(key.to(dev), value.to(dev), kc, vc, slots.to(dev), ks, vs, scaled=scaled)
    torch.cuda.synchronize()
    res = [kc.view(torch.uint8).cpu().numpy(), vc.view(torch.uint8).cpu().numpy()]
    if with_scales:
        res += [ks.cpu().numpy(), vs.cpu().numpy()]
    return res


def _oracle(key, value, nb, bs, kvh, slots, scaled=False, with_scales=False, init=0x55):
    kc = np.full((nb, bs, kvh, 128), init, dtype=np.uint8)
    vc = np.full((nb, bs, kvh, 128), init, dtype=np.uint8)
    ks = vs = None
    if with_scales:
        ks = np.full((nb, bs, kvh), -7.0, dtype=np.float32)
        vs = np.full((nb, bs, kvh), -7.0, dtype=np.float32)
    ostore.store_kvcache(bits(key), bits(value), kc, vc, slots.numpy(), ks, vs, scaled=scaled)
    return [kc, vc] + ([ks, vs] if with_scales else [])


def test_store_golden_placement(golden):
    g = golden("store_placement")
    qkv = bf16(g["qkv"]).cuda()
    hq, kvh = int(g["hq"]), int(g["kvh"])
    key = qkv[:, hq:hq + kvh].contiguous()
    value = qkv[:, hq + kvh:]                       # strided rows, as in the engine
    nb, bs = g["k_cache"].shape[:2]
    kc, vc = _run(key, value, nb, bs, kvh, torch.from_numpy(g["slots"]))
    assert np.array_equal(kc, g["k_cache"]) and np.array_equal(vc, g["v_cache"])


@pytest.mark.parametrize("kvh", [1, 2, 8])
def test_store_rounding_all_bf16_patterns(kvh):
    # every bf16 bit pattern (finite, inf and NaN) goes through the kernel once
    allbits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    per_row = kvh * 128
    n = (allbits.size + per_row - 1) // per_row
    pad = np.zeros(n * per_row, dtype=np.uint16)
    pad[:allbits.size] = allbits
    key = bf16(pad.reshape(n, kvh, 128))
    value = bf16(np.roll(pad, 12345).reshape(n, kvh, 128))
    bs = 16
    nb = (n + bs - 1) // bs
    slots = torch.randperm(nb * bs, generator=torch.Generator().manual_seed(kvh))[:n].to(torch.int32)
    got = _run(key, value, nb, bs, kvh, slots)
    ref = _oracle(key, value, nb, bs, kvh, slots)
    for a, b in zip(got, ref):
        same = a == b
        # NaN inputs: any NaN code is acceptable (sign of a NaN is not specified)
        nan_ok = ((a & 0x7F) == 0x7F) & ((b & 0x7F) == 0x7F)
        assert np.all(same | nan_ok)


def test_store_engine_shapes_and_skip():
    gen = torch.Generator().manual_seed(0)
    n, hq, kvh, bs, nb = 777, 32, 8, 256, 9
    qkv = (torch.randn(n, hq + 2 * kvh, 128, generator=gen) * 3).to(torch.bfloat16)
    key = qkv[:, hq:hq + kvh].contiguous()
    value = qkv[:, hq + kvh:]
    slots = torch.randperm(nb * bs, generator=gen)[:n].to(torch.int32)
    slots[::7] = -1
    got = _run(key, value, nb, bs, kvh, slots)
    ref = _oracle(key, value, nb, bs, kvh, slots)
    for a, b in zip(got, ref):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("scaled", [False, True])
def test_store_scales(scaled):
    gen = torch.Generator().manual_seed(1)
    n, kvh, bs, nb = 300, 4, 32, 12
    key = (torch.randn(n, kvh, 128, generator=gen) * 50).to(torch.bfloat16)
    value = (torch.randn(n, kvh, 128, generator=gen) * 0.01).to(torch.bfloat16)
    key[5] = 0                                   # all-zero rows: scale 1
    key[6, 1, 3] = 1e30                          # far beyond e4m3 range
    slots = torch.randperm(nb * bs, generator=gen)[:n].to(torch.int32)
    slots[-3:] = -1
    got = _run(key, value, nb, bs, kvh, slots, scaled=scaled, with_scales=True)
    ref = _oracle(key, value, nb, bs, kvh, slots, scaled=scaled, with_scales=True)
    for a, b in zip(got, ref):
        assert np.array_equal(a, b)


def test_store_empty_and_unaligned_rows():
    from nanovllm_b200 import store_kvcache
    kc = torch.zeros(2, 16, 1, 128, dtype=torch.uint8, device="cuda").view(torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    e = torch.empty(0, 1, 128, dtype=torch.bfloat16, device="cuda")
    store_kvcache(e, e, kc, vc, torch.empty(0, dtype=torch.int32, device="cuda"))
    # rows that are not 16-byte aligned take the scalar path
    base = torch.randn(10 * 129 + 1, dtype=torch.float32).to(torch.bfloat16).cuda()
    key = base[1:1 + 10 * 129].view(10, 129)[:, :128].unsqueeze(1)
    slots = torch.arange(10, dtype=torch.int32, device="cuda")
    store_kvcache(key, key, kc, vc, slots)
    torch.cuda.synchronize()
    ref = key.float().cpu().to(torch.bfloat16).to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(kc.view(torch.uint8).view(-1, 128)[:10].cpu(), ref.view(10, 128))
