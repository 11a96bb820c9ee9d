"""The C-ABI boundary without a GPU: the library loads, exports every function include/fp8attn.h
declares, and rejects bad arguments before touching a device."""
import ctypes
import subprocess

import pytest

from nanovllm_b200 import _lib
from nanovllm_b200.build import LIB_PATH


def test_library_exports_every_header_symbol():
    declared = _lib.header_symbols()
    assert len(declared) >= 7
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    for s in declared:
        assert hasattr(_lib.lib, s)


def test_library_has_no_hard_cuda_driver_dependency():
    # the driver is resolved at run time, so the library also loads on GPU-less hosts
    out = subprocess.run(["ldd", LIB_PATH], capture_output=True, text=True).stdout
    assert "libcuda.so" not in out


def test_version_and_min_chunk_knob():
    assert _lib.lib.fp8attn_version() >= 100
    prev = _lib.lib.fp8attn_set_decode_min_chunk(256)
    assert prev == 128
    assert _lib.lib.fp8attn_set_decode_min_chunk(192) == -1      # not a multiple of 128
    assert _lib.lib.fp8attn_set_decode_min_chunk(prev) == 256


def _decode_call(**over):
    a = dict(out=16, q=16, q_row_stride=32 * 128, k=16, v=16, ks=None, vs=None, bt=16,
             bt_stride=4, max_blocks=4, ctx=16, num_seqs=2, hq=32, kvh=8, d=128, nb=10, bs=256,
             scale=0.088, ws=16, ws_bytes=1 << 20, stream=None)
    a.update(over)
    return _lib.lib.fp8attn_decode(a["out"], a["q"], a["q_row_stride"], a["k"], a["v"], a["ks"],
                                   a["vs"], a["bt"], a["bt_stride"], a["max_blocks"], a["ctx"],
                                   a["num_seqs"], a["hq"], a["kvh"], a["d"], a["nb"], a["bs"],
                                   a["scale"], a["ws"], a["ws_bytes"], a["stream"])


@pytest.mark.parametrize("bad,msg", [
    (dict(d=64), "head_dim"),
    (dict(hq=30), "multiple"),
    (dict(bs=24), "block_size"),
    (dict(bt_stride=2), "block table"),
    (dict(q=8), "aligned"),
    (dict(k=None), "null"),
    (dict(num_seqs=5000), "num_seqs"),
    (dict(max_blocks=1 << 20, bt_stride=1 << 20), "2^24"),
    (dict(ks=16), "both"),
])
def test_decode_rejects_bad_arguments(bad, msg):
    rc = _decode_call(**bad)
    assert rc == _lib.EINVAL
    assert msg in _lib.lib.fp8attn_last_error().decode()


def test_store_rejects_bad_arguments():
    f = _lib.lib.fp8attn_store_kvcache
    assert f(16, 1024, 16, 1024, 16, 16, None, None, 16, 4, 8, 64, 100, 0, None) == _lib.EINVAL
    assert f(16, 1024, 16, 1024, 8, 16, None, None, 16, 4, 8, 128, 100, 0, None) == _lib.EINVAL
    assert f(16, 1024, 16, 1024, 16, 16, None, None, 16, 4, 8, 128, 100, 1, None) == _lib.EINVAL
    assert f(16, 1024, 16, 1024, 16, 16, None, None, 16, 0, 8, 128, 100, 0, None) == _lib.OK


def test_prefill_rejects_bad_arguments():
    f = _lib.lib.fp8attn_prefill
    args = [16, 16, 4096, 16, 16, 1024, None, None, None, 0, 0, 16, 16, 2, 8, 8, 32, 8, 128, 100,
            1, 0.088, 16, 1 << 20, None]
    bad = list(args)
    bad[18] = 96                                   # head_dim
    assert f(*bad) == _lib.EINVAL
    bad = list(args)
    bad[5] = 100                                   # contiguous kv row stride < KVH*128
    assert f(*bad) == _lib.EINVAL
    bad = list(args)
    bad[13] = 0                                    # no sequences: nothing to do
    assert f(*bad) == _lib.OK


def test_fp8_linear_rejects_bad_arguments():
    lib = _lib.lib
    assert lib.fp8attn_fp8_gemm_workspace_bytes(4, 0, 128) == -1
    assert lib.fp8attn_fp8_linear_workspace_bytes(-1, 128, 128) == -1
    # a grid that covers the SMs without split-K: only the control words
    assert lib.fp8attn_fp8_gemm_workspace_bytes(1024, 4096, 1024) == 256
    assert lib.fp8attn_fp8_linear_workspace_bytes(1024, 4096, 1024) == \
        256 + 1024 * 1024 + 1024 * 8 * 2
    split = lib.fp8attn_fp8_gemm_workspace_bytes(4, 256, 4096)       # thin: split-K partials
    assert split > 256 and (split - 256) % (4 * 256 * 4) == 0
    q = lib.fp8attn_fp8_dyn_quant
    assert q(4096, 1024, 4096, 1024, 4096, 4, 100, None) == _lib.EINVAL     # K not a multiple of 128
    assert q(4098, 1024, 4096, 1024, 4096, 4, 1024, None) == _lib.EINVAL    # x misaligned
    assert q(4096, 1020, 4096, 1024, 4096, 4, 1024, None) == _lib.EINVAL    # x stride < K
    assert q(None, 1024, 4096, 1024, 4096, 4, 1024, None) == _lib.EINVAL
    assert q(4096, 1024, 4096, 1024, 4096, 0, 1024, None) == _lib.OK        # empty batch
    g = lib.fp8attn_fp8_block_gemm
    args = [4096, 1024, 4096, 4096, 4096, 4096, 256, 4, 256, 1024, 4096, 1 << 20, None]
    bad = list(args)
    bad[8] = 200                                   # N not a multiple of 128
    assert g(*bad) == _lib.EINVAL
    bad = list(args)
    bad[1] = 1032                                  # xq row stride not a multiple of 16
    assert g(*bad) == _lib.EINVAL
    bad = list(args)
    bad[11] = 16                                   # workspace too small
    assert g(*bad) == _lib.EWORKSPACE
    bad = list(args)
    bad[7] = 0                                     # empty batch: nothing to do
    assert g(*bad) == _lib.OK
    lin = lib.fp8attn_fp8_block_linear
    assert lin(4096, 1024, 4096, 4096, 4096, 256, 4, 256, 1000, 4096, 1 << 20, None) == _lib.EINVAL
    assert lin(4096, 1024, 4096, 4096, 4096, 256, 4, 256, 1024, 4096, 64, None) == _lib.EWORKSPACE
    assert "workspace" in lib.fp8attn_last_error().decode()


def test_tp_linear_layout_and_rejects_bad_arguments():
    lib = _lib.lib
    out_off, recv_off = ctypes.c_int64(), ctypes.c_int64()
    total = lib.fp8attn_tp_linear_layout(1000, 1024, 2, ctypes.byref(out_off),
                                         ctypes.byref(recv_off))
    tiles = 8 * 8                                   # ceil(1000 / 128) token tiles x 1024 / 128
    assert out_off.value == (3 * tiles * 8 + 255) // 256 * 256
    assert recv_off.value == out_off.value + 1000 * 1024 * 2
    assert total == recv_off.value + 2 * 1000 * 1024 * 2
    assert lib.fp8attn_tp_linear_layout(1000, 1000, 2, None, None) == -1
    assert lib.fp8attn_tp_linear_layout(1000, 1024, 0, None, None) == -1
    assert lib.fp8attn_fp8_tp_linear_workspace_bytes(10, 100) == -1
    table = (ctypes.c_void_p * 2)(4096, 8192)
    f = lib.fp8attn_fp8_tp_linear
    args = [4096, 1024, 4096, 4096, table, 0, 2, 1, 256, 64, 1024, 1024, 4096, 1 << 20, None]
    for i, v in ((5, 2), (6, 9), (7, 0), (8, 32), (10, 1000)):   # rank, world, epoch, max, N
        bad = list(args)
        bad[i] = v
        assert f(*bad) == _lib.EINVAL, (i, v)
    bad = list(args)
    bad[4] = (ctypes.c_void_p * 2)(4096, 8200)       # a buffer not 256-byte aligned
    assert f(*bad) == _lib.EINVAL
    bad = list(args)
    bad[13] = 64                                      # workspace too small
    assert f(*bad) == _lib.EWORKSPACE
    bad = list(args)
    bad[9] = 0                                        # no rows: nothing to do
    assert f(*bad) == _lib.OK


def _splits(m, n, k, sms=148):
    """The GEMM's split-K rule: only with fewer output tiles (128 tokens x 128 features) than SMs,
    the number of K ranges s minimising ceil(units / SMs) * ceil(blocks / s), the smaller on ties,
    with every range non-empty."""
    base = (n // 128) * ((m + 127) // 128)
    kc = k // 128
    if base >= sms:
        return 1
    best, best_cost = 1, -(-base // sms) * kc
    for s in range(2, min(16, kc) + 1):
        per = -(-kc // s)
        if -(-kc // per) != s:
            continue
        cost = -(-(base * s) // sms) * per
        if cost < best_cost:
            best, best_cost = s, cost
    return best


def test_fp8_gemm_split_policy_and_workspace_sizes():
    """Without a GPU the library assumes 148 SMs (a B200).  Without split-K the output equals the
    reference's Triton kernel bit for bit; with it, within the accumulation-order bound."""
    lib = _lib.lib
    for m in (1, 37, 128, 256, 1000, 8192):
        for n in (1024, 4096, 6144):
            for k in (1024, 4096, 12288):
                s = _splits(m, n, k)
                want = 256 + (s * m * n * 4 if s > 1 else 0)
                assert lib.fp8attn_fp8_gemm_workspace_bytes(m, n, k) == want, (m, n, k, s)
    assert _splits(8192, 6144, 4096) == 1      # the prefill-size QKV projection: no split
    assert _splits(256, 6144, 4096) == 3       # the decode-size one: three K ranges
