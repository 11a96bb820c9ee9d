"""The oracle is pinned here: against the reference's own kernels (golden fixtures produced by
running them under TRITON_INTERPRET=1, see tests/golden/make_golden.py) and against torch's
bf16 -> float8_e4m3fn cast for every bf16 bit pattern."""
import numpy as np
import pytest
import torch

from helpers import bf16, bits, fp8, u8, assert_close
from oracle import attention as oatt
from oracle import e4m3
from oracle import store as ostore

DECODE_CASES = ["decode_bs32", "decode_bs256", "decode_bs16_g8"]
PREFILL_CASES = ["prefill_paged", "prefill_paged_small", "prefill_paged_bs256", "prefill_contig"]


def test_e4m3_cast_matches_torch_for_all_bf16():
    allbits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    x = torch.from_numpy(allbits.view(np.int16)).view(torch.bfloat16)
    torch_codes = x.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    ours = e4m3.from_bf16_bits(allbits, e4m3.TORCH)
    xf = x.float().numpy()
    finite = np.isfinite(xf)
    assert np.array_equal(ours[finite], torch_codes[finite])
    # NaN inputs: both produce a NaN code
    nan_codes = ours[np.isnan(xf)] & 0x7F
    assert np.all(nan_codes == 0x7F)
    # satfinite mode agrees wherever |x| <= 464 and saturates beyond
    sat = e4m3.from_bf16_bits(allbits, e4m3.SATFINITE)
    small = finite & (np.abs(xf) <= 464)
    assert np.array_equal(sat[small], torch_codes[small])
    big = finite & (np.abs(xf) > 464)
    assert np.all((sat[big] & 0x7F) == 0x7E)
    assert np.array_equal(sat[big] >> 7, (allbits[big] >> 15).astype(np.uint8))


def test_e4m3_widen_matches_torch():
    codes = np.arange(256, dtype=np.uint8)
    ours = e4m3.to_f32(codes)
    ref = u8(codes).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(ours), np.isnan(ref))
    ok = ~np.isnan(ref)
    assert np.array_equal(ours[ok], ref[ok])


def test_scaled_quantiser_roundtrip():
    rng = np.random.default_rng(0)
    x = torch.from_numpy(rng.standard_normal((64, 128)).astype(np.float32) * 5).to(torch.bfloat16)
    x[3] = 0
    codes, scales = e4m3.quant_rows(bits(x))
    assert scales[3] == 1.0 and np.all(codes[3] == 0)
    back = e4m3.to_f32(codes) * scales[:, None]
    amax = x.float().abs().amax(dim=1).numpy()
    np.testing.assert_allclose(scales[amax > 0], amax[amax > 0] / 448.0, rtol=1e-6)
    # rounding error of e4m3 is <= 2^-4 relative (plus subnormal quantum)
    err = np.abs(back - x.float().numpy())
    assert np.all(err <= np.abs(x.float().numpy()) / 16 + scales[:, None] * 2.0 ** -9 + 1e-30)


def test_store_placement_matches_reference(golden):
    g = golden("store_placement")
    qkv = g["qkv"]
    hq, kvh = int(g["hq"]), int(g["kvh"])
    key = qkv[:, hq:hq + kvh]
    value = qkv[:, hq + kvh:]
    nb, bs = g["k_cache"].shape[:2]
    kc = np.full(g["k_cache"].shape, int(g["init"]), dtype=np.uint8)
    vc = np.full(g["v_cache"].shape, int(g["init"]), dtype=np.uint8)
    ostore.store_kvcache(key, value, kc, vc, g["slots"])
    assert np.array_equal(kc, g["k_cache"])
    assert np.array_equal(vc, g["v_cache"])


@pytest.mark.parametrize("name", DECODE_CASES)
def test_decode_oracle_matches_reference(golden, name):
    g = golden(name)
    out = oatt.decode(bf16(g["q"]), fp8(g["k_cache"]), fp8(g["v_cache"]),
                      torch.from_numpy(g["block_tables"]), torch.from_numpy(g["context_lens"]),
                      float(g["scale"]))
    ref = bf16(g["out"])
    # same fp32 math up to summation order: agreement to a few bf16 ulps
    assert_close(out, ref, atol=4e-3, rtol=8e-3, what=name)


@pytest.mark.parametrize("name", PREFILL_CASES)
def test_prefill_oracle_matches_reference(golden, name):
    g = golden(name)
    tables = torch.from_numpy(g["block_tables"]) if "block_tables" in g else None
    out = oatt.prefill(bf16(g["q"]), fp8(g["k"]), fp8(g["v"]), tables,
                       torch.from_numpy(g["cu_seqlens_q"]), torch.from_numpy(g["cu_seqlens_k"]),
                       float(g["scale"]))
    assert_close(out, bf16(g["out"]), atol=4e-3, rtol=8e-3, what=name)


def test_qk_epilogue_oracle_matches_reference_outputs(golden):
    """oracle/qknorm.py against the reference's compiled RMSNorm -> RotaryEmbedding -> Triton
    store on the same inputs (tests/golden/make_golden_qk.py, run on a GPU): q and k nearly all
    identical and otherwise within what one step of a normalised value allows (the restatement
    rounds the sum of squares and the rsqrt correctly, the GPU does not), cache bytes equal
    wherever k is."""
    import torch
    from oracle import qknorm as oqk
    g = golden("qk_epilogue")
    n = g["qkv"].shape[0]
    hq, kvh = int(g["hq"]), int(g["kvh"])
    kc = np.full(g["k_cache"].shape, 0x55, dtype=np.uint8)
    vc = kc.copy()
    q, k = oqk.qk_norm_rope_store(bf16(g["qkv"]), torch.arange(n), bf16(g["q_weight"]),
                                  bf16(g["k_weight"]), float(g["eps"]),
                                  torch.from_numpy(g["cos_sin_rows"]), hq, kvh, kc, vc, g["slots"])
    for name, got in (("q", q), ("k", k)):
        ref = torch.from_numpy(g[name].view(np.int16)).view(torch.bfloat16).float()
        err = (got.float() - ref).abs()
        # one bf16 step of a normalised value moves a rotated output by at most 2^-7 of its
        # head's largest value (plus its own rounding); nearly all outputs are identical
        bound = 2.0 ** -7 * ref.abs().amax(-1, keepdim=True) + 2.0 ** -8 * ref.abs()
        assert bool((err <= bound).all()), (name, float(err.max()))
        exact = (got.view(torch.int16).numpy() == g[name].view(np.int16)).mean()
        assert exact >= 0.999, (name, exact)
    assert np.array_equal(vc, g["v_cache"])
    same = (k.view(torch.int16).numpy() == g["k"].view(np.int16))
    s = g["slots"]
    keep = s >= 0
    got = kc.reshape(-1, kvh, 128)[s[keep]]
    exp = g["k_cache"].reshape(-1, kvh, 128)[s[keep]]
    assert np.array_equal(got[same[keep]], exp[same[keep]])


def test_fp8_linear_oracle_matches_reference_fixture(golden):
    """oracle/fp8_linear.py against the reference's fp8_dyn_quant_kernel and fp8_block_linear run
    on a GPU (tests/golden/make_golden_fp8linear.py).  Quantisation: scales identical, bytes
    identical except where the quotient x / s lies within a few ulp of an e4m3 rounding midpoint
    (the reference divides with the GPU's approximate fp32 division; the restatement's quotient is
    the IEEE one), and there the neighbouring code.  GEMM, on the reference's own quantised bytes:
    within one bf16 step of the reference plus 1e-3 of the output's largest magnitude (fp32
    accumulation order), nearly all identical."""
    from oracle import fp8_linear as ofl
    g = golden("fp8_linear")
    for i, (m, k, n) in enumerate(g["shapes"].tolist()):
        x, w, ws = g[f"x_{i}"], g[f"w_{i}"], g[f"ws_{i}"]
        xq, xs = ofl.dyn_quant(x)
        assert np.array_equal(xs, g[f"xs_{i}"]), i
        differ = xq != g[f"xq_{i}"]
        assert bool(ofl.near_midpoint(x, ulps=4)[differ].all()), (i, int(differ.sum()))
        a, b = xq[differ].astype(np.int16), g[f"xq_{i}"][differ].astype(np.int16)
        assert bool((np.abs((a & 0x7F) - (b & 0x7F)) == 1).all()) and bool(((a ^ b) & 0x80 == 0).all())
        if i == 0:
            assert int(xs[0, 0]) == 0x3F80                 # the all-zero group: scale 1
        y = ofl.block_gemm_f32(g[f"xq_{i}"], g[f"xs_{i}"], w, ws)
        r = ofl.bf16_bits_to_f32(g[f"y_{i}"])
        err = np.abs(ofl.bf16_bits_to_f32(ofl.f32_to_bf16_bits(y)).astype(np.float64) - r)
        bound = 2.0 ** -7 * np.abs(r) + 1e-3 * float(np.abs(r).max())
        assert bool((err <= bound).all()), (i, float(err.max()))
        assert (ofl.f32_to_bf16_bits(y) == g[f"y_{i}"]).mean() >= 0.97, i
