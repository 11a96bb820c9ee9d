"""FP8 block-scaled linear layer (fp8attn_fp8_dyn_quant / _block_gemm / _block_linear).

* Against the CPU restatement (oracle/fp8_linear.py) on seeded inputs: quantised bytes identical
  except where the fp32 quotient lies within a few ulp of an e4m3 rounding midpoint (there the
  kernel, like the reference, divides with the GPU's approximate fp32 division and may round to
  the neighbouring code), scales identical but for a rare one-step difference of the same
  origin; GEMM outputs within one bf16 step plus the fp32 accumulation-order allowance, over
  shapes with partial token tiles, single and split-K grids.
* Against the reference's own Triton kernels run on the same GPU from its unmodified install under
  baseline/_ref: quantised bytes and scales identical bit for bit, outputs within the same bound.
* Against the committed fixture of the reference's outputs (tests/golden/fp8_linear.npz).
* Empty batch, strided activations, determinism, the device error word.
"""
import os
import sys

import numpy as np
import pytest
import torch

from oracle import fp8_linear as ofl

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
GOLDEN = os.path.join(ROOT, "tests", "golden", "fp8_linear.npz")


def _bits16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _bits8(t):
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


def _inputs(m, k, n, seed, sd=2.0):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(m, k, generator=g) * sd).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.5).to(torch.float8_e4m3fn)
    ws = (torch.rand(n // 128, k // 128, generator=g) * 0.02 + 0.001).to(torch.bfloat16)
    return x, w, ws


def _assert_quant_close(xq, xs, x_bits, ref_xq, ref_xs, ulps=6):
    """xq / ref_xq e4m3 codes, xs / ref_xs bf16 scale bits.  The GPU's scale amax / 448 is also
    an approximate quotient (within 2 fp32 ulp), so a scale whose fp32 value lies next to a bf16
    rounding midpoint may be one bf16 step away, and the quotients x / s (each within 2 ulp, over
    scales up to 2 ulp apart) within ``ulps`` of an e4m3 midpoint may round the other way."""
    sd = xs != ref_xs
    assert sd.mean() < 1e-3
    assert bool((np.abs(xs[sd].astype(np.int32) - ref_xs[sd].astype(np.int32)) == 1).all())
    differ = xq != ref_xq
    if differ.any():
        near = ofl.near_midpoint(x_bits, ulps=ulps)
        assert bool(near[differ].all()), int((differ & ~near).sum())
        # the neighbouring code of the same sign
        a, b = xq[differ].astype(np.int16), ref_xq[differ].astype(np.int16)
        assert bool(((a & 0x80) == (b & 0x80)).all())
        assert bool((np.abs((a & 0x7F) - (b & 0x7F)) == 1).all())
    assert differ.mean() < 5e-3                  # exact midpoints are common with bf16 inputs


def _assert_out_close(y_bits, ref_f32_or_bits, what, min_exact=0.97):
    """Within one bf16 step of the reference value plus 1e-3 of the output's largest magnitude
    (fp32 accumulation in another order, split-K partial sums)."""
    y = ofl.bf16_bits_to_f32(y_bits)
    r = ref_f32_or_bits
    if r.dtype == np.uint16:
        r = ofl.bf16_bits_to_f32(r)
    err = np.abs(y.astype(np.float64) - r.astype(np.float64))
    bound = 2.0 ** -7 * np.abs(r) + 1e-3 * max(float(np.abs(r).max()), 1e-30)
    assert bool((err <= bound).all()), (what, float(err.max()))
    if ref_f32_or_bits.dtype == np.uint16:
        exact = float((y_bits == ref_f32_or_bits).mean())
        assert exact >= min_exact, (what, exact)


@pytest.mark.parametrize("m,k", [(1, 128), (5, 4096), (300, 1024), (64, 7168)])
def test_quant_matches_oracle(m, k):
    from nanovllm_b200.fp8_linear import fp8_dyn_quant
    x, _, _ = _inputs(m, k, 128, seed=m * 7 + k)
    x[0, :128] = 0                              # all-zero group: scale 1
    if m > 1:
        x[1, 3] = 5000.0                        # a large value: the rest of its group is tiny
    xq, xs = fp8_dyn_quant(x.cuda())
    torch.cuda.synchronize()
    ref_xq, ref_xs = ofl.dyn_quant(_bits16(x))
    _assert_quant_close(_bits8(xq), _bits16(xs), _bits16(x), ref_xq, ref_xs)
    assert int(_bits16(xs)[0, 0]) == 0x3F80    # bf16 1.0


@pytest.mark.parametrize("m,k,n", [
    (1, 128, 128),        # one K block, one token
    (4, 4096, 256),       # thin decode GEMM: split-K
    (37, 2048, 1024),     # partial token tile, split-K
    (130, 1024, 512),     # three token tiles, the last partial
    (512, 1024, 4096),    # 128 units, no split
    (1000, 1024, 4096),   # 256 units on the persistent grid: CTAs run two, the last tile partial
])
def test_gemm_matches_oracle(m, k, n):
    from nanovllm_b200.fp8_linear import fp8_block_gemm, fp8_dyn_quant
    x, w, ws = _inputs(m, k, n, seed=m + k + n)
    xd = x.cuda()
    xq, xs = fp8_dyn_quant(xd)
    y = fp8_block_gemm(xq, xs, w.cuda(), ws.cuda())
    torch.cuda.synchronize()
    ref = ofl.block_gemm_f32(_bits8(xq), _bits16(xs), _bits8(w), _bits16(ws))
    _assert_out_close(_bits16(y), ref, f"gemm {m}x{k}x{n}")
    exact = float((_bits16(y) == ofl.f32_to_bf16_bits(ref)).mean())
    assert exact >= 0.97, exact


def test_linear_strided_input_deterministic_and_error_word():
    from nanovllm_b200.fp8_attention import device_error
    from nanovllm_b200.fp8_linear import fp8_block_linear, fp8_dyn_quant
    m, k, n = 70, 1536, 768
    x, w, ws = _inputs(m, k, n, seed=5)
    base = torch.zeros(m, k + 64, dtype=torch.bfloat16, device="cuda")
    base[:, :k] = x.cuda()
    xs_view = base[:, :k]                       # rows k + 64 elements apart
    wd, wsd = w.cuda(), ws.cuda()
    y1 = fp8_block_linear(xs_view, wd, wsd)
    y2 = fp8_block_linear(xs_view, wd, wsd)
    y3 = fp8_block_linear(x.cuda(), wd, wsd)
    torch.cuda.synchronize()
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))
    assert torch.equal(y1.view(torch.int16), y3.view(torch.int16))
    # against the restatement's GEMM on the kernel's own quantised bytes (the bytes themselves
    # are checked by test_quant_matches_oracle: a code one step away moves an output by more
    # than the accumulation-order bound)
    xq, xsc = fp8_dyn_quant(xs_view)
    torch.cuda.synchronize()
    ref = ofl.block_gemm_f32(_bits8(xq), _bits16(xsc), _bits8(w), _bits16(ws))
    _assert_out_close(_bits16(y1), ref, "linear")
    assert device_error() == 0


def test_empty_batch_and_rejected_shapes():
    from nanovllm_b200 import _lib
    from nanovllm_b200.fp8_linear import fp8_block_linear
    w = torch.zeros(256, 256, dtype=torch.float8_e4m3fn, device="cuda")
    ws = torch.ones(2, 2, dtype=torch.bfloat16, device="cuda")
    y = fp8_block_linear(torch.empty(0, 256, dtype=torch.bfloat16, device="cuda"), w, ws)
    assert tuple(y.shape) == (0, 256)
    x = torch.ones(3, 256, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(3, 200, dtype=torch.bfloat16, device="cuda")
    rc = _lib.lib.fp8attn_fp8_block_linear(x.data_ptr(), 256, w.data_ptr(), ws.data_ptr(),
                                           out.data_ptr(), 200, 3, 200, 256, None, 0, None)
    assert rc == _lib.EINVAL


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "nanovllm")):
        pytest.skip("the reference is not installed under baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    from nanovllm.kernels.fp8_linear import fp8_block_linear, fp8_dyn_quant_kernel
    return fp8_dyn_quant_kernel, fp8_block_linear


@pytest.mark.parametrize("m,k,n", [(1, 4096, 6144), (64, 4096, 1024), (257, 2048, 768),
                                   (1024, 1024, 2048)])
def test_against_reference_kernels(ref, m, k, n):
    quant_kernel, ref_linear = ref
    from nanovllm_b200.fp8_linear import fp8_block_linear, fp8_dyn_quant
    x, w, ws = _inputs(m, k, n, seed=11 * m + n)
    xd, wd, wsd = x.cuda(), w.cuda(), ws.cuda()
    rq = torch.empty(m, k, dtype=torch.float8_e4m3fn, device="cuda")
    rs = torch.empty(m, k // 128, dtype=torch.bfloat16, device="cuda")
    quant_kernel[(m, k // 128)](xd, rq, rs, k // 128, xd.stride(0), rq.stride(0), BLOCK_K=128,
                                num_warps=4)
    ry = ref_linear(xd, wd, wsd)
    xq, xs = fp8_dyn_quant(xd)
    y = fp8_block_linear(xd, wd, wsd)
    torch.cuda.synchronize()
    assert np.array_equal(_bits8(xq), _bits8(rq))        # the same approximate division
    assert np.array_equal(_bits16(xs), _bits16(rs))
    _assert_out_close(_bits16(y), _bits16(ry), f"vs reference {m}x{k}x{n}")


@pytest.mark.skipif(not os.path.exists(GOLDEN), reason="fixture not generated")
def test_recorded_reference_fixture():
    from nanovllm_b200.fp8_linear import fp8_block_linear, fp8_dyn_quant
    g = dict(np.load(GOLDEN))
    for i, (m, k, n) in enumerate(g["shapes"].tolist()):
        x = torch.from_numpy(g[f"x_{i}"].view(np.int16)).view(torch.bfloat16).cuda()
        w = torch.from_numpy(g[f"w_{i}"]).view(torch.float8_e4m3fn).cuda()
        ws = torch.from_numpy(g[f"ws_{i}"].view(np.int16)).view(torch.bfloat16).cuda()
        xq, xs = fp8_dyn_quant(x)
        y = fp8_block_linear(x, w, ws)
        torch.cuda.synchronize()
        assert np.array_equal(_bits8(xq), g[f"xq_{i}"]), i
        assert np.array_equal(_bits16(xs), g[f"xs_{i}"]), i
        _assert_out_close(_bits16(y), g[f"y_{i}"], f"fixture {i}")
