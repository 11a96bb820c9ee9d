"""Device-side mechanisms checked on their own, through the C-ABI diagnostics entry points.

Failure detection: every wait of the engines on an mbarrier is bounded by wall-clock time and, when
the bound passes, records kDevErrWaitTimeout (1) in the workspace's error word and gives up instead
of hanging or trapping.  fp8attn_diag_wait_timeout makes such a wait run out on purpose (a barrier
that nothing arrives on, a 1 ms limit) and the test reads the status the host sees: the launch
ends, the error word is 1, the work counters are back at zero, the context is still usable, and the
stream-ordered error reader returns and clears the word.

exp2 on the FMA pipe: the prefill softmax computes some exponentials with exp2_poly_x2 (range
reduction x = n + f with n = rint(x), 2^n placed in the exponent field, 2^f on [-0.5, 0.5] by a
degree-3 polynomial fitted for relative error) instead of the MUFU ex2.approx; its documented bound
is a relative error below 1e-4 over the arguments the softmax produces ([-125, 8]).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from nanovllm_b200 import _lib
    return _lib


def test_bounded_wait_times_out_and_reports():
    L = _lib()
    ws = torch.zeros(64, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    assert L.lib.fp8attn_diag_wait_timeout(ws.data_ptr(), 1_000_000, 8, stream) == L.OK
    b.record()
    torch.cuda.synchronize()
    ctrl = ws[:3].tolist()
    assert ctrl == [1, 0, 0], ctrl        # wait timed out; work counters released
    assert a.elapsed_time(b) >= 1.0       # it did wait for (at least) its 1 ms limit
    # the stream-ordered reader returns the word and clears it
    host = torch.full((1,), -1, dtype=torch.int32).pin_memory()
    L.check(L.lib.fp8attn_read_error(ws.data_ptr(), host.data_ptr(), 1, stream))
    torch.cuda.synchronize()
    assert int(host[0]) == 1 and int(ws[0]) == 0
    # the context is still usable: a decode call right after is correct and error-free
    from nanovllm_b200 import fp8_decode_attention, workloads
    from nanovllm_b200.fp8_attention import device_error
    from oracle import attention as oatt
    from helpers import assert_close
    c = workloads.decode_case(3, 8, 2, 100, 700, seed=77, device="cuda", block_size=64)
    out = fp8_decode_attention(c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale)
    ref = oatt.decode(c.q.cpu(), c.k_cache.cpu(), c.v_cache.cpu(), c.block_tables.cpu(),
                      c.context_lens.cpu(), c.scale)
    assert_close(out, ref, what="decode after a timed-out diagnostic wait")
    assert device_error() == 0


def test_exp2_poly_relative_error_bound():
    L = _lib()
    x = np.concatenate([np.linspace(-125.0, 8.0, 1 << 21), np.arange(-125, 9, 0.5),
                        [0.0, -0.0, 0.49999997, -0.49999997, 7.9999995, -124.99999]])
    xt = torch.from_numpy(x.astype(np.float32)).cuda()
    poly, mufu = torch.empty_like(xt), torch.empty_like(xt)
    L.check(L.lib.fp8attn_diag_exp2(xt.data_ptr(), poly.data_ptr(), mufu.data_ptr(), xt.numel(),
                                    torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    xf = xt.cpu().double().numpy()
    truth = np.exp2(xf)
    rel_poly = np.abs(poly.cpu().double().numpy() / truth - 1.0)
    rel_mufu = np.abs(mufu.cpu().double().numpy() / truth - 1.0)
    assert rel_poly.max() < 1e-4, (rel_poly.max(), xf[rel_poly.argmax()])
    assert rel_mufu.max() < 1e-6          # the MUFU result it stands in for
    # below the range the result stays tiny (it is clamped at 2^-125), never inf or NaN
    far = torch.tensor([-200.0, -1e30, float("-inf")], device="cuda")
    p2, m2 = torch.empty_like(far), torch.empty_like(far)
    L.check(L.lib.fp8attn_diag_exp2(far.data_ptr(), p2.data_ptr(), m2.data_ptr(), 3,
                                    torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert torch.all(p2.cpu() <= 2.0 ** -124) and torch.all(p2.cpu() >= 0)
