"""Row-parallel FP8 linear with the tensor-parallel all-reduce in one kernel (fp8attn_fp8_tp_linear).

* One GPU, world 1, through the C-ABI on a plain zero-filled buffer: the output equals the
  reference's Triton fp8_block_linear bit for bit (the fused path never splits K), and this
  library's fp8_block_linear within the split-K bound (it splits K when there are fewer output
  tiles than SMs), over calls with growing and shrinking M on the same buffers.
* One GPU, the failure path: a world-2 call whose second rank never runs (its buffer is local
  memory that nothing stamps).  The cross-rank waits give up after their limit, the call ends,
  the workspace's error word reads 1 (wait timed out), and the next call works.
* Two GPUs (skipped with fewer), one process per GPU over NCCL (tests/tp_linear_worker.py): the
  fused output against the reference's Triton fp8_block_linear + NCCL all_reduce
  (RowParallelLinear.forward, nanovllm/layers/linear.py:235-239) on the same K slices, bit for
  bit; against this library's fp8_block_linear + NCCL all_reduce within the split-K bound; and
  against the CPU restatement (oracle/fp8_linear.py) on the GPU's quantised bytes.
"""
import ctypes
import os
import socket
import subprocess
import sys
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _inputs(m, k, n, seed):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(m, k, generator=g) * 2).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.5).to(torch.float8_e4m3fn)
    ws = (torch.rand(n // 128, k // 128, generator=g) * 0.02 + 0.001).to(torch.bfloat16)
    return x.cuda(), w.cuda(), ws.cuda()


def _call(x, w, ws, buffers, rank, world, epoch, max_tokens, workspace):
    from nanovllm_b200 import _lib
    m, k = x.shape
    n = w.shape[0]
    table = (ctypes.c_void_p * world)(*[b.data_ptr() for b in buffers])
    return _lib.lib.fp8attn_fp8_tp_linear(
        x.data_ptr(), x.stride(0), w.data_ptr(), ws.data_ptr(), table, rank, world, epoch,
        max_tokens, m, n, k, workspace.data_ptr(), workspace.numel(),
        torch.cuda.current_stream().cuda_stream)


def _layout(max_tokens, n, world):
    from nanovllm_b200 import _lib
    out_off = ctypes.c_int64()
    total = _lib.lib.fp8attn_tp_linear_layout(max_tokens, n, world, ctypes.byref(out_off), None)
    assert total > 0
    return total, out_off.value


def _ref_linear():
    ref_dir = os.path.join(os.path.dirname(HERE), "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "nanovllm")):
        return None
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    from nanovllm.kernels.fp8_linear import fp8_block_linear
    return fp8_block_linear


def _assert_close(got, want, what, of_max=1e-3):
    """Within one bf16 step plus ``of_max`` of the largest output (fp32 sums in another order)."""
    g, w = got.float(), want.float()
    bound = 2.0 ** -7 * w.abs() + of_max * w.abs().max()
    assert bool(((g - w).abs() <= bound).all()), (what, float((g - w).abs().max()))


def test_world1_equals_block_linear():
    from nanovllm_b200 import _lib
    from nanovllm_b200.fp8_linear import fp8_block_linear
    ref_linear = _ref_linear()
    max_tokens, n = 1024, 2048
    total, out_off = _layout(max_tokens, n, 1)
    buf = torch.zeros(total, dtype=torch.uint8, device="cuda")
    ws_bytes = _lib.lib.fp8attn_fp8_tp_linear_workspace_bytes(max_tokens, 4096)
    wk = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    for epoch, (m, k, seed) in enumerate([(1000, 4096, 1), (37, 2048, 2), (1, 4096, 3),
                                          (640, 1024, 4)], start=1):
        x, w, ws = _inputs(m, k, n, seed)
        assert _call(x, w, ws, [buf], 0, 1, epoch, max_tokens, wk) == _lib.OK
        want = fp8_block_linear(x, w, ws)
        ref = ref_linear(x, w, ws) if ref_linear is not None else None
        torch.cuda.synchronize()
        got = buf[out_off:out_off + m * n * 2].view(torch.bfloat16).view(m, n)
        _assert_close(got, want, (m, k))
        if ref is not None:
            assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), (m, k)
        assert int(wk[:4].view(torch.int32).item()) == 0


def test_missing_peer_times_out_with_error_word():
    from nanovllm_b200 import _lib
    max_tokens, n, m, k = 256, 1024, 200, 1024
    total, _ = _layout(max_tokens, n, 2)
    mine = torch.zeros(total, dtype=torch.uint8, device="cuda")
    absent = torch.zeros(total, dtype=torch.uint8, device="cuda")  # "rank 1": never runs
    wk = torch.zeros(_lib.lib.fp8attn_fp8_tp_linear_workspace_bytes(m, k), dtype=torch.uint8,
                     device="cuda")
    x, w, ws = _inputs(m, k, n, 7)
    t0 = time.time()
    assert _call(x, w, ws, [mine, absent], 0, 2, 1, max_tokens, wk) == _lib.OK
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    assert int(wk[:4].view(torch.int32).item()) == 1     # a wait timed out
    assert elapsed < 30, elapsed                          # one limit per waiting thread, not per tile
    # the context is still usable: a world-1 call right after is correct
    total1, out_off = _layout(max_tokens, n, 1)
    buf = torch.zeros(total1, dtype=torch.uint8, device="cuda")
    wk.zero_()
    assert _call(x, w, ws, [buf], 0, 1, 1, max_tokens, wk) == _lib.OK
    from nanovllm_b200.fp8_linear import fp8_block_linear
    want = fp8_block_linear(x, w, ws)
    torch.cuda.synchronize()
    got = buf[out_off:out_off + m * n * 2].view(torch.bfloat16).view(m, n)
    _assert_close(got, want, "after the timeout")
    assert int(wk[:4].view(torch.int32).item()) == 0


def test_rejects_bad_arguments():
    from nanovllm_b200 import _lib
    total, _ = _layout(256, 1024, 2)
    buf = torch.zeros(total, dtype=torch.uint8, device="cuda")
    wk = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    x, w, ws = _inputs(64, 1024, 1024, 8)
    assert _call(x, w, ws, [buf, buf], 2, 2, 1, 256, wk) == _lib.EINVAL      # rank >= world
    assert _call(x, w, ws, [buf, buf], 0, 2, 0, 256, wk) == _lib.EINVAL      # epoch 0
    assert _call(x, w, ws, [buf, buf], 0, 2, 1, 32, wk) == _lib.EINVAL       # M > max_tokens
    assert _lib.lib.fp8attn_tp_linear_layout(256, 1024, 9, None, None) == -1  # world > 8


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_ranks_against_nccl_and_reference(tmp_path):
    world, port = 2, _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "tp_linear_worker.py"),
                                       str(tmp_path)], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    outs = []
    for p in procs:
        try:
            outs.append(p.communicate(timeout=300)[0])
        except subprocess.TimeoutExpired:
            p.kill()
            outs.append(p.communicate()[0])
    assert all(p.returncode == 0 for p in procs), "\n".join(o[-3000:] for o in outs)
    sys.path.insert(0, HERE)
    import tp_linear_worker as wkr
    from oracle import fp8_linear as ofl
    res = [dict(np.load(tmp_path / f"rank{r}.npz")) for r in range(world)]
    for r in range(world):
        assert int(res[r]["device_error"]) == 0
        assert int(res[r]["epoch"]) == len(wkr.CASES)
    for i in range(len(wkr.CASES)):
        fused = res[0][f"fused_{i}"]
        for r in range(1, world):
            assert np.array_equal(res[r][f"fused_{i}"], fused), i     # every rank holds the sum
        # this library's fp8_block_linear splits K on these thin GEMMs: each rank's bf16 partial
        # may be one step of the partial away, and a partial can be larger than the sum, so the
        # bound is a bf16 step of the largest output
        _assert_close(torch.from_numpy(fused.view(np.int16)).view(torch.bfloat16),
                      torch.from_numpy(res[0][f"nccl_{i}"].view(np.int16)).view(torch.bfloat16),
                      i, of_max=2.0 ** -7)
        # two ranks: NCCL adds the two bf16 partials in fp32 and rounds once, as the kernel does,
        # and the reference's per-rank GEMM is the fused kernel's bit for bit
        if f"ref_{i}" in res[0]:
            assert np.array_equal(fused, res[0][f"ref_{i}"]), i
    # the CPU restatement on case 0, on the quantised bytes this GPU's fp8_dyn_quant gives each
    # rank's slice (the restatement's IEEE quotients flip ~0.1 % of the codes at rounding
    # midpoints, which moves an output by more than the accumulation bound): per rank the block
    # GEMM rounded to bf16, then the ranks' sum in fp32 (oracle.fp8_linear.row_parallel_linear's
    # arithmetic)
    from nanovllm_b200.fp8_linear import fp8_dyn_quant
    x, w, ws = res[0]["x_0"], res[0]["w_0"], res[0]["ws_0"]
    acc = None
    for r in range(world):
        xr, wr, wsr = ofl.rank_slices(x, w, ws, r, world)
        xq, xs = fp8_dyn_quant(torch.from_numpy(xr.view(np.int16)).view(torch.bfloat16).cuda())
        part = ofl.bf16_bits_to_f32(ofl.block_gemm(
            xq.cpu().view(torch.uint8).numpy(), xs.cpu().view(torch.int16).numpy().view(np.uint16),
            wr, wsr))
        acc = part if acc is None else (acc + part).astype(np.float32)
    want = ofl.f32_to_bf16_bits(acc)
    _assert_close(torch.from_numpy(res[0]["fused_0"].view(np.int16)).view(torch.bfloat16),
                  torch.from_numpy(want.view(np.int16)).view(torch.bfloat16), "oracle",
                  of_max=2.0 ** -7)
    assert (res[0]["fused_0"] == want).mean() >= 0.99
