"""fp8attn_decode_noalloc (no counterpart in the reference): the decode entry point whose split-KV
scratch is the library's static device array.  Called through the C-ABI and compared with
fp8attn_decode (caller workspace) within the attention tolerance, on two consecutive calls so that
the second call meets the scratch the first one left behind.  The file name sorts last so the
suite also runs it after every other test."""
import ctypes

import pytest
import torch

from helpers import assert_close

pytestmark = pytest.mark.gpu


def _noalloc(c, out):
    from nanovllm_b200 import _lib
    nb, bs, kvh, hd = c.k_cache.shape
    return _lib.lib.fp8attn_decode_noalloc(
        out.data_ptr(), c.q.data_ptr(), c.q.stride(0), c.k_cache.data_ptr(), c.v_cache.data_ptr(),
        None, None, c.block_tables.data_ptr(), c.block_tables.stride(0), c.block_tables.shape[1],
        c.context_lens.data_ptr(), c.q.shape[0], c.q.shape[1], kvh, hd, nb, bs,
        ctypes.c_float(c.scale), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("config", ["config1", "config2"])
def test_noalloc_matches_workspace_entry(config):
    from nanovllm_b200 import _lib, fp8_decode_attention, workloads
    c = getattr(workloads, config)("cuda")
    ref = fp8_decode_attention(c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale)
    for call in range(2):
        out = torch.full_like(c.q, float("nan"))
        _lib.check(_noalloc(c, out))
        torch.cuda.synchronize()
        assert_close(out, ref, what=f"{config} no-alloc call {call}")


def test_noalloc_rejects_shapes_beyond_its_scratch():
    # GQA 16 keeps 16 partial rows per work item: more than the static scratch holds
    from nanovllm_b200 import _lib, workloads
    c = workloads.decode_case(8, 64, 4, 64, 300, seed=3, device="cuda", block_size=64)
    need = _lib.lib.fp8attn_workspace_bytes(8, 64, 4, 1)
    assert need > _lib.NOALLOC_SCRATCH_BYTES
    out = torch.zeros_like(c.q)
    rc = _noalloc(c, out)
    assert rc == _lib.EWORKSPACE
    msg = _lib.lib.fp8attn_last_error().decode()
    assert str(need) in msg and str(_lib.NOALLOC_SCRATCH_BYTES) in msg
    torch.cuda.synchronize()
    assert torch.all(out == 0)
