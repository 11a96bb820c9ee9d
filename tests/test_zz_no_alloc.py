"""fp8attn_decode_noalloc (no counterpart in the reference): the decode entry point whose split-KV
scratch is the library's static device array, for hosts that cannot allocate device memory on the
decode path.  Called through the C-ABI and compared with fp8attn_decode (caller workspace): both
run the same kernels with the same plan, so the outputs must be bit-identical, on consecutive calls
(the later ones meet the scratch the earlier ones left behind).  After every call the scratch's
error word must read 0, and the device's free memory must not move across calls.  The file name
sorts last so the suite also runs it after every other test."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc(c, out):
    from nanovllm_b200 import _lib
    nb, bs, kvh, hd = c.k_cache.shape
    return _lib.lib.fp8attn_decode_noalloc(
        out.data_ptr(), c.q.data_ptr(), c.q.stride(0), c.k_cache.data_ptr(), c.v_cache.data_ptr(),
        None, None, c.block_tables.data_ptr(), c.block_tables.stride(0), c.block_tables.shape[1],
        c.context_lens.data_ptr(), c.q.shape[0], c.q.shape[1], kvh, hd, nb, bs,
        ctypes.c_float(c.scale), torch.cuda.current_stream().cuda_stream)


def _scratch_error():
    from nanovllm_b200 import _lib
    host = torch.full((1,), -1, dtype=torch.int32).pin_memory()
    _lib.check(_lib.lib.fp8attn_noalloc_read_error(host.data_ptr(), 0,
                                                   torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return int(host[0])


@pytest.mark.parametrize("config", ["config1", "config2"])
def test_noalloc_matches_workspace_entry(config):
    from nanovllm_b200 import _lib, fp8_decode_attention, workloads
    c = getattr(workloads, config)("cuda")
    ref = fp8_decode_attention(c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale)
    outs = [torch.full_like(c.q, float("nan")) for _ in range(3)]
    torch.cuda.synchronize()
    free = []
    errors = []
    for out in outs:  # nothing in this loop allocates device memory but the calls under test
        free.append(torch.cuda.mem_get_info()[0])
        _lib.check(_noalloc(c, out))
        torch.cuda.synchronize()
        errors.append(_scratch_error())
    free.append(torch.cuda.mem_get_info()[0])
    assert errors == [0, 0, 0], errors
    # the first call may load the library's module on this device; later calls allocate nothing
    assert free[1] == free[2] == free[3], free
    for call, out in enumerate(outs):
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), \
            f"{config} no-alloc call {call} differs from fp8attn_decode"


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
