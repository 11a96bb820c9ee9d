"""Generate tests/golden/qk_epilogue.npz from the reference's own attention-input epilogue.

Run on a machine with a CUDA GPU and the reference installed under baseline/_ref (it is NOT
needed at test time):

    python tests/golden/make_golden_qk.py OUT_DIR

On seeded bf16 inputs it runs the reference's compiled RMSNorm (nanovllm/layers/layernorm.py:16-26)
on q and k, its compiled RotaryEmbedding (nanovllm/layers/rotary_embedding.py:37-47) and its Triton
store_kvcache (nanovllm/layers/attention.py:11-40), as Qwen3Attention.forward chains them
(nanovllm/models/qwen3.py:102-111), and writes the inputs and the outputs (rotated q and k, and the
K/V cache bytes) to OUT_DIR/qk_epilogue.npz; of the cos/sin table it keeps the rows of the tokens'
positions (cos_sin_rows[i] is the row of positions[i]).  The compiled functions are first called on another
shape, as in the engine, so the recorded outputs come from their dynamic-shape kernels.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def main(out_dir: str) -> None:
    sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
    import torch
    from nanovllm.layers.attention import store_kvcache
    from nanovllm.layers.layernorm import RMSNorm
    from nanovllm.layers.rotary_embedding import get_rope

    bits = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    n, hq, kvh, bs = 96, 8, 2, 16
    g = torch.Generator().manual_seed(20261202)
    qkv = (torch.randn(n, (hq + 2 * kvh) * 128, generator=g) * 1.5).to(torch.bfloat16)
    qw = (torch.randn(128, generator=g) * 0.2 + 1).to(torch.bfloat16)
    kw = (torch.randn(128, generator=g) * 0.2 + 1).to(torch.bfloat16)
    pos = torch.randint(0, 4096, (n,), generator=g)
    nb = n // bs + 2
    slots = torch.randperm(nb * bs, generator=g)[:n].to(torch.int32)
    slots[::7] = -1
    rope = get_rope(128, 128, 4096, 1000000.0).to("cuda")
    qn, kn = RMSNorm(128).cuda(), RMSNorm(128).cuda()
    with torch.no_grad():
        qn.weight.copy_(qw.float())
        kn.weight.copy_(kw.float())
    qn, kn = qn.to(torch.bfloat16), kn.to(torch.bfloat16)
    x = qkv.cuda()
    q, k, v = x.split([hq * 128, kvh * 128, kvh * 128], dim=-1)
    with torch.no_grad():
        rope(pos[:5].cuda(), qn(q[:5].reshape(-1, hq, 128)), kn(k[:5].reshape(-1, kvh, 128)))
        q3, k3 = rope(pos.cuda(), qn(q.reshape(-1, hq, 128)), kn(k.reshape(-1, kvh, 128)))
    kc = torch.full((nb, bs, kvh, 128), 0x55, dtype=torch.uint8, device="cuda")
    vc = torch.full_like(kc, 0x55)
    store_kvcache(k3, v.reshape(-1, kvh, 128), kc.view(torch.float8_e4m3fn),
                  vc.view(torch.float8_e4m3fn), slots.cuda())
    torch.cuda.synchronize()
    np.savez_compressed(
        os.path.join(out_dir, "qk_epilogue.npz"), qkv=bits(qkv), q_weight=bits(qw),
        k_weight=bits(kw), positions=pos.numpy(), slots=slots.numpy(),
        cos_sin_rows=rope.cos_sin_cache[pos.cuda()].reshape(n, 128).cpu().numpy(), hq=hq, kvh=kvh,
        eps=1e-6, q=bits(q3),
        k=bits(k3), k_cache=kc.cpu().numpy(), v_cache=vc.cpu().numpy())


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
