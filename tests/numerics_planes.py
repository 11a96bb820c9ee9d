"""Numerics of the tensor-core operand planes of the prefill engine (design check, CPU).

q and P enter the e4m3 tensor-core products either as one e4m3 plane (4 significant bits) or as
hi + lo planes (hi = e4m3(x), lo = e4m3(x - hi): about 8 bits); P can also enter an f16 product
(11 bits) against V converted exactly to f16.  This script emulates these combinations on a
benchmark configuration -- exact e4m3 casts of q (after the engine's per-row power-of-two scale)
and e4m3 or f16 casts of P = 16 2^(s - m), everything else in fp32, the output through fp16 to
bf16 as in the reference (nanovllm/kernels/fp8_attention.py:310-312) -- and prints the error
against the fp32 reference with the tests' tolerance 2e-2 + 1e-2 |ref|.

    python tests/numerics_planes.py config3
"""
from __future__ import annotations

import os
import sys
import time

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "my-nano-vllm_b200")]

E4 = torch.float8_e4m3fn


def _e4(x):
    return x.clamp(-448, 448).to(E4).float()


def _planes(x, n):
    if n == "f16":
        return x.to(torch.float16).float()
    hi = _e4(x)
    return hi + _e4(x - hi) if n == 2 else hi


def run(c, q_planes: int, p_planes: int):
    """Max abs error, max error / tolerance and mean abs error of the emulated engine."""
    q = c.q.float()
    hq, kvh = q.shape[1], c.k.shape[2]
    g = hq // kvh
    amax = q.abs().amax(-1, keepdim=True)
    s = torch.exp2(torch.floor(torch.log2(amax.clamp_min(1e-30))) - 7)  # |q| / s < 256
    qe = _planes(q / s, q_planes) * s
    cq, ck = c.cu_seqlens_q.tolist(), c.cu_seqlens_k.tolist()
    bs = c.k.shape[1]
    refs, outs = [], []
    for si in range(len(cq) - 1):
        nq, nk = cq[si + 1] - cq[si], ck[si + 1] - ck[si]
        blocks = c.block_tables[si, :(nk + bs - 1) // bs].long()
        k = c.k[blocks].float().reshape(-1, kvh, 128)[:nk].repeat_interleave(g, 1)
        v = c.v[blocks].float().reshape(-1, kvh, 128)[:nk].repeat_interleave(g, 1)
        mask = torch.arange(nk)[None, :] <= torch.arange(nq)[:, None] + (nk - nq)
        for variant, qq in (("ref", q), ("emu", qe)):
            sc = torch.einsum("qhd,khd->hqk", qq[cq[si]:cq[si + 1]], k) * c.scale * 1.4426950408889634
            sc = sc.masked_fill(~mask[None], float("-inf"))
            p = 16 * torch.exp2(sc - sc.amax(-1, keepdim=True))
            l = p.sum(-1, keepdim=True)
            pe = p if variant == "ref" else _planes(p, p_planes)
            o = torch.einsum("hqk,khd->qhd", pe, v) / l.permute(1, 0, 2)
            (refs if variant == "ref" else outs).append(o)
    ref = torch.cat(refs)
    out = torch.cat(outs).to(torch.float16).to(torch.bfloat16).float()
    err = (out - ref).abs()
    return float(err.max()), float((err / (2e-2 + 1e-2 * ref.abs())).max()), float(err.mean())


def main(name: str) -> None:
    from nanovllm_b200 import workloads
    torch.set_num_threads(os.cpu_count() or 1)
    c = getattr(workloads, name)("cpu")
    for qp, pp in ((2, "f16"), (2, 2), (1, 2), (2, 1), (1, 1)):
        t = time.time()
        mx, ratio, mean = run(c, qp, pp)
        print(f"{name}: q planes {qp}, P planes {pp}: max abs err {mx:.3e}, max err / tolerance "
              f"{ratio:.3f}, mean abs err {mean:.2e} ({time.time() - t:.0f} s)", flush=True)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "config3")
