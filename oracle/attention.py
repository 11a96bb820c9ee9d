"""torch fp32 restatement of the reference FP8 attention kernels (test infrastructure only).

Decode follows nanovllm/kernels/fp8_attention.py:88-171 (``fp8_paged_attention_decode_kernel``):
  * grid (seq, q head); kv head = head // (Hq // KVH) (:104-105);
  * positions ``< context_lens[b]`` over ``max_num_blocks = block_tables.shape[1]`` table columns
    (:123-136) -- positions at or beyond ``max_num_blocks * block_size`` are never visited;
  * scores = q . k * softmax_scale in fp32, online softmax, ``out = acc / max(s, 1e-10)`` cast to
    fp16 and stored into the bf16 output (:169-171), so ``context_len == 0`` gives 0.

Prefill follows nanovllm/kernels/fp8_attention.py:209-312 (``fp8_paged_attention_prefill_kernel``):
  * per sequence s: q rows ``cu_q[s]..cu_q[s+1]``, ``nk = cu_k[s+1]-cu_k[s]``,
    ``computed = nk - nq`` (:229-237);
  * contiguous branch (:254-278): K/V rows ``cu_k[s]..cu_k[s+1]`` of ``[Tk, KVH, D]`` tensors;
  * paged branch (:279-308): key position j lives in ``cache[block_tables[s, j // BS], j % BS]``,
    only the first ``max_num_blocks`` table columns are visited;
  * causal mask ``kv <= q + computed`` together with ``kv < nk`` (:267-268, :297-298);
  * ``out = where(l > 0, acc / l, 0)`` cast to fp16 and stored into the bf16 output (:310-312).

Both are computed in fp32 from the exactly-widened e4m3 values (the reference upcasts the FP8
loads with ``.to(tl.float32)``); optional per-(slot, kv-head) fp32 scales multiply K/V (the scaled
extension).  Inputs are torch CPU tensors; caches are uint8 (raw e4m3 bytes) or float8_e4m3fn.
"""
from __future__ import annotations

import numpy as np
import torch

from . import e4m3

_TABLE = None


def _lut() -> torch.Tensor:
    global _TABLE
    if _TABLE is None:
        _TABLE = torch.from_numpy(e4m3.to_f32(np.arange(256, dtype=np.uint8)))
    return _TABLE


def widen(codes: torch.Tensor) -> torch.Tensor:
    """e4m3 bytes (uint8 or float8_e4m3fn tensor) -> float32, exactly."""
    if codes.dtype == torch.float8_e4m3fn:
        codes = codes.view(torch.uint8)
    return _lut()[codes.long()]


def _finish(o: torch.Tensor) -> torch.Tensor:
    # fp32 -> fp16 (the reference's .to(tl.float16)) -> bf16 (store into the bf16 output buffer)
    return o.to(torch.float16).to(torch.bfloat16)


def _gather_paged(cache: torch.Tensor, scale: torch.Tensor | None, table_row: torch.Tensor,
                  n: int) -> torch.Tensor:
    """First n key positions of one sequence from a paged cache -> fp32 [n, KVH, D]."""
    nb, bs, kvh, d = cache.shape
    nblk = (n + bs - 1) // bs
    blocks = table_row[:nblk].long()
    x = widen(cache[blocks].reshape(nblk * bs, kvh, d)[:n])
    if scale is not None:
        s = scale.reshape(nb, bs, kvh)[blocks].reshape(nblk * bs, kvh)[:n]
        x = x * s.float().unsqueeze(-1)
    return x


def decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
           block_tables: torch.Tensor, context_lens: torch.Tensor, softmax_scale: float,
           k_scale: torch.Tensor | None = None, v_scale: torch.Tensor | None = None,
           return_fp32: bool = False) -> torch.Tensor:
    """Paged single-query decode.  q ``[B, Hq, D]`` -> out ``[B, Hq, D]`` bf16."""
    bsz, hq, d = q.shape
    nb, bs, kvh, _ = k_cache.shape
    g = hq // kvh
    max_blocks = block_tables.shape[1]
    out = torch.zeros(bsz, hq, d, dtype=torch.float32)
    for b in range(bsz):
        n = min(max(int(context_lens[b]), 0), max_blocks * bs)
        if n == 0:
            continue
        kf = _gather_paged(k_cache, k_scale, block_tables[b], n)   # [n, KVH, D]
        vf = _gather_paged(v_cache, v_scale, block_tables[b], n)
        qb = q[b].float().reshape(kvh, g, d)
        s = torch.einsum("hgd,nhd->hgn", qb, kf) * softmax_scale
        p = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("hgn,nhd->hgd", p, vf).reshape(hq, d)
    return out if return_fp32 else _finish(out)


def prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_tables: torch.Tensor | None,
            cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor, softmax_scale: float,
            k_scale: torch.Tensor | None = None, v_scale: torch.Tensor | None = None,
            return_fp32: bool = False) -> torch.Tensor:
    """Varlen causal attention.  q ``[Tq, Hq, D]``; k/v either paged caches
    ``[nb, BS, KVH, D]`` (with ``block_tables``) or contiguous ``[Tk, KVH, D]`` (``None``)."""
    tq, hq, d = q.shape
    kvh = k.shape[2] if block_tables is not None else k.shape[1]
    g = hq // kvh
    out = torch.zeros(tq, hq, d, dtype=torch.float32)
    cq = [int(x) for x in cu_seqlens_q]
    ck = [int(x) for x in cu_seqlens_k]
    for s in range(len(cq) - 1):
        q0, nq = cq[s], cq[s + 1] - cq[s]
        k0, nk = ck[s], ck[s + 1] - ck[s]
        if nq <= 0:
            continue
        computed = nk - nq
        if block_tables is not None:
            bs = k.shape[1]
            n = max(min(nk, block_tables.shape[1] * bs), 0)
            kf = _gather_paged(k, k_scale, block_tables[s], n) if n else None
            vf = _gather_paged(v, v_scale, block_tables[s], n) if n else None
        else:
            n = max(nk, 0)
            kf = widen(k[k0:k0 + n]) if n else None
            vf = widen(v[k0:k0 + n]) if n else None
            if n and k_scale is not None:
                kf = kf * k_scale[k0:k0 + n].float().unsqueeze(-1)
            if n and v_scale is not None:
                vf = vf * v_scale[k0:k0 + n].float().unsqueeze(-1)
        if n == 0:
            continue
        qs = q[q0:q0 + nq].float().reshape(nq, kvh, g, d)
        sc = torch.einsum("ihgd,jhd->hgij", qs, kf) * softmax_scale        # [KVH, G, nq, n]
        i = torch.arange(nq).unsqueeze(1)
        j = torch.arange(n).unsqueeze(0)
        allowed = j <= i + computed                                          # [nq, n]
        sc = sc.masked_fill(~allowed, float("-inf"))
        row_any = allowed.any(dim=1)                                         # rows with l > 0
        p = torch.softmax(sc, dim=-1)
        p = torch.where(row_any.view(1, 1, nq, 1), p, torch.zeros_like(p))
        o = torch.einsum("hgij,jhd->ihgd", p, vf).reshape(nq, hq, d)
        out[q0:q0 + nq] = o
    return out if return_fp32 else _finish(out)
