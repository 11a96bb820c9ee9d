"""Benchmark of the FP8 PagedAttention hot path (BASELINE.json metric).

Headline workload (a "step"): one paged FP8 decode call over BASELINE config 5 -- Qwen3-32B heads
(64 q / 8 kv, head_dim 128), 64 sequences at context 32768, block 256, about 2.1M cached tokens --
split by kv-head group over the N GPUs of one node, as the reference's tensor-parallel head split
does: rank r holds kv heads [r*8/N, (r+1)*8/N) and their q heads, with the same lengths and block
tables on every rank and no collective in the path.  The total work is fixed, so ``scaling`` is
"strong"; ``value`` is the algorithmic HBM throughput of the whole job (TB/s): the sum over ranks
of every visible K and V byte once plus q, out, block tables and lengths, divided by the device
time of the step (max over ranks).  The KV working set (4.3 GB at N=1, 0.54 GB per GPU at N=8) is
far larger than the 126 MB L2, so no flush is needed between steps.

Secondary figures on the N=1 line (outside the headline's timed region): config 2 (large-batch
decode), config 1 (the small reference decode case), config 3 (chunked prefill, TFLOP/s, and its
K/V store) and config 4 (mixed spec-verify + prefill call), each with its roofline; and
``reference_gpu``: the reference's own Triton kernels (installed unmodified under baseline/_ref)
timed on the same inputs and the same GPU, next to ours.

``--impl reference`` times the reference algorithm on the host cores instead (the CPU oracle, a
torch fp32 restatement of fp8_paged_attention_decode_kernel) on a bounded sample of the headline
workload; it does not load this repository's CUDA library.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "my-nano-vllm_b200")
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
sys.path.insert(0, PKG)
sys.path.insert(0, ROOT)

METRIC = "FP8 paged decode HBM TB/s (% of 8 TB/s); varlen prefill TFLOP/s (% peak)"
WORKLOAD = ("config5: FP8 paged decode, Qwen3-32B heads (64q/8kv, d128), 64 seqs x 32768 ctx, "
            "block 256, kv-head groups split over the GPUs")


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return (float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


def _traffic(key: str):
    """DRAM bytes (read + write) per algorithmic byte of a kernel on a workload, from the ncu
    capture summarised in profiles/ (scaled to the launch by the caller)."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f).get(key)
    return None


class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons while the timed region runs: NVML
    polled every 0.5 ms (the timed region is a few ms), or nvidia-smi every 200 ms without NVML."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}

    def __init__(self, index: int):
        self.index = index
        self.samples = []  # (sm_mhz, max_mhz, set of reasons)
        self._stop = threading.Event()
        self._t = None
        self._nvml = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            h = None
            try:  # the CUDA device (CUDA_VISIBLE_DEVICES may renumber) by its PCI address
                pr = torch.cuda.get_device_properties(index)
                bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
                h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self._nvml = (pynvml, h)
        except Exception:
            self._nvml = None

    def _run_nvml(self):
        nv, h = self._nvml
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons",
                              getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons", None))
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                bits = get_reasons(h) if get_reasons else 0
                self.samples.append((float(sm), float(mx),
                                     {n for n, b in self.REASON_BITS.items() if bits & b}))
            except Exception:
                pass
            self._stop.wait(0.0005)

    def _run_smi(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.index}",
                                      f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits"],
                                     capture_output=True, text=True, timeout=5).stdout.strip()
                if out:
                    f = [x.strip() for x in out.split(",")]
                    self.samples.append((float(f[1]), float(f[2]),
                                         {n for n, v in zip(names, f[5:9]) if v.lower() == "active"}))
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run_nvml if self._nvml else self._run_smi,
                                   daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = set()
        for _, _, r in self.samples:
            reasons |= r
        return {"sm_mhz": statistics.median(x[0] for x in self.samples),
                "sm_max_mhz": max(x[1] for x in self.samples), "reasons": sorted(reasons),
                "samples": len(self.samples), "source": "nvml" if self._nvml else "nvidia-smi"}


# ------------------------------------------------------------------------------ ranks
def _dist_init():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def _reduce(x: float, world: int, op: str) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _load_workloads():
    """The seeded input generator, loaded without importing the ``nanovllm_b200`` package's entry
    points (so the reference leg never maps the CUDA library)."""
    import nanovllm_b200.workloads as w  # the package __init__ loads nothing
    return w


# ------------------------------------------------------------------------------ CPU leg
def cpu_baseline(case, max_seconds: float = 20.0, label: str = "config-5"):
    """Time the CPU oracle (torch fp32 restatement of the reference decode) on a bounded sample
    of the same workload: whole sequences in order until ~max_seconds of CPU work."""
    import torch
    from oracle import attention as oatt
    torch.set_num_threads(os.cpu_count() or 1)
    q, kc, vc, bt, ctx = (case.q.cpu(), case.k_cache, case.v_cache, case.block_tables.cpu(),
                          case.context_lens.cpu())
    done_bytes, t_total, n = 0, 0.0, 0
    kvh, d = kc.shape[2], kc.shape[3]
    bs = kc.shape[1]
    while n < q.shape[0] and t_total < max_seconds:
        b = n
        L = int(ctx[b])
        nblk = (L + bs - 1) // bs
        blocks = bt[b, :nblk].long()
        kb = kc[blocks.to(kc.device)].cpu()          # the sequence's blocks, host copy
        vb = vc[blocks.to(vc.device)].cpu()
        sub_bt = torch.arange(nblk, dtype=torch.int32).unsqueeze(0)
        t0 = time.perf_counter()
        oatt.decode(q[b:b + 1], kb, vb, sub_bt, ctx[b:b + 1], case.scale)
        t_total += time.perf_counter() - t0
        done_bytes += L * kvh * d * 2 + 2 * q.shape[1] * d * 2 + 4 * nblk + 4
        n += 1
    return {"value": done_bytes / t_total / 1e12, "unit": "TB/s",
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"first {n} of {q.shape[0]} {label} sequences ({done_bytes / 1e6:.1f} MB "
                      f"of K/V), torch fp32 oracle, {t_total:.1f} s"}


def run_reference(args, world, rank):
    """--impl reference: the reference algorithm on the host cores (the CPU oracle port; the
    reference's own path is Triton GPU code with no CPU implementation).  Rank 0 alone runs it;
    every step is a bounded sample of the headline workload.  This repository's CUDA library is
    never loaded here."""
    if rank != 0:
        return
    import torch
    workloads = _load_workloads()
    case = workloads.config5("cpu", gpus=1, rank=0, batch=8)
    per_step = max(0.5, min(3.0, args.cpu_seconds / max(1, args.steps)))
    for _ in range(args.warmup):
        cpu_baseline(case, max_seconds=0.2)
    steps = [cpu_baseline(case, max_seconds=per_step) for _ in range(args.steps)]
    assert "nanovllm_b200._lib" not in sys.modules, "the reference leg must not load libfp8attn.so"
    value = statistics.median(s["value"] for s in steps)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s",
            "n_gpus": world, "steps": len(steps), "warmup": args.warmup,
            "ms_per_step": None, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "parallelism": f"kv-head-split{world}",
                       "note": "host cores; each step a bounded sample of whole config-5 "
                               "sequences (see cpu_baseline.sample)"},
            "cpu_baseline": dict(steps[-1], value=value),
            "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "library_loaded": False}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ GPU helpers
def _flush_l2(buf):
    buf.add_(1)  # writes 256 MB, twice the 126 MB L2


def _time_calls(fn, iters=10, warm=3, flush=None):
    """Median CUDA-event time (ms) of ``fn`` on the current stream, L2 flushed before each call
    when ``flush`` is given."""
    import torch
    for _ in range(warm):
        fn()
    ts = []
    for _ in range(iters):
        if flush is not None:
            _flush_l2(flush)
        # keep the GPU busy while the host enqueues the call, so that the events bracket device
        # work only (not the host-side launch of a short call)
        torch.cuda._sleep(200000)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def _fp8_peak(dev):
    """Dense e4m3 GEMM rate of this GPU (cuBLASLt through torch._scaled_mm, 8192^3, best of 10):
    the tensor roofline of the prefill, measured here because the driver's file holds bf16 only."""
    import torch
    try:
        n = 8192
        a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn).t()
        one = torch.ones((), device=dev)
        f = lambda: torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        f()
        ms = min(_time_calls(f, iters=1, warm=0) for _ in range(10))
        return 2 * n ** 3 / (ms * 1e-3) / 1e12
    except Exception:
        return None


def _reference_module():
    """The reference's own entry points from its unmodified install under baseline/_ref, or the
    reason they cannot be loaded."""
    if not os.path.isdir(os.path.join(REF_DIR, "nanovllm")):
        return None, "baseline/_ref is not installed"
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        from nanovllm.kernels import fp8_attention as rk
        from nanovllm.layers import attention as ra
        entries = {"decode": rk.fp8_decode_attention, "prefill": rk.fp8_prefill_attention,
                   "store": ra.store_kvcache}
    except Exception as e:  # pragma: no cover - depends on the box
        return None, f"{type(e).__name__}: {e}"
    try:
        from nanovllm.kernels import fp8_linear as rl
        entries["linear"] = rl.fp8_block_linear
    except Exception:  # pragma: no cover - older reference without the FP8 linear layer
        pass
    return entries, None


def _maxdiff(a, b):
    return float((a.float() - b.float()).abs().max())


PARTS = ("config2", "config1", "config3", "store", "config4", "epilogue", "fp8linear")
# half of a part, for profile captures that want one launch shape only
SUBPARTS = ("fp8linear_decode", "fp8linear_prefill")


def _store_sets(c, nsets, dev):
    """``nsets`` independent copies of config 3's store inputs (new K/V rows drawn from their own
    seeds, the same slot mapping, each set with its own caches): back-to-back stores over them
    touch more than the L2 holds, so each call streams from HBM like a fresh one."""
    import torch
    sets = []
    n, kvh = c.new_k.shape[0], c.new_k.shape[1]
    for i in range(nsets):
        g = torch.Generator(device=dev).manual_seed(1000 + i)
        k = torch.randn(n, kvh, 128, generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn(n, kvh, 128, generator=g, device=dev).to(torch.bfloat16)
        sets.append((k, v, torch.empty_like(c.k), torch.empty_like(c.v), c.slot_mapping))
    return sets


def _time_graph_calls(fn_all, ncalls, iters=20, warm=3):
    """Per-call device time (ms) of a CUDA graph of ``ncalls`` back-to-back calls: the median
    over replays of the graph's CUDA-event time, divided by ``ncalls``.  Short calls (~10 us) are
    timed this way because a single call is near the event timer's resolution."""
    import torch
    fn_all()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn_all()
    ms = _time_calls(graph.replay, iters=iters, warm=warm) / ncalls
    del graph
    return ms


def secondary(dev, peaks, with_reference: bool, only=None):
    """Configs 2, 1, 3 (+ store) and 4 on one GPU, each timed with CUDA events after warm-up, and
    the reference's Triton kernels on the same inputs where ``with_reference``.  ``only`` names a
    subset of PARTS (profile captures run one part by itself)."""
    import torch
    from nanovllm_b200 import fp8_decode_attention, fp8_prefill_attention, store_kvcache
    workloads = _load_workloads()
    parts = set(only or PARTS)
    hbm_peak, bf16_peak = peaks[0], peaks[1]
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    ref, ref_err = _reference_module() if with_reference else (None, "not requested")
    out = {}
    refgpu = {"source": "baseline/_ref (unmodified reference, stock entry points), same inputs, "
                        "same GPU, CUDA events, median"}
    if ref is None:
        refgpu["unavailable"] = ref_err

    def ref_time(name, fn, ours_ms, ours_out=None, iters=5, warm=2, flush_l2=None, ncalls=None):
        if ref is None:
            return
        try:
            if ncalls is not None:
                r_ms = _time_graph_calls(fn, ncalls)
            else:
                r_ms = _time_calls(fn, iters=iters, warm=warm, flush=flush_l2)
            entry = {"ms": r_ms, "ours_ms": ours_ms, "speedup": r_ms / ours_ms}
            if ours_out is not None:
                entry["max_abs_diff_vs_ours"] = _maxdiff(fn(), ours_out)
            refgpu[name] = entry
        except Exception as e:  # pragma: no cover
            refgpu[name] = {"unavailable": f"{type(e).__name__}: {e}"}

    fp8_peak, fp8_kind = None, "measured e4m3 GEMM (torch._scaled_mm)"
    lin_decode = bool(parts & {"fp8linear", "fp8linear_decode"})
    lin_prefill = bool(parts & {"fp8linear", "fp8linear_prefill"})
    if "config3" in parts or lin_prefill:
        fp8_peak = _fp8_peak(dev)
    if fp8_peak is None:
        fp8_peak, fp8_kind = 2 * bf16_peak, "2 x measured bf16 GEMM"

    # ---- decode: config 2 (HBM bound, 1.2 GB) and config 1 (9 MB, latency bound)
    for name, make, l2 in (("config2", workloads.config2, "inputs larger than L2"),
                           ("config1", workloads.config1, "flushed before each call")):
        if name not in parts:
            continue
        c = make(dev)
        args = (c.q, c.k_cache, c.v_cache, c.block_tables, c.context_lens, c.scale)
        fl = flush if name == "config1" else None
        ms = _time_calls(lambda: fp8_decode_attention(*args), iters=20, warm=5, flush=fl)
        nbytes = c.kv_bytes()
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"ms": ms, "tb_s": gbs / 1e3, "bytes": nbytes, "l2": l2,
                     "tokens_per_s": c.q.shape[0] / (ms * 1e-3),
                     "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak,
                                  "unit": "GB/s", "frac": gbs / hbm_peak}}
        if ref is not None:
            ours = fp8_decode_attention(*args)
            ref_time(f"decode_{name}", lambda: ref["decode"](*args), ms, ours, flush_l2=fl)
        del c, args
        torch.cuda.empty_cache()

    # ---- config 3: chunked prefill (tensor bound) and its K/V store (HBM bound)
    if parts & {"config3", "store"}:
        c = workloads.config3(dev)
        store_kvcache(c.new_k, c.new_v, c.k, c.v, c.slot_mapping)
        torch.cuda.synchronize()
    if "store" in parts:
        n = c.new_k.shape[0]
        store_bytes = n * (2 * 8 * 128 * 2 + 2 * 8 * 128 + 4)
        sets = _store_sets(c, 8, dev)
        st_ms = _time_graph_calls(lambda: [store_kvcache(*x) for x in sets], len(sets))
        sgbs = store_bytes / (st_ms * 1e-3) / 1e9
        out["config3_store"] = {
            "ms": st_ms, "gbs": sgbs, "rows": n, "bytes": store_bytes,
            "timing": "CUDA graph of 8 back-to-back calls on 8 independent input sets "
                      "(300 MB in all, more than L2), per-call time",
            "roofline": {"bound": "hbm", "achieved": sgbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": sgbs / hbm_peak}}
        if ref is not None:
            ref_sets = [(k, v, kc.clone(), vc.clone(), sl) for k, v, kc, vc, sl in sets]
            ref_time("store_config3", lambda: [ref["store"](*x) for x in ref_sets], st_ms,
                     ncalls=len(ref_sets))
            if "store_config3" in refgpu and "ms" in refgpu["store_config3"]:
                refgpu["store_config3"]["bytes_equal_to_ours"] = all(
                    torch.equal(a[2].view(torch.uint8), b[2].view(torch.uint8)) and
                    torch.equal(a[3].view(torch.uint8), b[3].view(torch.uint8))
                    for a, b in zip(sets, ref_sets))
            del ref_sets
        del sets
        torch.cuda.empty_cache()
    if "config3" in parts:
        flops = c.causal_flops()
        pf = lambda: fp8_prefill_attention(
            c.q, c.k, c.v, block_tables=c.block_tables, cu_seqlens_q=c.cu_seqlens_q,
            cu_seqlens_k=c.cu_seqlens_k, max_seqlen_q=c.max_seqlen_q,
            max_seqlen_k=c.max_seqlen_k, softmax_scale=c.scale)
        pf_ms = _time_calls(pf, flush=flush)
        tflops = flops / (pf_ms * 1e-3) / 1e12
        out["config3_prefill"] = {
            "workload": "16 seqs, new U[128,512], cached prefix U[0,3584], Qwen3-8B heads, paged "
                        "block 256", "ms": pf_ms, "tflops": tflops, "causal_flops": flops,
            "tokens_per_s": int(c.q.shape[0]) / (pf_ms * 1e-3), "l2": "flushed before each call",
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": fp8_peak,
                         "unit": "TFLOP/s", "frac": tflops / fp8_peak, "peak_kind": fp8_kind,
                         "frac_of_bf16_sustained": tflops / peaks[2]}}
        if ref is not None:
            ours = pf()
            ref_time("prefill_config3", lambda: ref["prefill"](
                c.q, c.k, c.v, block_tables=c.block_tables, cu_seqlens_q=c.cu_seqlens_q,
                cu_seqlens_k=c.cu_seqlens_k, max_seqlen_q=c.max_seqlen_q,
                max_seqlen_k=c.max_seqlen_k, softmax_scale=c.scale), pf_ms, ours, iters=3,
                warm=1, flush_l2=flush)
    if parts & {"config3", "store"}:
        del c
        torch.cuda.empty_cache()

    # ---- config 4: one mixed call (192 spec-verify sequences of 5 rows + 2 fresh 512-row chunks)
    if "config4" in parts:
        c = workloads.config4(dev)
        store_kvcache(c.new_k, c.new_v, c.k, c.v, c.slot_mapping)
        cq, ck = c.cu_seqlens_q.tolist(), c.cu_seqlens_k.tolist()
        nks = [ck[i + 1] - ck[i] for i in range(len(ck) - 1)]
        nqs = [cq[i + 1] - cq[i] for i in range(len(cq) - 1)]
        spec_bytes = sum(nk * 8 * 128 * 2 + 2 * nq * 32 * 128 * 2
                         for nk, nq in zip(nks, nqs) if nq <= 16)
        mixed = lambda: fp8_prefill_attention(
            c.q, c.k, c.v, block_tables=c.block_tables, cu_seqlens_q=c.cu_seqlens_q,
            cu_seqlens_k=c.cu_seqlens_k, max_seqlen_q=c.max_seqlen_q,
            max_seqlen_k=c.max_seqlen_k, softmax_scale=c.scale)
        m_ms = _time_calls(mixed, iters=10, warm=3)
        gbs = spec_bytes / (m_ms * 1e-3) / 1e9
        out["config4_mixed"] = {
            "workload": "192 spec-verify seqs (1+4 rows, ctx U[1024,8187]) + 2 fresh 512-token "
                        "chunks, one prefill call, Qwen3-8B heads, paged block 256",
            "ms": m_ms, "tokens_per_s": int(c.q.shape[0]) / (m_ms * 1e-3),
            "spec_bytes": spec_bytes, "l2": "inputs larger than L2",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": gbs / hbm_peak,
                         "note": "spec-part bytes over the whole call's time (the two fresh "
                                 "chunks run in the same call)"}}
        if ref is not None:
            ours = mixed()
            ref_time("mixed_config4", lambda: ref["prefill"](
                c.q, c.k, c.v, block_tables=c.block_tables, cu_seqlens_q=c.cu_seqlens_q,
                cu_seqlens_k=c.cu_seqlens_k, max_seqlen_q=c.max_seqlen_q,
                max_seqlen_k=c.max_seqlen_k, softmax_scale=c.scale), m_ms, ours, iters=2,
                warm=1)
        del c
        torch.cuda.empty_cache()
    # ---- the fused attention-input epilogue (q/k norm + rope + K/V store) on config 3's new rows
    if "epilogue" in parts:
        from nanovllm_b200.qk_epilogue import qk_norm_rope_store
        c = workloads.config3(dev)
        n, hq, kvh = c.q.shape[0], 32, 8
        g = torch.Generator(device=dev).manual_seed(77)
        qkvs = [torch.randn(n, (hq + 2 * kvh) * 128, generator=g, device=dev).to(torch.bfloat16)
                for _ in range(8)]
        qw = (torch.randn(128, generator=g, device=dev) * 0.2 + 1).to(torch.bfloat16)
        kw = (torch.randn(128, generator=g, device=dev) * 0.2 + 1).to(torch.bfloat16)
        pos = torch.randint(0, 40960, (n,), generator=g, device=dev)
        inv_freq = 1.0 / (1000000.0 ** (torch.arange(0, 128, 2, dtype=torch.float) / 128))
        freqs = torch.einsum("i,j -> ij", torch.arange(40960, dtype=torch.float), inv_freq)
        cos_sin = torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1).to(dev)
        caches = [(torch.empty_like(c.k), torch.empty_like(c.v)) for _ in range(8)]
        ep_ms = _time_graph_calls(lambda: [qk_norm_rope_store(
            x, pos, qw, kw, 1e-6, cos_sin, hq, kvh, kc, vc, c.slot_mapping)
            for x, (kc, vc) in zip(qkvs, caches)], 8)
        ep_bytes = n * ((hq + 2 * kvh) * 256 + hq * 256 + 2 * kvh * 128 + 8 + 4 + 512)
        gbs = ep_bytes / (ep_ms * 1e-3) / 1e9
        out["epilogue_config3"] = {
            "workload": "q/k RMSNorm + RoPE + K/V e4m3 store of config 3's 5,561 new rows "
                        "(Qwen3-8B heads), one kernel", "ms": ep_ms, "bytes": ep_bytes,
            "timing": "CUDA graph of 8 back-to-back calls on 8 independent input sets, per call",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": gbs / hbm_peak}}
        if ref is not None:
            try:
                from nanovllm.layers.layernorm import RMSNorm
                from nanovllm.layers.rotary_embedding import get_rope
                rope = get_rope(128, 128, 40960, 1000000.0).to(dev)
                qn, kn = RMSNorm(128).to(dev), RMSNorm(128).to(dev)
                with torch.no_grad():
                    qn.weight.copy_(qw.float())
                    kn.weight.copy_(kw.float())
                qn, kn = qn.to(torch.bfloat16), kn.to(torch.bfloat16)

                def ref_chain():
                    with torch.no_grad():
                        for x, (kc, vc) in zip(qkvs, caches):
                            q, k, v = x.split([hq * 128, kvh * 128, kvh * 128], dim=-1)
                            q3, k3 = rope(pos, qn(q.reshape(-1, hq, 128)),
                                          kn(k.reshape(-1, kvh, 128)))
                            ref["store"](k3, v.reshape(-1, kvh, 128), kc, vc, c.slot_mapping)
                ref_chain()  # compiles the reference's functions outside the timing
                ref_time("epilogue_config3", ref_chain, ep_ms, ncalls=8)
            except Exception as e:  # pragma: no cover
                refgpu["epilogue_config3"] = {"unavailable": f"{type(e).__name__}: {e}"}
        del c, qkvs, caches
        torch.cuda.empty_cache()
    # ---- FP8 block-scaled linear: Qwen3-8B's QKV projection (K 4096 -> N 6144) at config 2's
    # decode batch (256 tokens, weight-streaming) and at the 8192-token prefill budget (tensor)
    if lin_decode or lin_prefill:
        from nanovllm_b200.fp8_linear import fp8_block_linear
        K, N = 4096, 6144
        g = torch.Generator(device=dev).manual_seed(91)
        sets = []
        for _ in range(8 if lin_decode else 1):
            w = (torch.randn(N, K, generator=g, device=dev) * 0.5).to(torch.float8_e4m3fn)
            ws = (torch.rand(N // 128, K // 128, generator=g, device=dev) * 0.02 + 0.001).to(
                torch.bfloat16)
            x = torch.randn(256, K, generator=g, device=dev).to(torch.bfloat16)
            sets.append((x, w, ws))
        lin = out["fp8linear_qkv"] = {
            "workload": "y = x . w^T, e4m3 weight 6144 x 4096 in 128 x 128 blocks (Qwen3-8B QKV "
                        "projection), bf16 x quantised per token and 128-column group"}
        if lin_decode:
            d_ms = _time_graph_calls(lambda: [fp8_block_linear(*a) for a in sets], len(sets))
            d_bytes = N * K + (N // 128) * (K // 128) * 2 + 256 * K * 2 + 256 * N * 2
            d_gbs = d_bytes / (d_ms * 1e-3) / 1e9
            lin["decode_m256"] = {
                "ms": d_ms, "bytes": d_bytes, "tokens_per_s": 256 / (d_ms * 1e-3),
                "timing": "CUDA graph of 8 back-to-back calls on 8 independent weight and input "
                          "sets (200 MB, more than L2), per call; quantise + GEMM",
                "roofline": {"bound": "hbm", "achieved": d_gbs, "peak": hbm_peak, "unit": "GB/s",
                             "frac": d_gbs / hbm_peak}}
            if ref is not None and "linear" in ref:
                ref_time("fp8linear_decode_m256", lambda: [ref["linear"](*a) for a in sets],
                         d_ms, ncalls=len(sets))
        if lin_prefill:
            xp = torch.randn(8192, K, generator=g, device=dev).to(torch.bfloat16)
            w0, ws0 = sets[0][1], sets[0][2]
            p_ms = _time_calls(lambda: fp8_block_linear(xp, w0, ws0), iters=10, warm=3,
                               flush=flush)
            p_flops = 2 * 8192 * N * K
            p_tf = p_flops / (p_ms * 1e-3) / 1e12
            lin["prefill_m8192"] = {
                "ms": p_ms, "flops": p_flops, "tokens_per_s": 8192 / (p_ms * 1e-3),
                "l2": "flushed before each call",
                "roofline": {"bound": "tensor", "achieved": p_tf, "peak": fp8_peak,
                             "unit": "TFLOP/s", "frac": p_tf / fp8_peak, "peak_kind": fp8_kind}}
            if ref is not None and "linear" in ref:
                ours = fp8_block_linear(xp, w0, ws0)
                ref_time("fp8linear_prefill_m8192", lambda: ref["linear"](xp, w0, ws0), p_ms,
                         ours, iters=5, warm=2, flush_l2=flush)
            del xp
        del sets
        torch.cuda.empty_cache()
    return out, refgpu


def tp_linear_bench(world, rank, local, with_reference=True):
    """Row-parallel FP8 o_proj with its all-reduce (one rank per GPU, N > 1; `--only tp_linear`
    under torchrun): Qwen3-32B's o_proj (64 heads x 128 = 8,192 in, 5,120 out), each rank its
    8,192 / N input columns, at 256 tokens (decode) and 8,192 tokens (prefill budget).  Three ways:
    the fused kernel (fp8attn_fp8_tp_linear), this library's fp8_block_linear + NCCL all_reduce,
    and the reference's Triton fp8_block_linear + NCCL all_reduce (RowParallelLinear.forward).
    Each timed with CUDA events after a barrier, median of 10, max over ranks."""
    import torch
    import torch.distributed as dist
    from nanovllm_b200.fp8_attention import device_error
    from nanovllm_b200.fp8_linear import fp8_block_linear
    from nanovllm_b200.tp_linear import TpLinearBuffers, fp8_row_parallel_linear
    dev = torch.device("cuda", local)
    ref, ref_err = _reference_module() if with_reference else (None, "not requested")
    K, N = 8192, 5120
    kl = K // world
    fp8_peak = _fp8_peak(dev) or 2 * _peaks()[1]
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    w = (torch.randn(N, kl, generator=g, device=dev) * 0.5).to(torch.float8_e4m3fn)
    ws = (torch.rand(N // 128, kl // 128, generator=g, device=dev) * 0.02 + 0.001).to(
        torch.bfloat16)
    bufs = TpLinearBuffers(8192, N, device=dev)

    def timed(fn, iters=10, warm=3):
        for _ in range(warm):
            fn()
        ts = []
        for _ in range(iters):
            dist.barrier()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b))
        return _reduce(statistics.median(ts), world, "max")

    line = {"metric": "row-parallel FP8 o_proj + all-reduce", "n_gpus": world,
            "workload": "Qwen3-32B o_proj, 8192 -> 5120, K split over the ranks, block-quantised "
                        "e4m3 weight, bf16 activations; synthetic"}
    for m in (256, 8192):
        x = torch.randn(m, kl, generator=g, device=dev).to(torch.bfloat16)

        def fused():
            return fp8_row_parallel_linear(x, w, ws, bufs)

        def nccl():
            y = fp8_block_linear(x, w, ws)
            dist.all_reduce(y)
            return y

        entry = {"fused_ms": timed(fused), "ours_gemm_plus_nccl_ms": timed(nccl)}
        flops = 2 * m * N * K / world                    # per rank
        link = 2 * m * N * 2 * (world - 1) / world       # bytes each rank sends over NVLink
        target_ms = max(flops / (fp8_peak * 1e12), link / 770e9) * 1e3
        entry["roofline"] = {"target_ms": target_ms, "frac": target_ms / entry["fused_ms"],
                             "flops_per_rank": flops, "nvlink_bytes_per_rank": link,
                             "fp8_peak_tflops": fp8_peak, "link_gbs": 770}
        if ref is not None and "linear" in ref:
            def refn():
                y = ref["linear"](x, w, ws)
                dist.all_reduce(y)
                return y
            entry["reference_ms"] = timed(refn)
            entry["speedup_vs_reference"] = entry["reference_ms"] / entry["fused_ms"]
            d = (fused().float() - refn().float()).abs().max()
            dist.all_reduce(d, op=dist.ReduceOp.MAX)
            entry["max_abs_diff_vs_reference"] = float(d)
        line[f"m{m}"] = entry
    if ref is None:
        line["reference"] = ref_err
    torch.cuda.synchronize()
    err = torch.tensor([float(device_error(dev))], device=dev)
    dist.all_reduce(err, op=dist.ReduceOp.MAX)
    line["device_error"] = int(err.item())
    del bufs
    if rank == 0:
        print(json.dumps(line), flush=True)


def _e2e(case, steps, warmup, world, stream):
    """The headline call through the public API with host buffers: every step copies its inputs
    (q, block tables, lengths) from pinned host memory and its output back.  The copies run on a
    second stream with double-buffered device inputs (events order them), so step i+1's upload
    and step i's download overlap a kernel; all of them are inside the timed region."""
    import torch
    from nanovllm_b200 import fp8_decode_attention
    dev = case.q.device
    q_h = case.q.cpu().pin_memory()
    bt_h = case.block_tables.cpu().pin_memory()
    ctx_h = case.context_lens.cpu().pin_memory()
    out_h = [torch.empty(case.q.shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    q_d = [torch.empty_like(case.q) for _ in range(2)]
    bt_d = [torch.empty_like(case.block_tables) for _ in range(2)]
    ctx_d = [torch.empty_like(case.context_lens) for _ in range(2)]
    h2d = q_h.numel() * 2 + bt_h.numel() * 4 + ctx_h.numel() * 4
    d2h = out_h[0].numel() * 2
    copy_stream = torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]  # buffer b's output copied: reusable
    for e in ev_free:
        e.record(copy_stream)

    def upload(b):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(ev_free[b])
            q_d[b].copy_(q_h, non_blocking=True)
            bt_d[b].copy_(bt_h, non_blocking=True)
            ctx_d[b].copy_(ctx_h, non_blocking=True)
            ev_in[b].record(copy_stream)

    def run(b):
        stream.wait_event(ev_in[b])
        o = fp8_decode_attention(q_d[b], case.k_cache, case.v_cache, bt_d[b], ctx_d[b], case.scale)
        ev_out[b].record(stream)
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(ev_out[b])
            o.record_stream(copy_stream)
            out_h[b].copy_(o, non_blocking=True)
            ev_free[b].record(copy_stream)

    def loop(n):
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload((i + 1) % 2)
            run(i % 2)
        stream.wait_stream(copy_stream)

    loop(warmup)
    torch.cuda.synchronize()
    _barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    copy_stream.wait_event(a)  # the first upload starts inside the timed region
    loop(steps)
    b.record(stream)
    torch.cuda.synchronize()
    return _reduce(a.elapsed_time(b), world, "max"), h2d, d2h


def run_ours(args, world, rank, local):
    import torch
    from nanovllm_b200 import _lib, fp8_decode_attention
    from nanovllm_b200.fp8_attention import device_error
    workloads = _load_workloads()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peaks = _peaks()
    hbm_peak = peaks[0]
    if 8 % world:
        raise SystemExit(f"config 5's 8 kv heads do not split over {world} GPUs")

    # rank r: its kv-head group of config 5 (strong scaling: the total work is fixed)
    case = workloads.config5(dev, gpus=world, rank=rank, batch=args.batch)
    step_bytes = case.kv_bytes()
    total_bytes = _reduce(float(step_bytes), world, "sum")
    stream = torch.cuda.current_stream(dev)

    def step():
        return fp8_decode_attention(case.q, case.k_cache, case.v_cache, case.block_tables,
                                    case.context_lens, case.scale)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _barrier(world)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for s, e in ev:
            s.record(stream)
            step()
            e.record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
        if not clk.samples:  # nvidia-smi fallback: make sure at least one sample is taken
            time.sleep(0.25)
    total_ms = _reduce(t_start.elapsed_time(t_end), world, "max")
    per_launch_ms = statistics.mean(s.elapsed_time(e) for s, e in ev)
    per_launch_max = _reduce(per_launch_ms, world, "max")
    err = int(_reduce(float(device_error(dev)), world, "max"))

    e2e_ms, h2d, d2h = _e2e(case, args.steps, args.warmup, world, stream)
    h2d = int(_reduce(float(h2d), world, "sum"))
    d2h = int(_reduce(float(d2h), world, "sum"))
    ctas = int(_lib.lib.fp8attn_decode_ctas(case.q.shape[0], case.q.shape[1],
                                            case.k_cache.shape[2], 1))
    if rank != 0:
        return
    ms = total_ms / args.steps
    value = total_bytes / (ms * 1e-3) / 1e12
    achieved_gbs = step_bytes / (per_launch_ms * 1e-3) / 1e9  # rank 0's decode + combine launches
    tr = _traffic("decode_config5")
    line = {
        "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "e4m3",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "parallelism": f"kv-head-split{world}",
                   "kv_heads_per_gpu": 8 // world, "q_heads_per_gpu": 64 // world,
                   "batch": int(case.q.shape[0]), "context": 32768,
                   "bytes_per_step": int(total_bytes), "bytes_per_step_rank0": step_bytes,
                   "l2": "inputs larger than L2 (K/V per GPU per step > 126 MB)",
                   "fraction_of_8TBs_per_gpu": value / world / 8.0,
                   "max_gpu_step_ms": per_launch_max},
        "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved_gbs / hbm_peak, "peak_kind": peaks[3],
                     "kernel": "decode_kernel + combine_rows_kernel (rank 0, per step)",
                     "traffic": (int(tr * step_bytes) if tr is not None else None)},
        "e2e": {"value": total_bytes / (e2e_ms / args.steps * 1e-3) / 1e12, "unit": "TB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": 2 * args.steps,  # decode + split-KV combine per step
        "decode_ctas": ctas,
        "clocks": clk.summary(),
        "device_error": err,
    }
    if world == 1 and args.batch == 64 and not args.no_reference_gpu:
        ref, why = _reference_module()
        if ref is None:
            line["reference_gpu_decode_config5"] = {"unavailable": why}
        else:  # the reference's own Triton decode on the headline inputs (same GPU)
            args5 = (case.q, case.k_cache, case.v_cache, case.block_tables, case.context_lens,
                     case.scale)
            ours = step()
            r_ms = _time_calls(lambda: ref["decode"](*args5), iters=5, warm=2)
            line["reference_gpu_decode_config5"] = {
                "ms": r_ms, "ours_ms": ms, "speedup": r_ms / ms,
                "max_abs_diff_vs_ours": _maxdiff(ref["decode"](*args5), ours)}
    if world == 1 and args.batch == 64:
        del case
        torch.cuda.empty_cache()
        sec, refgpu = secondary(dev, peaks, not args.no_reference_gpu)
        line.update(sec)
        line["reference_gpu"] = refgpu
        line["device_error"] = max(line["device_error"], device_error(dev))
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(workloads.config5("cpu", batch=8),
                                                max_seconds=args.cpu_seconds)
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's Triton kernels on the GPU")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--batch", type=int, default=64,
                    help="config-5 sequences (64 = the benchmark; fewer for profile captures, "
                         "which then skip the secondary figures)")
    ap.add_argument("--only", default=None,
                    help="comma-separated secondary parts (%s) to run alone on one GPU, "
                         "without the headline (profile captures); or tp_linear under torchrun "
                         "with N > 1 (the fused row-parallel o_proj)" % ",".join(PARTS + SUBPARTS))
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = _dist_init() if args.impl == "ours" else (
        int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.only == "tp_linear":
            assert world > 1, "tp_linear runs under torchrun with N > 1"
            tp_linear_bench(world, rank, local, not args.no_reference_gpu)
        elif args.only:
            import torch
            from nanovllm_b200.fp8_attention import device_error
            only = args.only.split(",")
            assert set(only) <= set(PARTS) | set(SUBPARTS), only
            torch.cuda.set_device(0)
            sec, _ = secondary(torch.device("cuda", 0), _peaks(), False, only)
            sec["device_error"] = device_error()
            print(json.dumps(sec), flush=True)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
