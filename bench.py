"""Benchmark of the FP8 PagedAttention hot path (BASELINE.json metric).

Headline workload (a "step"): one paged FP8 decode call over BASELINE config 2 (Qwen3-8B heads
32 q / 8 kv, 256 sequences, context U[512, 4096], block 256, pool 1.25x, seed 1).  ``value`` is
the decode's algorithmic HBM throughput (TB/s): every visible K and V byte once, plus q, out,
block tables and lengths, divided by the device time of the step; the KV working set (~1.2 GB)
is far larger than L2, so no flush is needed between steps.

Multi-GPU (``torchrun ... bench.py --gpus N``): KV-head-group sharding with no collective in the
path.  Every rank holds a config-2-sized shard (8 kv heads, 32 q heads, its own cache and seed),
so per-GPU work is fixed ("weak" scaling); the time is the max over ranks.

Secondary figures on the same line (not the headline): ``prefill`` = the varlen causal chunked
prefill of BASELINE config 3 (TFLOP/s of causal-useful FLOPs, L2 flushed before every timed
call) and ``store`` = the K/V store of the same call's 5.1k new rows (GB/s).

``--impl reference`` times the reference algorithm on the host cores instead (the CPU oracle,
a torch fp32 restatement of fp8_paged_attention_decode_kernel) on a bounded sample.
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
sys.path.insert(0, os.path.join(ROOT, "my-nano-vllm_b200"))
sys.path.insert(0, ROOT)

METRIC = "FP8 paged decode HBM TB/s (% of 8 TB/s); varlen prefill TFLOP/s (% peak)"
WORKLOAD = "config2: FP8 paged decode, Qwen3-8B heads (32q/8kv, d128), 256 seqs, ctx U[512,4096], block 256"


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def _traffic(kernel: str):
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f).get(kernel)
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


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def cpu_baseline(case, max_seconds: float = 20.0):
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
            "sample": f"first {n} of {q.shape[0]} config-2 sequences ({done_bytes / 1e6:.1f} MB "
                      f"of K/V), torch fp32 oracle, {t_total:.1f} s"}


def run_reference(args, world, rank):
    """--impl reference: the reference algorithm on the host cores (CPU oracle port)."""
    import torch
    if rank != 0:
        return
    from nanovllm_b200 import workloads
    case = workloads.config2("cpu")
    for _ in range(args.warmup):
        pass
    steps = []
    for _ in range(max(1, min(args.steps, 3))):
        r = cpu_baseline(case, max_seconds=15.0)
        steps.append(r)
    value = statistics.median(s["value"] for s in steps)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s",
            "n_gpus": world, "steps": len(steps), "warmup": args.warmup,
            "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "parallelism": f"kv-head-shard{world}",
                       "note": "bounded sample per step; see cpu_baseline.sample"},
            "cpu_baseline": dict(steps[-1], value=value),
            "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _flush_l2(buf):
    buf.add_(1)  # writes 256 MB, twice the 126 MB L2


def secondary(dev, hbm_peak, bf16_peak):
    """Config-3 prefill (tensor bound) and its K/V store (HBM bound), CUDA-event timed per call
    with L2 flushed in between.  FP8 dense peak = 2 x the measured bf16 GEMM peak (the e4m3
    tensor rate is twice the bf16 rate on sm_100a)."""
    import torch
    from nanovllm_b200 import fp8_prefill_attention, store_kvcache, workloads
    c = workloads.config3(dev)
    flops = c.causal_flops()
    n = c.new_k.shape[0]
    store_bytes = n * (2 * 8 * 128 * 2 + 2 * 8 * 128 + 4)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)

    def timed(fn, iters=10, warm=3):
        for _ in range(warm):
            fn()
        ts = []
        for _ in range(iters):
            _flush_l2(flush)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    # the store is ~10 us of device work: time a CUDA graph of the call so that the host-side
    # launch (the Python wrapper) is not measured
    store_kvcache(c.new_k, c.new_v, c.k, c.v, c.slot_mapping)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        store_kvcache(c.new_k, c.new_v, c.k, c.v, c.slot_mapping)
    st_ms = timed(graph.replay)
    del graph
    pf_ms = timed(lambda: fp8_prefill_attention(
        c.q, c.k, c.v, block_tables=c.block_tables, cu_seqlens_q=c.cu_seqlens_q,
        cu_seqlens_k=c.cu_seqlens_k, max_seqlen_q=c.max_seqlen_q, max_seqlen_k=c.max_seqlen_k,
        softmax_scale=c.scale))
    tflops = flops / (pf_ms * 1e-3) / 1e12
    fp8_peak = 2 * bf16_peak
    return {
        "prefill": {"workload": "config3: 16 seqs, new U[128,512], cached prefix U[0,3584], "
                                "Qwen3-8B heads, paged block 256",
                    "ms": pf_ms, "tflops": tflops, "causal_flops": flops,
                    "roofline": {"bound": "tensor", "achieved": tflops, "peak": fp8_peak,
                                 "unit": "TFLOP/s", "frac": tflops / fp8_peak,
                                 "peak_note": "e4m3 dense = 2 x measured bf16 GEMM"},
                    "l2": "flushed before each call"},
        "store": {"ms": st_ms, "gbs": store_bytes / (st_ms * 1e-3) / 1e9, "rows": n,
                  "timing": "CUDA-graph replay, L2 flushed before each call",
                  "bytes": store_bytes, "frac": store_bytes / (st_ms * 1e-3) / 1e9 / hbm_peak},
    }


def run_ours(args, world, rank, local):
    import torch
    from nanovllm_b200 import fp8_decode_attention, workloads
    from nanovllm_b200.fp8_attention import device_error
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    hbm_peak, bf16_peak, peak_kind = _peaks()

    # rank r: its own config-2-sized shard (weak scaling)
    case = workloads.decode_case(256, 32, 8, 512, 4096, seed=1 + 1000 * rank, device=dev,
                                 pool_factor=1.25)
    step_bytes = case.kv_bytes()
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
    total_ms = t_start.elapsed_time(t_end)
    per_launch_ms = statistics.mean(s.elapsed_time(e) for s, e in ev)
    total_ms = _max_over_ranks(total_ms, world)
    per_launch_ms = _max_over_ranks(per_launch_ms, world)
    err = device_error(dev)

    # ---- end to end through the public API with host buffers: every step copies its inputs
    # (q, block tables, lengths) from pinned host memory and its output back.  The copies run on a
    # second stream with double-buffered device inputs (events order them), so step i+1's
    # upload and step i's download overlap a kernel; all of them are inside the timed region.
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

    def e2e_loop(n):
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload((i + 1) % 2)
            run(i % 2)
        stream.wait_stream(copy_stream)

    e2e_loop(args.warmup)
    torch.cuda.synchronize()
    _barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    copy_stream.wait_event(a)  # the first upload starts inside the timed region
    e2e_loop(args.steps)
    b.record(stream)
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(a.elapsed_time(b), world)

    if rank != 0:
        return
    ms = total_ms / args.steps
    value = world * step_bytes / (ms * 1e-3) / 1e12
    achieved_gbs = step_bytes / (per_launch_ms * 1e-3) / 1e9
    e2e_val = world * step_bytes / (e2e_ms / args.steps * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e4m3",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "parallelism": f"kv-head-shard{world}",
                   "bytes_per_step_per_gpu": step_bytes,
                   "l2": "inputs larger than L2 (1.2 GB of K/V per step)",
                   "fraction_of_8TBs": value / world / 8.0},
        "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved_gbs / hbm_peak, "peak_kind": peak_kind,
                     "traffic": _traffic("decode_kernel")},
        "e2e": {"value": e2e_val, "unit": "TB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": 2 * args.steps,  # decode + split-KV combine per step
        "decode_ctas": int(__import__("nanovllm_b200._lib", fromlist=["lib"]).lib.fp8attn_decode_ctas(256, 32, 8, 1)),
        "clocks": clk.summary(),
        "device_error": err,
    }
    if world == 1:
        # outside the headline's timed region; a paged prefill call launches 3 kernels (the
        # split-KV engine for short sequences + its combine, then the prefill engine), a store 1
        line.update(secondary(dev, hbm_peak, bf16_peak))
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(case, max_seconds=args.cpu_seconds)
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = _dist_init() if args.impl == "ours" else (
        int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
