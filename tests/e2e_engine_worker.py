"""One end-to-end run of the reference engine (nano-vLLM ``LLM.generate``) on a tiny random Qwen3,
for tests/test_e2e_engine_gpu.py.  Run as a script in its own process (the engine owns a process
group and CUDA graphs):

    python tests/e2e_engine_worker.py MODEL_DIR MODE RECORD.pt

MODE ``reference``: the engine's own Triton kernels; the sampled tokens and the logits of every
step are written to RECORD.pt.  MODE ``b200``: ``nanovllm_b200.patch.install()`` first, the tokens
of RECORD.pt are replayed in place of sampling (teacher forcing, so both runs schedule the same
batches: chunked prefill over a cached prefix, n-gram speculative verification, CUDA-graph decode)
and the logits are written to RECORD.pt.b200.  MODE ``b200fused``: the same, and the fused q/k
norm + rope + K/V store epilogue (``nanovllm_b200.qk_epilogue.install()``) in place of the model's
norm, rotary and store steps; logits to RECORD.pt.b200fused.

The sampler is replaced in both modes by an eager restatement of the reference's (temperature,
softmax, exponential race; nanovllm/layers/sampler.py) so no compilation is needed.
"""
from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def main(model_dir: str, mode: str, record: str) -> None:
    sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
    sys.path.insert(0, os.path.join(ROOT, "my-nano-vllm_b200"))
    import torch
    from nanovllm import LLM, SamplingParams
    from nanovllm.engine import model_runner as mr
    from nanovllm.layers import sampler as smp

    calls = {"store_kvcache": 0, "fp8_decode_attention": 0, "fp8_prefill_attention": 0}
    if mode in ("b200", "b200fused"):
        import nanovllm_b200.patch
        from nanovllm.layers import attention as att
        nanovllm_b200.patch.install()
        for name in list(calls):  # count the engine's calls into the library (no graph replays)
            def counted(*args, _f=getattr(att, name), _n=name, **kw):
                calls[_n] += 1
                return _f(*args, **kw)
            setattr(att, name, counted)
        if mode == "b200fused":  # also the fused q/k norm + rope + K/V store epilogue
            from nanovllm_b200 import qk_epilogue
            qk_epilogue.install()
            calls["qk_norm_rope_store"] = 0

            def counted_epilogue(*args, _f=qk_epilogue.qk_norm_rope_store, **kw):
                calls["qk_norm_rope_store"] += 1
                return _f(*args, **kw)
            qk_epilogue.qk_norm_rope_store = counted_epilogue
        replay = list(torch.load(record)["tokens"])
    steps, tokens = [], []
    orig_run_model = mr.ModelRunner.run_model

    def run_model(self, has_prefill, input_ids, positions):
        logits = orig_run_model(self, has_prefill, input_ids, positions)
        steps.append(logits.float().cpu())
        return logits

    def sample(self, logits, temperatures):
        if mode != "reference":
            return replay.pop(0).to(logits.device)
        probs = torch.softmax(logits.float().div(temperatures.unsqueeze(1)), dim=-1)
        out = probs.div(torch.empty_like(probs).exponential_(1).clamp_min_(1e-10)).argmax(dim=-1)
        tokens.append(out.cpu())
        return out

    mr.ModelRunner.run_model = run_model
    smp.Sampler.forward = sample
    torch.manual_seed(0)
    llm = LLM(model_dir, max_num_batched_tokens=2048, max_model_len=2048, max_num_seqs=64,
              gpu_memory_utilization=0.25, kvcache_block_size=256)
    gen = torch.Generator().manual_seed(5)
    prompts = []
    for n in (900, 1300, 700, 1100, 600, 1500):
        base = torch.randint(2, 1000, (n // 4,), generator=gen).tolist()
        prompts.append((base * 4)[:n])  # repeated segments give the n-gram proposer drafts
    outs = llm.generate(prompts, SamplingParams(temperature=1.0, max_tokens=40, ignore_eos=True))
    assert len(outs) == len(prompts) and all(len(o["token_ids"]) >= 40 for o in outs)
    if mode == "reference":
        torch.save({"tokens": tokens, "logits": steps}, record)
    else:
        assert not replay, f"{len(replay)} recorded samples were not consumed"
        torch.save({"logits": steps, "calls": calls}, record + "." + mode)
    # the engine's own exit (registered with atexit) releases its graphs and process group


if __name__ == "__main__":
    main(*sys.argv[1:4])
