"""End to end: the reference engine's LLM.generate on a tiny random-weight Qwen3 (8 q / 2 kv heads,
head_dim 128, 2 layers) with the FP8 KV cache, once on its own Triton kernels and once with
nanovllm_b200 patched in (nanovllm_b200.patch.install), the second run replaying the first run's
sampled tokens.  Both runs schedule the same batches (CUDA-graph decode, chunked prefill over a
cached prefix, n-gram speculative verification), so their logits are compared step by step.

Needs the reference installed under baseline/_ref (skipped otherwise); each run is a separate
process (tests/e2e_engine_worker.py) because the engine owns a process group and CUDA graphs.
"""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF = os.path.join(ROOT, "baseline", "_ref")


def _model_dir(path):
    from transformers import PreTrainedTokenizerFast, Qwen3Config, Qwen3ForCausalLM
    from tokenizers import Tokenizer, models, pre_tokenizers
    cfg = Qwen3Config(vocab_size=1024, hidden_size=512, intermediate_size=1024,
                      num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                      head_dim=128, max_position_embeddings=4096, rope_theta=1e6,
                      tie_word_embeddings=False, initializer_range=0.05, dtype=torch.bfloat16)
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(cfg).to(torch.bfloat16)
    model.save_pretrained(path, safe_serialization=True)
    vocab = {"<unk>": 0, "<eos>": 1, **{f"t{i}": i for i in range(2, 1024)}}
    tok = Tokenizer(models.WordLevel(vocab, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="<unk>",
                            eos_token="<eos>").save_pretrained(path)


def _run(model_dir, mode, record):
    env = dict(os.environ)
    env.setdefault("NCCL_NVLS_ENABLE", "0")
    r = subprocess.run([sys.executable, os.path.join(HERE, "e2e_engine_worker.py"), model_dir, mode,
                        record], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, f"{mode} run failed:\n{r.stdout[-3000:]}\n{r.stderr[-6000:]}"


def _compare(ref, ours, what):
    assert len(ref) == len(ours) and len(ref) > 10
    worst, agree, rows = 0.0, 0, 0
    for a, b in zip(ref, ours):
        assert a.shape == b.shape
        assert torch.isfinite(b).all()
        scale = a.abs().max().clamp_min(1e-3)
        worst = max(worst, float((a - b).abs().max() / scale))
        agree += int((a.argmax(-1) == b.argmax(-1)).sum())
        rows += a.shape[0]
    # attention differences of ~1e-2 (the kernels' tolerance) move logits by a small fraction
    # of their range; the argmax almost never flips
    print(f"e2e {what}: {len(ref)} steps, {rows} logit rows, worst |dlogit|/max|logit| "
          f"{worst:.4f}, argmax agreement {agree / rows:.4f}")
    assert worst < 0.05, worst
    assert agree / rows > 0.97, agree / rows


@pytest.fixture(scope="module")
def reference_run(tmp_path_factory):
    if not os.path.isdir(os.path.join(REF, "nanovllm")):
        pytest.skip("reference engine not installed under baseline/_ref")
    tmp = tmp_path_factory.mktemp("e2e")
    model_dir = str(tmp / "qwen3-tiny")
    _model_dir(model_dir)
    record = str(tmp / "record.pt")
    _run(model_dir, "reference", record)
    return model_dir, record


def test_generate_drop_in_matches_reference_logits(reference_run):
    model_dir, record = reference_run
    _run(model_dir, "b200", record)
    ref = torch.load(record)["logits"]
    got = torch.load(record + ".b200")
    # every entry point served the engine: the store, decode (eager and at graph capture) and the
    # paged prefill (chunked prefill over a cached prefix, speculative verification)
    assert all(n > 0 for n in got["calls"].values()), got["calls"]
    _compare(ref, got["logits"], f"drop-in, library calls {got['calls']}")


def test_generate_with_fused_epilogue_matches_reference_logits(reference_run):
    """The same run with the fused q/k norm + rope + K/V store epilogue in Qwen3Attention: the
    store entry point is then never called (the epilogue stores), the attention entry points
    still are."""
    model_dir, record = reference_run
    _run(model_dir, "b200fused", record)
    ref = torch.load(record)["logits"]
    got = torch.load(record + ".b200fused")
    calls = got["calls"]
    assert calls["store_kvcache"] == 0 and calls["qk_norm_rope_store"] > 0, calls
    assert calls["fp8_decode_attention"] > 0 and calls["fp8_prefill_attention"] > 0, calls
    _compare(ref, got["logits"], f"fused epilogue, library calls {calls}")
