"""End-to-end run of this backend inside vLLM (the drop-in check).

Mirrors the reference's ``flash_attention_backend/test_self_flash_attn_backend.py``: the
backend is registered as ``CUSTOM`` (``:11-15``) and an ``LLM`` generates greedily with
``attention_backend="CUSTOM"`` and bf16 KV cache (``:30-34,88-97``). The model weights of
the reference's runs (gpt2 / Qwen2.5-0.5B-Instruct from the HF hub) are not available
offline, so the model is a Qwen2.5-0.5B-shaped ``Qwen2ForCausalLM`` config written to a
temporary directory and loaded with vLLM's random weights (``load_format="dummy"``), which
are then redrawn from a seeded N(0, 0.02) per parameter (vLLM's dummy values are so small
that attention is nearly uniform); prompts are token ids (no tokenizer). The same run with one of vLLM's own attention
backends gives the comparison: same weights, same prompts, greedy tokens and their
log-probabilities side by side.

Usage (one GPU)::

    python -m toy_flash_attn.vllm_e2e --backend CUSTOM --out custom.json
    python -m toy_flash_attn.vllm_e2e --backend TRITON_ATTN --out triton.json

Prints one JSON object and writes it to ``--out``.
"""

from __future__ import annotations

import argparse
import json
import os
import tempfile
import time
from pathlib import Path

# Qwen2.5-0.5B architecture: 14 q heads, 2 kv heads, head_dim 64 (BASELINE config C2's shape).
QWEN2_SMALL = {
    "architectures": ["Qwen2ForCausalLM"],
    "model_type": "qwen2",
    "hidden_size": 896,
    "intermediate_size": 4864,
    "num_attention_heads": 14,
    "num_key_value_heads": 2,
    "num_hidden_layers": 24,
    "max_position_embeddings": 4096,
    "max_window_layers": 24,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1000000.0,
    "hidden_act": "silu",
    "vocab_size": 151936,
    "tie_word_embeddings": True,
    "torch_dtype": "bfloat16",
    "use_sliding_window": False,
    "sliding_window": None,
    "bos_token_id": 151643,
    "eos_token_id": 151645,
}


def _prompts(n: int, vocab: int) -> list[list[int]]:
    """Deterministic token-id prompts of different lengths (prefill of mixed lengths)."""
    out = []
    for i in range(n):
        length = 17 + 37 * i
        out.append([(1000 + 7919 * (i + 1) * (j + 1)) % vocab for j in range(length)])
    return out


def _reinit(std: float):
    """Returns a function that redraws every parameter from N(0, std) (norm weights stay
    1) with a generator seeded per parameter name, so two runs get identical weights."""
    import zlib

    import torch

    def fn(model):
        for name, prm in model.named_parameters():
            if name.endswith("norm.weight") or "layernorm" in name:
                continue
            g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
            with torch.no_grad():
                prm.copy_((torch.randn(prm.shape, generator=g) * std).to(prm.dtype))
        return None

    return fn


def run(backend: str, num_prompts: int, max_tokens: int, std: float, max_batched_tokens: int | None = None) -> dict:
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")  # keep the engine in this process
    os.environ.setdefault("HF_HUB_OFFLINE", "1")
    os.environ.setdefault("TRANSFORMERS_OFFLINE", "1")
    from vllm import LLM, SamplingParams
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend

    register_backend(AttentionBackendEnum.CUSTOM, "toy_flash_attn.ToyFlashAttentionBackend")
    from toy_flash_attn import flash_attention_func as faf

    calls = {"n": 0}
    inner = faf.flash_attn_varlen_with_block_cu_bf16

    def counted(*a, **k):
        calls["n"] += 1
        return inner(*a, **k)

    faf.flash_attn_varlen_with_block_cu_bf16 = counted

    with tempfile.TemporaryDirectory() as d:
        (Path(d) / "config.json").write_text(json.dumps(QWEN2_SMALL))
        t0 = time.time()
        extra = {}
        if max_batched_tokens:  # small budgets make chunked prefill mix prompt chunks with decodes
            extra = dict(max_num_batched_tokens=max_batched_tokens, enable_chunked_prefill=True)
        llm = LLM(model=d, skip_tokenizer_init=True, load_format="dummy", dtype="bfloat16", seed=0,
                  max_model_len=2048, gpu_memory_utilization=0.5, max_num_seqs=num_prompts, enforce_eager=True,
                  attention_backend=backend, kv_cache_dtype="bfloat16" if backend == "CUSTOM" else "auto",
                  **extra)
        t_init = time.time() - t0
        if std > 0:
            llm.apply_model(_reinit(std))
        prompts = [{"prompt_token_ids": p} for p in _prompts(num_prompts, QWEN2_SMALL["vocab_size"])]
        sp = SamplingParams(temperature=0.0, max_tokens=max_tokens, logprobs=1, detokenize=False, ignore_eos=True)
        t1 = time.time()
        outs = llm.generate(prompts, sp)
        t_gen = time.time() - t1
    result = {"backend": backend, "weight_std": std, "init_s": round(t_init, 1), "generate_s": round(t_gen, 2),
              "custom_attention_calls": calls["n"], "sequences": []}
    for o in outs:
        c = o.outputs[0]
        lps = [float(lp[t].logprob) for t, lp in zip(c.token_ids, c.logprobs)] if c.logprobs else []
        result["sequences"].append({"prompt_len": len(o.prompt_token_ids), "tokens": list(c.token_ids),
                                    "logprobs": lps})
    return result


def compare(a: dict, b: dict) -> dict:
    """Greedy-token agreement and log-prob gap between two runs (up to the first divergence)."""
    same, total, max_gap = 0, 0, 0.0
    first_div = []
    for sa, sb in zip(a["sequences"], b["sequences"]):
        n = min(len(sa["tokens"]), len(sb["tokens"]))
        k = 0
        while k < n and sa["tokens"][k] == sb["tokens"][k]:
            max_gap = max(max_gap, abs(sa["logprobs"][k] - sb["logprobs"][k]))
            k += 1
        first_div.append(k)
        same += k
        total += n
    return {"tokens_identical_prefix": same, "tokens_total": total, "first_divergence": first_div,
            "max_logprob_gap_before_divergence": max_gap}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--backend", default="CUSTOM")
    ap.add_argument("--num-prompts", type=int, default=4)
    ap.add_argument("--max-tokens", type=int, default=64)
    ap.add_argument("--out", default=None)
    ap.add_argument("--std", type=float, default=0.02, help="redraw weights from N(0, std); 0 keeps vLLM's dummy init")
    ap.add_argument("--max-batched-tokens", type=int, default=None,
                    help="vLLM max_num_batched_tokens (small values mix prompt chunks with decode steps)")
    ap.add_argument("--compare", nargs=2, default=None, help="two result files to compare instead of running")
    args = ap.parse_args()
    if args.compare:
        a, b = (json.loads(Path(f).read_text()) for f in args.compare)
        res = compare(a, b)
    else:
        res = run(args.backend, args.num_prompts, args.max_tokens, args.std, args.max_batched_tokens)
    text = json.dumps(res)
    print(text)
    if args.out:
        Path(args.out).write_text(text)


if __name__ == "__main__":
    main()
