"""The backend inside vLLM, as the reference proves its own
(flash_attention_backend/test_self_flash_attn_backend.py:83-147): a Qwen2.5-0.5B-shaped
model with seeded random weights (the reference's checkpoints are not available offline)
generates greedily with the backend registered as CUSTOM, and the same run with vLLM's
TRITON_ATTN backend is the comparison. Each run is a child process (one vLLM engine per
process). Checks: the custom attention path was called, and up to the first token where
the two greedy sequences differ (a near-tie that bf16 rounding can decide either way), the
log-probabilities of the generated tokens agree within 5e-3."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parent.parent
LOGPROB_TOL = 5e-3


def _run(backend: str, out: Path) -> dict:
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(REPO / "cuda-learn_b200"), str(REPO), env.get("PYTHONPATH", "")])
    cmd = [sys.executable, "-m", "toy_flash_attn.vllm_e2e", "--backend", backend, "--num-prompts", "2",
           "--max-tokens", "8", "--out", str(out)]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, f"{backend} run failed:\n{res.stdout[-2000:]}\n{res.stderr[-4000:]}"
    return json.loads(out.read_text())


def test_vllm_custom_backend_matches_triton(tmp_path):
    pytest.importorskip("vllm")
    from toy_flash_attn.vllm_e2e import compare

    custom = _run("CUSTOM", tmp_path / "custom.json")
    triton = _run("TRITON_ATTN", tmp_path / "triton.json")
    assert custom["custom_attention_calls"] > 0, "vLLM did not call the custom backend"
    assert triton["custom_attention_calls"] == 0
    cmp = compare(custom, triton)
    assert cmp["tokens_identical_prefix"] >= 1, cmp
    assert cmp["max_logprob_gap_before_divergence"] <= LOGPROB_TOL, cmp
