"""Pins the CPU oracle to outputs of the reference's own paged path.

The fixtures in ``tests/golden`` were produced by running the reference function
``flash_attn_varlen_with_block`` (``flash_attention_func.py:314-408``) itself, see
``tests/golden/make_golden.py``. No GPU needed.
"""

from __future__ import annotations

import pytest
import torch

from conftest import golden_files, load_golden
from oracle.paged_attention import gather_kv, paged_attention_oracle, reference_port

GOLDEN = golden_files()


def test_golden_fixtures_present():
    assert len(GOLDEN) >= 20


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_oracle_matches_reference_fp32(path):
    g = load_golden(path)
    out, lse = paged_attention_oracle(
        g["q"], g["k"], g["v"], g["cu_seqlens_q"], g["seqused_k"], g["block_table"], g["causal"], g["window_size"]
    )
    ref = g["out_ref_fp32"]
    assert out.shape == ref.shape
    assert torch.isfinite(out).all()
    torch.testing.assert_close(out, ref.float(), atol=2e-5, rtol=2e-5)
    assert torch.isfinite(lse).all()


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_reference_port_matches_reference_bf16(path):
    g = load_golden(path)
    out = reference_port(
        g["q"], g["k"], g["v"], g["max_seqlen_q"], g["cu_seqlens_q"], g["max_seqlen_k"], g["seqused_k"],
        g["causal"], g["window_size"], g["block_table"],
    )
    # same torch ops in the same order as the reference: identical up to CPU-kernel ordering
    torch.testing.assert_close(out.float(), g["out_ref_bf16"].float(), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("path", GOLDEN[:6], ids=[p.stem for p in GOLDEN[:6]])
def test_oracle_lse_is_logsumexp(path):
    """The LSE the reference never returns: log of the softmax denominator of the same
    masked, scaled scores (checked by recomputing one row densely)."""
    g = load_golden(path)
    out, lse = paged_attention_oracle(
        g["q"], g["k"], g["v"], g["cu_seqlens_q"], g["seqused_k"], g["block_table"], g["causal"], g["window_size"]
    )
    K = gather_kv(g["k"], g["block_table"], g["seqused_k"]).float()
    kv0 = int(g["seqused_k"][0])
    q0 = g["q"][0].float()  # first token of sequence 0
    hq, hkv = g["q"].shape[1], g["k"].shape[2]
    q_len0 = int(g["cu_seqlens_q"][1] - g["cu_seqlens_q"][0])
    off = kv0 - q_len0
    wl, wr = (-1, -1) if g["window_size"] is None else g["window_size"]
    lo = 0 if wl < 0 else max(0, off - wl)
    hi = off if g["causal"] else (kv0 - 1 if wr < 0 else off + wr)
    hi = min(hi, kv0 - 1)
    for h in range(hq):
        s = (K[lo:hi + 1, h // (hq // hkv)] @ q0[h]) / (g["q"].shape[2] ** 0.5)
        torch.testing.assert_close(lse[0, h], torch.logsumexp(s, 0), atol=1e-5, rtol=1e-5)


def test_gather_kv_restates_reference_indexing():
    g = load_golden(GOLDEN[0])
    dense = gather_kv(g["k"], g["block_table"], g["seqused_k"])
    bs = g["k"].shape[1]
    rows = []
    for b in range(g["seqused_k"].numel()):
        for t in range(int(g["seqused_k"][b])):
            rows.append(g["k"][int(g["block_table"][b][t // bs]), t % bs])
    assert torch.equal(dense, torch.stack(rows))
