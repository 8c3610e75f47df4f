"""Replay of dumped attention calls.

With ``TOY_FLASH_ATTN_DUMP_DIR`` set, every paged call saves its inputs and result as
``NNNNN_with_block.pt`` (PyTorch path) or ``NNNNN_with_block_cu.pt`` (sm_100a path); the
payload keys are those of the reference's dumps (``flash_attention_func.py:89-99,393-407``
and ``:583-597``). This module loads such a file and runs the same call again, so a call
captured inside vLLM can be re-checked offline, as the reference's ``replay_dump_close``
does (``toy_flash_attn/test_utils.py:87-104,332-356``).
"""

from __future__ import annotations

from pathlib import Path

import torch

from .flash_attention_func import flash_attn_varlen_func

REPLAY_KEYS = frozenset({
    "q", "k", "v", "max_seqlen_q", "cu_seqlens_q", "max_seqlen_k", "seqused_k", "causal", "window_size",
    "block_table", "result",
})


def load_dump(path: str | Path) -> dict:
    """Loads a dump onto the CPU; raises ``AssertionError`` naming missing keys."""
    path = Path(path)
    payload = torch.load(path, map_location="cpu", weights_only=False)
    missing = sorted(REPLAY_KEYS - payload.keys())
    if missing:
        raise AssertionError(f"Replay dump {path} missing keys: {missing}")
    return payload


def replay(path: str | Path, device: str | torch.device = "cuda") -> tuple[torch.Tensor, torch.Tensor]:
    """Runs the dumped call again on ``device`` through ``flash_attn_varlen_func`` (so
    ``TOY_FLASH_ATTN_USE`` picks the path, as for any call) and returns
    ``(new_output, dumped_result)``, both on ``device``."""
    p = load_dump(path)
    dev = torch.device(device)
    out = flash_attn_varlen_func(
        q=p["q"].to(dev), k=p["k"].to(dev), v=p["v"].to(dev),
        max_seqlen_q=p["max_seqlen_q"], cu_seqlens_q=p["cu_seqlens_q"].to(dev),
        max_seqlen_k=p["max_seqlen_k"], cu_seqlens_k=None, seqused_k=p["seqused_k"].to(dev),
        causal=p["causal"], window_size=p["window_size"], block_table=p["block_table"].to(dev),
    )
    return out, p["result"].to(dev)
