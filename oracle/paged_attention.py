"""CPU oracle for the paged-KV attention forward.

TEST INFRASTRUCTURE ONLY. Nothing in the product path imports this module: only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` use it, and there only as the checker or as the timed CPU
baseline. The CUDA path never falls back to it.

It restates the reference's pure-PyTorch paged path,
``flash_attention_backend/toy_flash_attn/flash_attention_func.py:314-408``
(``flash_attn_varlen_with_block``), in two forms:

* :func:`paged_attention_oracle` -- vectorised, fp32 math on the (bf16) inputs, plus the
  natural-log LSE which the reference never returns. This is the checker.
* :func:`reference_port` -- the same steps in the same order and with the same cost
  structure as the reference (a per-token Python list for the page gather, a per-row
  Python loop for the mask, math in the input dtype). This is what the CPU baseline
  times, standing in for ``TOY_FLASH_ATTN_USE=reference``.

Both are pinned to outputs of the reference function itself, captured by
``tests/golden/make_golden.py`` into ``tests/golden/*.pt``.

Semantics kept from the reference (line numbers in ``flash_attention_func.py``):

* gather: token ``t`` of sequence ``b`` lives at ``k[block_table[b][t // bs], t % bs]``
  (``:343-346``), for ``t < seqused_k[b]``;
* GQA: q head ``qh`` reads kv head ``qh // (Hq // Hkv)`` (``:359-363``);
* scale: ``S = Q K^T / sqrt(head_dim)`` unless a scale is given (``:365``);
* window: ``None`` or ``(-1, -1)`` means unbounded; ``causal`` forces the right window
  to 0 (``:367-371``); query row ``i`` of a sequence sees kv positions
  ``[max(0, i + off - wl), min(kv_len, i + off + 1 + wr))`` with ``off = kv_len - q_len``
  (q and kv are tail aligned, ``:372-376``).

One deliberate extension: a single ``-1`` inside an otherwise bounded window, e.g.
``(-1, 0)``, is treated as unbounded on that side (the convention of the reference's
CUDA kernels, ``v8/flash_attn_func.cu:369-373``); the Python reference only recognises
the pair ``(-1, -1)``. Rows with no visible key produce 0 output and ``-inf`` LSE (the
reference's CUDA kernels write 0, ``v8/flash_attn_func.cu:679``; its Python path
produces NaN there).
"""

from __future__ import annotations

import math

import torch

__all__ = [
    "effective_window",
    "gather_kv",
    "paged_attention_oracle",
    "reference_port",
]


def effective_window(window_size, causal: bool, kv_len: int) -> tuple[int, int]:
    """Window bounds as used for one sequence (``flash_attention_func.py:367-371``)."""
    if window_size is None:
        wl, wr = -1, -1
    else:
        wl, wr = int(window_size[0]), int(window_size[1])
    wl = kv_len if wl < 0 else wl
    wr = kv_len if wr < 0 else wr
    if causal:
        wr = 0
    return wl, wr


def gather_kv(cache: torch.Tensor, block_table: torch.Tensor, seqused_k: torch.Tensor) -> torch.Tensor:
    """Dense ``[sum(kv_len), Hkv, d]`` copy of the paged cache, in sequence order.

    Bit-exact restatement of ``flash_attention_func.py:343-346``.
    """
    bs = cache.shape[1]
    out = []
    for b in range(seqused_k.numel()):
        kv_len = int(seqused_k[b])
        t = torch.arange(kv_len)
        phys = block_table[b].long()[t // bs]
        out.append(cache[phys, t % bs])
    if not out:
        return cache.new_zeros((0,) + tuple(cache.shape[2:]))
    return torch.cat(out, 0)


def paged_attention_oracle(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    seqused_k: torch.Tensor,
    block_table: torch.Tensor,
    causal: bool = False,
    window_size=None,
    softmax_scale: float | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 paged attention with LSE. Inputs may live on any device; math runs on CPU.

    Returns ``(out [T_q, Hq, d] fp32, lse [T_q, Hq] fp32 natural log)``.
    """
    q = q.detach().cpu().float()
    k_cache = k_cache.detach().cpu()
    v_cache = v_cache.detach().cpu()
    cu = cu_seqlens_q.detach().cpu().long()
    used = seqused_k.detach().cpu().long()
    bt = block_table.detach().cpu().long()
    total_q, hq, d = q.shape
    hkv = k_cache.shape[2]
    if hq % hkv != 0:
        raise ValueError(f"GQA requires q_heads divisible by kv_heads, got {hq} and {hkv}")
    group = hq // hkv
    scale = (1.0 / math.sqrt(d)) if softmax_scale is None else float(softmax_scale)
    bs = k_cache.shape[1]
    out = torch.zeros(total_q, hq, d, dtype=torch.float32)
    lse = torch.full((total_q, hq), float("-inf"), dtype=torch.float32)
    for b in range(used.numel()):
        q0, q1 = int(cu[b]), int(cu[b + 1])
        q_len, kv_len = q1 - q0, int(used[b])
        if q_len == 0 or kv_len == 0:
            continue  # nothing visible: output 0, LSE -inf
        t = torch.arange(kv_len)
        phys = bt[b][t // bs] if kv_len > 0 else t
        K = k_cache[phys, t % bs].float()  # [kv, Hkv, d]
        V = v_cache[phys, t % bs].float()
        heads = torch.arange(hq) // group
        K = K[:, heads]  # [kv, Hq, d]
        V = V[:, heads]
        Q = q[q0:q1]  # [q_len, Hq, d]
        S = torch.einsum("qhd,khd->hqk", Q, K) * scale
        wl, wr = effective_window(window_size, causal, kv_len)
        off = kv_len - q_len
        i = torch.arange(q_len).unsqueeze(1)
        j = torch.arange(kv_len).unsqueeze(0)
        visible = (j >= i + off - wl) & (j <= i + off + wr) & (j >= 0) & (j < kv_len)
        S = S.masked_fill(~visible.unsqueeze(0), float("-inf"))
        m = S.amax(dim=-1, keepdim=True)
        m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
        P = torch.exp(S - m_safe)
        den = P.sum(dim=-1, keepdim=True)
        O = torch.einsum("hqk,khd->qhd", P / torch.where(den > 0, den, torch.ones_like(den)), V)
        out[q0:q1] = O
        row_lse = (m_safe + torch.log(den)).squeeze(-1).transpose(0, 1)  # [q_len, Hq]
        lse[q0:q1] = torch.where(den.squeeze(-1).transpose(0, 1) > 0, row_lse, torch.full_like(row_lse, float("-inf")))
    return out, lse


def reference_port(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    max_seqlen_q: int,
    cu_seqlens_q: torch.Tensor,
    max_seqlen_k: int,
    seqused_k: torch.Tensor,
    causal=False,
    window_size=None,
    block_table=None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Step-for-step restatement of ``flash_attn_varlen_with_block``
    (``flash_attention_func.py:314-392``), without its debug hooks.

    Math runs in the dtype of the inputs, as in the reference. Used as the timed CPU
    baseline; the checker is :func:`paged_attention_oracle`.
    """
    assert block_table is not None
    if out is None:
        out = torch.empty_like(q)
    block_size = k.shape[1]
    for batch_id in range(len(seqused_k)):
        q_start = cu_seqlens_q[batch_id].item()
        q_end = cu_seqlens_q[batch_id + 1].item()
        kv_len = seqused_k[batch_id].item()
        Q = q[q_start:q_end]
        # per-token page lookup, as a Python list like the reference (:343-344)
        pages = [block_table[batch_id][pos // block_size] for pos in range(kv_len)]
        slots = [pos % block_size for pos in range(kv_len)]
        K = k[pages, slots]
        V = v[pages, slots]
        n_q, n_kv = Q.shape[1], K.shape[1]
        if n_q % n_kv != 0:
            raise ValueError(f"GQA requires q_heads divisible by kv_heads, got {n_q} and {n_kv}")
        if n_q != n_kv:
            idx = torch.arange(n_q, device=q.device) // (n_q // n_kv)
            K = K[:, idx, :]
            V = V[:, idx, :]
        S = Q.transpose(0, 1).matmul(K.permute(1, 2, 0)) / float(q.shape[2] ** 0.5)
        win = window_size
        if win is None or tuple(win) == (-1, -1):
            win = (kv_len, kv_len)
        if causal:
            win = (win[0], 0)
        hidden = torch.ones(S.shape[1:], dtype=torch.bool, device=S.device)
        shift = K.shape[0] - Q.shape[0]
        for row, line in enumerate(hidden):  # per-row Python loop, as the reference (:374-376)
            line[max(0, row + shift - win[0]):min(kv_len, row + shift + 1 + win[1])] = False
        P = S.masked_fill(hidden, float("-inf")).softmax(2)
        out[q_start:q_end] = P.matmul(V.transpose(0, 1)).transpose(0, 1)
    return out
