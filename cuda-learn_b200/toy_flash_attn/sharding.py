"""Sharding of a paged-attention batch over the GPUs of one node.

Attention forward is independent per (sequence, kv head), so the work splits with no
exchange step. Ranks first take equal groups of kv heads (with their q heads); when there
are more ranks than kv heads, each head group is further split by sequences, balanced by
attended kv length (longest first, onto the lightest rank). Outputs are reassembled after
an all-gather; nothing is communicated during the forward itself.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .workloads import PagedCase

__all__ = ["Shard", "plan_shards", "shard_case", "reassemble"]


@dataclass(frozen=True)
class Shard:
    rank: int
    kv_heads: tuple[int, int]       # [lo, hi)
    q_heads: tuple[int, int]        # [lo, hi)
    sequences: tuple[int, ...]      # sequence indices of the batch


def plan_shards(kv_lens: list[int], num_q_heads: int, num_kv_heads: int, world: int) -> list[Shard]:
    if world < 1:
        raise ValueError("world must be >= 1")
    group = num_q_heads // num_kv_heads
    head_groups = min(world, num_kv_heads)
    while num_kv_heads % head_groups or world % head_groups:
        head_groups -= 1
    per_group = world // head_groups
    hk = num_kv_heads // head_groups
    shards = []
    for g in range(head_groups):
        loads = [0] * per_group
        members: list[list[int]] = [[] for _ in range(per_group)]
        for b in sorted(range(len(kv_lens)), key=lambda i: -kv_lens[i]):
            j = min(range(per_group), key=lambda r: (loads[r], r))
            loads[j] += kv_lens[b]
            members[j].append(b)
        for j in range(per_group):
            shards.append(Shard(g * per_group + j, (g * hk, (g + 1) * hk), (g * hk * group, (g + 1) * hk * group),
                                tuple(sorted(members[j]))))
    return shards


def shard_case(case: PagedCase, shard: Shard) -> PagedCase:
    """The sub-problem of one rank (q heads, kv heads and sequences of the shard)."""
    seqs = list(shard.sequences)
    klo, khi = shard.kv_heads
    qlo, qhi = shard.q_heads
    cu = case.cu_seqlens_q.tolist()
    rows = [torch.arange(cu[b], cu[b + 1]) for b in seqs]
    idx = torch.cat(rows) if rows else torch.zeros(0, dtype=torch.long)
    q = case.q[idx.to(case.q.device)][:, qlo:qhi].contiguous()
    lens = [cu[b + 1] - cu[b] for b in seqs]
    new_cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32)
    sel = torch.tensor(seqs, dtype=torch.long)
    return PagedCase(
        f"{case.name}[rank {shard.rank}]", q,
        case.k_cache[:, :, klo:khi].contiguous(), case.v_cache[:, :, klo:khi].contiguous(),
        new_cu.to(case.q.device), case.seqused_k[sel.to(case.seqused_k.device)].contiguous(),
        case.block_table[sel.to(case.block_table.device)].contiguous(),
        max(lens) if lens else 0, int(case.seqused_k[sel].max()) if seqs else 0, case.causal, case.window_size,
    )


def reassemble(outputs: list[torch.Tensor], shards: list[Shard], case: PagedCase) -> torch.Tensor:
    """Full ``[total_q, Hq, d]`` output from every rank's shard output."""
    total_q, hq, d = case.q.shape
    full = torch.zeros(total_q, hq, d, dtype=outputs[0].dtype, device=outputs[0].device)
    cu = case.cu_seqlens_q.tolist()
    for out, sh in zip(outputs, shards):
        o = 0
        for b in sh.sequences:
            n = cu[b + 1] - cu[b]
            full[cu[b]:cu[b + 1], sh.q_heads[0]:sh.q_heads[1]] = out[o:o + n]
            o += n
    return full
