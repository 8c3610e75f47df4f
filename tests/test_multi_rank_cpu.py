"""Multi-rank host logic on the CPU (gloo, world sizes 2 and 4): every rank computes its
shard with the oracle, the outputs are all-gathered and reassembled, and rank 0 checks
the result against the unsharded oracle. No GPU involved."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from toy_flash_attn.sharding import plan_shards, reassemble, shard_case
from toy_flash_attn.workloads import baseline_config, reference_case


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _make_case(kind: str):
    if kind == "c4":
        return baseline_config("C4", batch=6, kv_range=(50, 400))
    return reference_case([1, 3, 1, 2, 1], [90, 40, 300, 17, 128], num_heads=8, num_kv_heads=2, causal=True,
                          block_size=16, seed=4)


def _worker(rank: int, world: int, port: int, kind: str, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        from pathlib import Path

        sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
        from oracle.paged_attention import paged_attention_oracle

        case = _make_case(kind)
        shards = plan_shards(case.seqused_k.tolist(), case.q.shape[1], case.k_cache.shape[2], world)
        sub = shard_case(case, shards[rank])
        out, _ = paged_attention_oracle(sub.q, sub.k_cache, sub.v_cache, sub.cu_seqlens_q, sub.seqused_k,
                                        sub.block_table, sub.causal, sub.window_size)
        sizes = [None] * world
        dist.all_gather_object(sizes, tuple(out.shape))
        padded = torch.zeros((max(s[0] for s in sizes),) + tuple(out.shape[1:]))
        padded[: out.shape[0]] = out
        gathered = [torch.zeros_like(padded) for _ in range(world)]
        dist.all_gather(gathered, padded)
        if rank == 0:
            outs = [g[: s[0]] for g, s in zip(gathered, sizes)]
            full = reassemble(outs, shards, case)
            ref, _ = paged_attention_oracle(case.q, case.k_cache, case.v_cache, case.cu_seqlens_q, case.seqused_k,
                                            case.block_table, case.causal, case.window_size)
            result_q.put(float((full - ref).abs().max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world, kind", [(2, "c4"), (4, "mixed"), (2, "mixed")])
def test_sharded_forward_reassembles_to_full_result(world, kind):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, kind, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert q.get(timeout=5) == 0.0


def test_plan_shards_heads_then_batch():
    s = plan_shards([100, 50, 400, 10], num_q_heads=8, num_kv_heads=2, world=4)
    assert [x.kv_heads for x in s] == [(0, 1), (0, 1), (1, 2), (1, 2)]
    assert [x.q_heads for x in s] == [(0, 4), (0, 4), (4, 8), (4, 8)]
    for g in (s[:2], s[2:]):
        assert sorted(b for x in g for b in x.sequences) == [0, 1, 2, 3]
    s8 = plan_shards([1] * 3, num_q_heads=32, num_kv_heads=8, world=8)
    assert [x.kv_heads for x in s8] == [(i, i + 1) for i in range(8)]
    assert all(x.sequences == (0, 1, 2) for x in s8)
