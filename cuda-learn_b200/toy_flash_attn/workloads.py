"""Seeded synthetic paged-attention workloads.

Two families:

* :func:`reference_case` restates the reference's own test fixtures
  (``flash_attention_backend/toy_flash_attn/test_utils.py:106-192``): dense
  ``randn`` q/k/v per sequence copied into a zero-filled paged cache whose block table is
  the non-identity "even ids first, then odd ids" permutation, unused table entries -1.
* :func:`baseline_config` builds the five benchmark configurations C1-C5 (GPT-2 causal
  prefill, Qwen GQA decode, Qwen varlen prefill, sliding-window decode, large-batch
  decode) with N(0, 1) bf16 values, random non-identity block tables and, where the
  configuration asks for it, NaN-filled unused cache slots. Sizes can be reduced with
  keyword overrides for tests.

All randomness comes from an explicit ``torch.Generator`` seeded per case.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch

__all__ = ["PagedCase", "reference_case", "baseline_config", "c5_kv_lengths", "BASELINE_CONFIGS", "kv_bytes",
           "prefill_flops", "compact_sample", "verify_sequences", "REFERENCE_OP_CASES", "reference_op_case"]


@dataclass
class PagedCase:
    name: str
    q: torch.Tensor            # [total_q, Hq, d]
    k_cache: torch.Tensor      # [num_blocks, block_size, Hkv, d]
    v_cache: torch.Tensor
    cu_seqlens_q: torch.Tensor  # int32 [batch + 1]
    seqused_k: torch.Tensor     # int32 [batch]
    block_table: torch.Tensor   # int32 [batch, max_blocks]
    max_seqlen_q: int
    max_seqlen_k: int
    causal: bool
    window_size: tuple[int, int] | None

    @property
    def batch(self) -> int:
        return self.seqused_k.numel()

    def to(self, device) -> "PagedCase":
        return replace(
            self,
            q=self.q.to(device),
            k_cache=self.k_cache.to(device),
            v_cache=self.v_cache.to(device),
            cu_seqlens_q=self.cu_seqlens_q.to(device),
            seqused_k=self.seqused_k.to(device),
            block_table=self.block_table.to(device),
        )

    def kwargs(self) -> dict:
        """Arguments of ``flash_attn_varlen_func`` (paged path)."""
        return dict(
            q=self.q, k=self.k_cache, v=self.v_cache, max_seqlen_q=self.max_seqlen_q,
            cu_seqlens_q=self.cu_seqlens_q, max_seqlen_k=self.max_seqlen_k, cu_seqlens_k=None,
            seqused_k=self.seqused_k, causal=self.causal, window_size=self.window_size,
            block_table=self.block_table,
        )


def _cu(lens: list[int]) -> torch.Tensor:
    out = [0]
    for n in lens:
        out.append(out[-1] + n)
    return torch.tensor(out, dtype=torch.int32)


def reference_case(
    q_lens: list[int],
    k_lens: list[int] | None = None,
    *,
    num_heads: int = 2,
    num_kv_heads: int | None = None,
    head_dim: int = 64,
    dtype: torch.dtype = torch.bfloat16,
    seed: int = 0,
    causal: bool = False,
    window_size: tuple[int, int] | None = None,
    block_size: int = 4,
    name: str = "reference_case",
) -> PagedCase:
    """Restatement of ``make_inputs`` + ``make_block_cache`` (``test_utils.py:106-192``)."""
    k_lens = list(q_lens) if k_lens is None else list(k_lens)
    num_kv_heads = num_heads if num_kv_heads is None else num_kv_heads
    g = torch.Generator().manual_seed(seed)
    total_q, total_k = sum(q_lens), sum(k_lens)
    q = torch.randn(total_q, num_heads, head_dim, generator=g).to(dtype)
    k = torch.randn(total_k, num_kv_heads, head_dim, generator=g).to(dtype)
    v = torch.randn(total_k, num_kv_heads, head_dim, generator=g).to(dtype)
    blocks = [(n + block_size - 1) // block_size for n in k_lens]
    total_blocks = max(sum(blocks), 1)
    k_cache = torch.zeros(total_blocks, block_size, num_kv_heads, head_dim, dtype=dtype)
    v_cache = torch.zeros_like(k_cache)
    table = torch.full((len(k_lens), max(max(blocks), 1)), -1, dtype=torch.int32)
    ids = list(range(total_blocks))
    ids = ids[::2] + ids[1::2]  # non-identity mapping, test_utils.py:174-175
    nxt, start = 0, 0
    for b, n in enumerate(k_lens):
        for lb in range(blocks[b]):
            phys = ids[nxt]
            nxt += 1
            table[b, lb] = phys
            t0 = start + lb * block_size
            t1 = min(t0 + block_size, start + n)
            k_cache[phys, : t1 - t0] = k[t0:t1]
            v_cache[phys, : t1 - t0] = v[t0:t1]
        start += n
    return PagedCase(name, q, k_cache, v_cache, _cu(q_lens), torch.tensor(k_lens, dtype=torch.int32), table,
                     max(q_lens), max(k_lens), causal, window_size)


# --------------------------------------------------------------------------------------
# Benchmark configurations
# --------------------------------------------------------------------------------------
BASELINE_CONFIGS = {
    "C1": "gpt2_causal_prefill: b1 L128 12q/12kv d64 bs16 pool64 causal",
    "C2": "qwen_gqa_decode: b1 kv2048 14q/2kv d64 bs16 pool4096 causal",
    "C3": "qwen_varlen_prefill: b4 L[512,384,256,128] 14q/2kv d64 bs16 causal",
    "C4": "sliding_window_decode: b16 kv U[2048,8192] window(1024,0) 32q/8kv d64 bs16 NaN slots",
    "C5": "large_batch_decode: b256 kv logU[1024,32768] 32q/8kv d128 bs16 pool 2^21 blocks",
    # scaled prefill points (not BASELINE configurations): long causal prompts that make
    # the prefill kernel compute-bound, to show tensor-pipe utilisation
    "P1": "scaled_prefill_d128: b1 L8192 32q/8kv d128 bs16 causal",
    "P2": "scaled_prefill_d64: b4 L4096 14q/2kv d64 bs16 causal",
}


def _fill_randn_(t: torch.Tensor, g: torch.Generator, chunk: int = 1 << 28) -> torch.Tensor:
    flat = t.view(-1)
    for s in range(0, flat.numel(), chunk):
        e = min(s + chunk, flat.numel())
        flat[s:e] = torch.randn(e - s, generator=g, device=t.device, dtype=t.dtype)
    return t


def _non_identity_perm(n: int, g: torch.Generator, device) -> torch.Tensor:
    perm = torch.randperm(n, generator=g, device=device)
    if n > 1 and bool((perm == torch.arange(n, device=device)).all()):
        perm = torch.roll(perm, 1)
    return perm


def c5_kv_lengths(batch: int = 256, seed: int = 5, kv_range: tuple[int, int] = (1024, 32768)) -> list[int]:
    """Log-uniform kv lengths of C5, drawn on the CPU (identical for every device)."""
    gc = torch.Generator().manual_seed(seed)
    lo, hi = kv_range
    u = torch.rand(batch, generator=gc, dtype=torch.float64)
    return torch.exp(math.log(lo) + u * (math.log(hi) - math.log(lo))).floor().to(torch.int64).tolist()


def baseline_config(
    name: str,
    device="cpu",
    seed: int | None = None,
    *,
    batch: int | None = None,
    num_blocks: int | None = None,
    kv_range: tuple[int, int] | None = None,
    kv_heads: int | None = None,
    q_heads: int | None = None,
    value_seed: int | None = None,
) -> PagedCase:
    """Builds configuration C1..C5. Overrides shrink a configuration for tests
    (``batch``, pool ``num_blocks``, ``kv_range``) or shard it (``kv_heads``/``q_heads``).

    Lengths and block tables are drawn from a CPU generator seeded with ``seed`` (the
    same on every device); q/K/V values from a generator on ``device`` seeded with
    ``value_seed`` (default ``seed``), so the shards of one configuration can share
    lengths and tables but hold different values."""
    name = name.upper()
    seed = {"C1": 1, "C2": 2, "C3": 3, "C4": 4, "C5": 5, "P1": 11, "P2": 12}[name] if seed is None else seed
    dev = torch.device(device)
    gc = torch.Generator().manual_seed(seed)
    bs = 16
    if name == "C1":
        hq, hkv, d = 12, 12, 64
        q_lens = kv_lens = [128]
        nb = num_blocks or 64
        causal, window, nan_fill = True, None, False
    elif name == "C2":
        hq, hkv, d = 14, 2, 64
        q_lens, kv_lens = [1], [2048]
        nb = num_blocks or 4096
        causal, window, nan_fill = True, None, False
    elif name == "C3":
        hq, hkv, d = 14, 2, 64
        q_lens = kv_lens = [512, 384, 256, 128]
        nb = num_blocks or 256
        causal, window, nan_fill = True, None, False
    elif name == "P1":
        hq, hkv, d = 32, 8, 128
        q_lens = kv_lens = [8192] * (batch or 1)
        nb = num_blocks or sum(n // bs for n in kv_lens) + 64
        causal, window, nan_fill = True, None, False
    elif name == "P2":
        hq, hkv, d = 14, 2, 64
        q_lens = kv_lens = [4096] * (batch or 4)
        nb = num_blocks or sum(n // bs for n in kv_lens) + 64
        causal, window, nan_fill = True, None, False
    elif name == "C4":
        hq, hkv, d = 32, 8, 64
        B = batch or 16
        lo, hi = kv_range or (2048, 8192)
        kv_lens = torch.randint(lo, hi + 1, (B,), generator=gc).tolist()
        q_lens = [1] * B
        nb = num_blocks or (sum((n + bs - 1) // bs for n in kv_lens) + 64)
        causal, window, nan_fill = True, (1024, 0), True
    elif name == "C5":
        hq, hkv, d = 32, 8, 128
        B = batch or 256
        kv_lens = c5_kv_lengths(B, seed, kv_range or (1024, 32768))
        q_lens = [1] * B
        nb = num_blocks or (1 << 21)
        causal, window, nan_fill = True, None, False
    else:
        raise KeyError(name)
    need = [(n + bs - 1) // bs for n in kv_lens]
    if nb < sum(need):
        raise ValueError(f"pool of {nb} blocks is smaller than the {sum(need)} live blocks")
    ids = _non_identity_perm(nb, gc, "cpu")[: sum(need)].to(torch.int32)
    table = torch.full((len(kv_lens), max(need)), -1, dtype=torch.int32)
    o = 0
    for b, n in enumerate(need):
        table[b, :n] = ids[o:o + n]
        o += n
    if kv_heads is not None:
        hq, hkv = (q_heads if q_heads is not None else hq * kv_heads // hkv), kv_heads
    g = torch.Generator(device=dev).manual_seed((seed if value_seed is None else value_seed) + 1000)
    total_q = sum(q_lens)
    q = _fill_randn_(torch.empty(total_q, hq, d, dtype=torch.bfloat16, device=dev), g)
    k_cache = _fill_randn_(torch.empty(nb, bs, hkv, d, dtype=torch.bfloat16, device=dev), g)
    v_cache = _fill_randn_(torch.empty_like(k_cache), g)
    table = table.to(dev)
    if nan_fill:
        live = torch.zeros(nb, dtype=torch.bool, device=dev)
        live[table[table >= 0].long()] = True
        k_cache[~live] = float("nan")
        v_cache[~live] = float("nan")
        for b, n in enumerate(kv_lens):
            r = n % bs
            if r:
                last = int(table[b, (n - 1) // bs])
                k_cache[last, r:] = float("nan")
                v_cache[last, r:] = float("nan")
    return PagedCase(name, q, k_cache, v_cache, _cu(q_lens).to(dev), torch.tensor(kv_lens, dtype=torch.int32,
                     device=dev), table, max(q_lens), max(kv_lens), causal, window)


def attended(case: PagedCase) -> list[list[int]]:
    """Per sequence, the number of visible kv positions of every query row."""
    cu = case.cu_seqlens_q.tolist()
    used = case.seqused_k.tolist()
    wl, wr = (-1, -1) if case.window_size is None else case.window_size
    out = []
    for b, kv_len in enumerate(used):
        q_len = cu[b + 1] - cu[b]
        off = kv_len - q_len
        rows = []
        for i in range(q_len):
            lo = 0 if wl < 0 else max(0, i + off - wl)
            hi = (i + off) if case.causal else (kv_len - 1 if wr < 0 else i + off + wr)
            hi = min(kv_len - 1, hi)
            rows.append(max(0, hi - lo + 1))
        out.append(rows)
    return out


def kv_bytes(case: PagedCase) -> int:
    """Algorithmic decode bytes: K and V of every attended position, once per kv head
    (the GQA group shares the read)."""
    hkv, d = case.k_cache.shape[2], case.k_cache.shape[3]
    total = 0
    for rows in attended(case):
        total += max(rows) if rows else 0
    return total * hkv * d * 2 * 2


def prefill_flops(case: PagedCase) -> int:
    """4 * d * Hq * (number of unmasked (query, key) pairs)."""
    hq, d = case.q.shape[1], case.q.shape[2]
    return 4 * d * hq * sum(sum(rows) for rows in attended(case))


def compact_sample(case: PagedCase, seqs: list[int], device=None) -> PagedCase:
    """The sequences ``seqs`` of ``case`` as a case of their own: q rows, lengths and only
    their live cache blocks, renumbered densely (block i of the sample is the i-th live
    block of the listed sequences, in order). The gather runs where ``case`` lives; the
    result is moved to ``device`` (default: stays there). Used to check a sample of a
    large call against a CPU reference without copying its whole pool."""
    dev = case.q.device
    cu = case.cu_seqlens_q.tolist()
    used = case.seqused_k.tolist()
    bs = case.k_cache.shape[1]
    need = [(used[b] + bs - 1) // bs for b in seqs]
    rows = [case.block_table[b, :n].long() for b, n in zip(seqs, need)]
    ids = torch.cat(rows) if rows else torch.empty(0, dtype=torch.long, device=dev)
    k = case.k_cache[ids]
    v = case.v_cache[ids]
    if k.shape[0] == 0:
        k = torch.zeros((1,) + tuple(case.k_cache.shape[1:]), dtype=case.k_cache.dtype, device=dev)
        v = torch.zeros_like(k)
    table = torch.full((len(seqs), max(max(need, default=1), 1)), -1, dtype=torch.int32)
    o = 0
    for i, n in enumerate(need):
        table[i, :n] = torch.arange(o, o + n, dtype=torch.int32)
        o += n
    q = torch.cat([case.q[cu[b]:cu[b + 1]] for b in seqs]) if seqs else case.q[:0]
    q_lens = [cu[b + 1] - cu[b] for b in seqs]
    out = PagedCase(f"{case.name}[{len(seqs)} seqs]", q, k, v, _cu(q_lens), torch.tensor([used[b] for b in seqs],
                    dtype=torch.int32), table, max(q_lens, default=0), max((used[b] for b in seqs), default=0),
                    case.causal, case.window_size)
    return out.to(device if device is not None else dev)


def verify_sequences(kv_lens: list[int], n_longest: int = 16, n_random: int = 16, seed: int = 77) -> list[int]:
    """Sequence indices of the verification sample of a large decode call: the
    ``n_longest`` longest sequences plus ``n_random`` others drawn with a fixed seed,
    sorted."""
    order = sorted(range(len(kv_lens)), key=lambda b: (-kv_lens[b], b))
    longest = order[:n_longest]
    rest = order[n_longest:]
    g = torch.Generator().manual_seed(seed)
    pick = torch.randperm(len(rest), generator=g)[:n_random].tolist()
    return sorted(longest + [rest[i] for i in pick])


# The reference's op-benchmark cases (flash_attention_backend/bench/op/cases_op.py:20-141):
# name -> (q_lens, k_lens, num_heads, num_kv_heads, head_dim, causal, window_size, seed); its
# bench builds them with make_block_cache at block_size 16 (bench_attention_op.py:120-125).
REFERENCE_OP_CASES = {
    "qwen_like_b1_s128_h64": ([1], [128], 14, 2, 64, True, None, 0),
    "qwen_like_b4_s128_h64": ([1] * 4, [128] * 4, 14, 2, 64, True, None, 0),
    "qwen_like_b1_s512_h64": ([1], [512], 14, 2, 64, True, None, 0),
    "qwen_like_b4_s512_h64": ([1] * 4, [512] * 4, 14, 2, 64, True, None, 0),
    "qwen_like_b1_s2048_h64": ([1], [2048], 14, 2, 64, True, None, 1),
    "mha_b1_s2048_h64_h14_kv14": ([1], [2048], 14, 14, 64, True, None, 1),
    "single_head_b1_s2048_h64_h1_kv1": ([1], [2048], 1, 1, 64, True, None, 1),
    "gpt2_like_b1_s128_h64": ([1], [128], 12, 12, 64, True, None, 0),
    "gqa_case_b1_s128": ([1], [128], 8, 2, 64, True, (64, 0), 7),
    "gqa_case_b4_s512": ([1] * 4, [512, 384, 512, 256], 8, 2, 64, True, None, 9),
}


def reference_op_case(name: str) -> PagedCase:
    q_lens, k_lens, hq, hkv, d, causal, window, seed = REFERENCE_OP_CASES[name]
    return reference_case(q_lens, k_lens, num_heads=hq, num_kv_heads=hkv, head_dim=d, causal=causal,
                          window_size=window, block_size=16, seed=seed, name=name)
