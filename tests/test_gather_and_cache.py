"""Bit-exact checks of the paged gather (the kernels' TMA staging path) and of the
KV-cache write kernel."""

from __future__ import annotations

import pytest
import torch

from oracle.paged_attention import gather_kv
from toy_flash_attn import flash_attention_func as faf
from toy_flash_attn.workloads import baseline_config, reference_case

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.int16)


@pytest.mark.parametrize("block_size", [1, 4, 16, 32])
@pytest.mark.parametrize("hd", [64, 128])
def test_gather_bit_exact(block_size, hd):
    case = reference_case([1, 1, 1], [300, 129, 5], num_heads=6, num_kv_heads=3, head_dim=hd, block_size=block_size,
                          seed=block_size)
    c = case.to("cuda")
    k_out, v_out = faf.gather_kv_cu(c.k_cache, c.v_cache, c.seqused_k, c.block_table, c.max_seqlen_k)
    assert torch.equal(_bits(k_out.cpu()), _bits(gather_kv(case.k_cache, case.block_table, case.seqused_k)))
    assert torch.equal(_bits(v_out.cpu()), _bits(gather_kv(case.v_cache, case.block_table, case.seqused_k)))
    assert faf.read_device_error() == 0


@pytest.mark.parametrize("name", ["C2", "C4"])
def test_gather_bit_exact_baseline(name):
    case = baseline_config(name) if name == "C2" else baseline_config(name, batch=6)
    c = case.to("cuda")
    k_out, v_out = faf.gather_kv_cu(c.k_cache, c.v_cache, c.seqused_k, c.block_table, c.max_seqlen_k)
    ref_k = gather_kv(case.k_cache, case.block_table, case.seqused_k)
    assert not torch.isnan(ref_k).any()  # NaN slots lie past kv_len and are never gathered
    assert torch.equal(_bits(k_out.cpu()), _bits(ref_k))
    assert torch.equal(_bits(v_out.cpu()), _bits(gather_kv(case.v_cache, case.block_table, case.seqused_k)))


@pytest.mark.parametrize("hd", [64, 128])
def test_kv_cache_update_matches_eager_scatter(hd):
    g = torch.Generator().manual_seed(0)
    nb, bs, hkv, n = 40, 16, 4, 70
    key = torch.randn(n, hkv, hd, generator=g).to(torch.bfloat16)
    value = torch.randn(n, hkv, hd, generator=g).to(torch.bfloat16)
    slots = torch.randperm(nb * bs, generator=g)[:n]
    slots[::7] = -1  # padding tokens
    kc = torch.randn(nb, bs, hkv, hd, generator=g).to(torch.bfloat16)
    vc = torch.randn(nb, bs, hkv, hd, generator=g).to(torch.bfloat16)
    # reference semantics: impl.py:121-144
    kref, vref = kc.clone(), vc.clone()
    valid = slots >= 0
    kref[slots[valid] // bs, slots[valid] % bs] = key[valid]
    vref[slots[valid] // bs, slots[valid] % bs] = value[valid]
    kd, vd = kc.cuda(), vc.cuda()
    faf.kv_cache_update_cu(key.cuda(), value.cuda(), kd, vd, slots.cuda())
    assert torch.equal(_bits(kd.cpu()), _bits(kref))
    assert torch.equal(_bits(vd.cpu()), _bits(vref))


def test_kv_cache_update_then_decode_reads_it():
    """Write a token through the cache kernel, then attend to it."""
    case = reference_case([1], [33], num_heads=4, num_kv_heads=2, block_size=16, seed=3)
    c = case.to("cuda")
    new_k = torch.randn(1, 2, 64, device="cuda").to(torch.bfloat16)
    new_v = torch.randn(1, 2, 64, device="cuda").to(torch.bfloat16)
    slot = int(case.block_table[0, 2]) * 16 + 1  # position 33 lives in logical block 2, offset 1
    faf.kv_cache_update_cu(new_k, new_v, c.k_cache, c.v_cache, torch.tensor([slot], device="cuda"))
    c.seqused_k[0] = 34
    k_out, _ = faf.gather_kv_cu(c.k_cache, c.v_cache, c.seqused_k, c.block_table, 34)
    assert torch.equal(_bits(k_out[33:34].cpu()), _bits(new_k.cpu()))
