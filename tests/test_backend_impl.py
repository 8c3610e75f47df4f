"""The vLLM-facing layer: ``ToyFlashAttentionBackend``, ``ToyFlashAttentionImpl`` and the
dump / replay path.

Mirrors what the reference checks at this layer: backend registration under ``CUSTOM``
(``tests/test_self_flash_attn_backend.py:12-15``), the impl's constructor guards and
``forward`` contract (``toy_flash_attn/impl.py:16-119``), ``do_kv_cache_update`` slot
semantics (``impl.py:121-144``), and replay of dumped calls
(``toy_flash_attn/test_utils.py:87-104,332-356``). The CPU tests run the
``TOY_FLASH_ATTN_USE=reference`` path; the GPU tests run the sm_100a kernels.
"""

from __future__ import annotations

import re
from types import SimpleNamespace

import pytest
import torch

from oracle.paged_attention import paged_attention_oracle
from toy_flash_attn.workloads import reference_case

OUT_TOL = 2e-2

backend = pytest.importorskip("toy_flash_attn.backend")
impl_mod = pytest.importorskip("toy_flash_attn.impl")
from toy_flash_attn import replay as replay_mod  # noqa: E402
from vllm.v1.attention.backend import AttentionType  # noqa: E402

Backend = backend.ToyFlashAttentionBackend
Impl = impl_mod.ToyFlashAttentionImpl
Metadata = backend.ToyFlashAttentionMetadata


def _metadata(case, causal=None):
    n = case.q.shape[0]
    return Metadata(
        num_actual_tokens=n, max_query_len=case.max_seqlen_q, query_start_loc=case.cu_seqlens_q,
        max_seq_len=case.max_seqlen_k, seq_lens=case.seqused_k, block_table=case.block_table,
        slot_mapping=torch.zeros(n, dtype=torch.int64, device=case.q.device),
        causal=case.causal if causal is None else causal,
    )


def _oracle(case, window):
    ref, _ = paged_attention_oracle(case.q.cpu(), case.k_cache.cpu(), case.v_cache.cpu(), case.cu_seqlens_q.cpu(),
                                    case.seqused_k.cpu(), case.block_table.cpu(), case.causal, window)
    return ref


# ------------------------------------------------------------------ backend surface (CPU)
def test_backend_static_surface():
    assert Backend.get_name() == "CUSTOM"
    assert Backend.get_impl_cls() is Impl
    assert Backend.get_builder_cls() is backend.ToyFlashAttentionMetadataBuilder
    assert Backend.get_kv_cache_shape(100, 16, 8, 128) == (2, 100, 16, 8, 128)
    assert Backend.get_kv_cache_stride_order() == (0, 1, 2, 3, 4)
    with pytest.raises(NotImplementedError):
        Backend.get_kv_cache_stride_order(include_num_layers_dimension=True)
    (sizes,) = Backend.get_supported_kernel_block_sizes()
    assert getattr(sizes, "base", None) == 16
    assert Backend.supports_head_size(64) and Backend.supports_head_size(128)
    assert not Backend.supports_head_size(96)
    assert Backend.supports_kv_cache_dtype("bfloat16") and Backend.supports_kv_cache_dtype(None)
    assert not Backend.supports_kv_cache_dtype("fp8")
    assert Backend.supports_attn_type(AttentionType.DECODER)
    assert not Backend.supports_attn_type(AttentionType.ENCODER)
    assert Backend.supports_compute_capability(SimpleNamespace(major=10, minor=0))
    assert not Backend.supports_compute_capability(SimpleNamespace(major=9, minor=0))
    assert Backend.supports_combination(64, torch.bfloat16, None, 16, False, True, False, None) is not None
    assert Backend.supports_combination(64, torch.bfloat16, None, 16, False, False, False, None) is None


def test_register_backend_as_custom():
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend

    register_backend(AttentionBackendEnum.CUSTOM, "toy_flash_attn.ToyFlashAttentionBackend")
    assert AttentionBackendEnum.CUSTOM.get_class() is Backend


def test_metadata_builder_copies_common_fields():
    b = backend.ToyFlashAttentionMetadataBuilder.__new__(backend.ToyFlashAttentionMetadataBuilder)
    common = SimpleNamespace(
        num_actual_tokens=5, max_query_len=3, query_start_loc=torch.tensor([0, 2, 5]), max_seq_len=40,
        seq_lens=torch.tensor([30, 40]), block_table_tensor=torch.zeros(2, 3, dtype=torch.int32),
        slot_mapping=torch.arange(5), causal=True,
    )
    md = b.build(0, common)
    assert md.num_actual_tokens == 5 and md.max_query_len == 3 and md.max_seq_len == 40 and md.causal
    assert md.block_table is common.block_table_tensor and md.seq_lens is common.seq_lens
    assert md.slot_mapping is common.slot_mapping and md.query_start_loc is common.query_start_loc


@pytest.mark.parametrize("kw", [
    dict(alibi_slopes=[1.0, 1.0]),
    dict(logits_soft_cap=30.0),
    dict(kv_sharing_target_layer_name="layers.0"),
    dict(kv_cache_dtype="fp8"),
    dict(attn_type=AttentionType.ENCODER),
])
def test_impl_rejects_unsupported_options(kw):
    with pytest.raises(NotImplementedError):
        Impl(2, 64, 0.125, **kw)


def test_impl_sliding_window_is_left_window_of_size_minus_one():
    assert Impl(4, 64, 0.125, 2, sliding_window=1025).sliding_window == (1024, 0)
    assert Impl(4, 64, 0.125, 2).sliding_window is None
    assert Impl(4, 64, 0.125).num_kv_heads == 4


def test_forward_without_metadata_returns_zeros():
    impl = Impl(2, 64, 0.125)
    q = torch.randn(3, 2, 64)
    z = impl.forward(None, q, q, q, torch.zeros(2, 1, 16, 2, 64), None)
    assert torch.equal(z, torch.zeros_like(q))
    out = torch.ones_like(q)
    assert impl.forward(None, q, q, q, torch.zeros(2, 1, 16, 2, 64), None, output=out) is out
    assert torch.equal(out, torch.zeros_like(q))


def test_forward_rejects_output_quantization():
    impl = Impl(2, 64, 0.125)
    q = torch.randn(3, 2, 64)
    with pytest.raises(NotImplementedError):
        impl.forward(None, q, q, q, torch.zeros(2, 1, 16, 2, 64), None, output_scale=torch.ones(1))


def test_forward_reference_mode_matches_oracle_cpu(monkeypatch):
    """Impl.forward with TOY_FLASH_ATTN_USE=reference: padded tail rows of the output
    buffer (beyond num_actual_tokens) are left untouched, as in the reference."""
    monkeypatch.setenv("TOY_FLASH_ATTN_USE", "reference")
    case = reference_case([3, 5], [6, 9], num_heads=4, num_kv_heads=2, causal=True, dtype=torch.float32)
    impl = Impl(4, 64, 0.125, 2, sliding_window=4)
    n = case.q.shape[0]
    pad = 2
    query = torch.cat([case.q, torch.randn(pad, 4, 64)])
    out = torch.full_like(query, 7.0)
    kv_cache = torch.stack([case.k_cache, case.v_cache])
    key = torch.zeros(n + pad, 2, 64)
    res = impl.forward(None, query, key, key, kv_cache, _metadata(case), output=out)
    assert res is out
    ref = _oracle(case, (3, 0))
    torch.testing.assert_close(out[:n], ref, atol=1e-5, rtol=1e-5)
    assert torch.all(out[n:] == 7.0)


# ------------------------------------------------------------------ dump / replay (CPU)
def test_dump_files_and_replay_reference_mode(monkeypatch, tmp_path):
    monkeypatch.setenv("TOY_FLASH_ATTN_USE", "reference")
    monkeypatch.setenv("TOY_FLASH_ATTN_DUMP_DIR", str(tmp_path))
    from toy_flash_attn import flash_attention_func as faf

    case = reference_case([2, 6], [8, 8], causal=True, window_size=(2, 0), dtype=torch.float32)
    out = faf.flash_attn_varlen_func(**case.kwargs())
    files = sorted(tmp_path.glob("*.pt"))
    assert len(files) == 1 and re.fullmatch(r"\d{5}_with_block\.pt", files[0].name)
    payload = replay_mod.load_dump(files[0])
    assert replay_mod.REPLAY_KEYS <= payload.keys()
    assert torch.equal(payload["result"], out)
    monkeypatch.delenv("TOY_FLASH_ATTN_DUMP_DIR")
    again, dumped = replay_mod.replay(files[0], device="cpu")
    torch.testing.assert_close(again, dumped, atol=0, rtol=0)


def test_load_dump_names_missing_keys(tmp_path):
    path = tmp_path / "00000_with_block.pt"
    torch.save({"q": torch.zeros(1)}, path)
    with pytest.raises(AssertionError, match="missing keys"):
        replay_mod.load_dump(path)


# ------------------------------------------------------------------ GPU: the sm_100a path
@pytest.mark.gpu
@pytest.mark.parametrize("num_heads,num_kv_heads,head_dim,q_lens,k_lens", [
    (8, 2, 64, [1, 1, 1], [40, 257, 1000]),   # decode kernel
    (4, 1, 128, [17, 3], [80, 150]),          # prefill kernel
])
def test_impl_cache_update_then_forward_gpu(monkeypatch, num_heads, num_kv_heads, head_dim, q_lens, k_lens):
    """vLLM's step order: do_kv_cache_update scatters the new tokens into an empty cache,
    then forward attends over it; the result matches the oracle on the case's cache."""
    monkeypatch.delenv("TOY_FLASH_ATTN_USE", raising=False)
    case = reference_case(q_lens, k_lens, num_heads=num_heads, num_kv_heads=num_kv_heads, head_dim=head_dim,
                          causal=True, block_size=16, seed=3).to("cuda")
    impl = Impl(num_heads, head_dim, head_dim ** -0.5, num_kv_heads)
    nb, bs = case.k_cache.shape[:2]
    kv_cache = torch.zeros(2, nb, bs, num_kv_heads, head_dim, dtype=torch.bfloat16, device="cuda")
    # every cached token of every sequence, with its slot, plus one padded slot (-1)
    keys, values, slots = [], [], []
    for b, kv_len in enumerate(k_lens):
        t = torch.arange(kv_len, device="cuda")
        blk = case.block_table[b, t // bs].long()
        slot = blk * bs + t % bs
        keys.append(case.k_cache[blk, t % bs])
        values.append(case.v_cache[blk, t % bs])
        slots.append(slot)
    key = torch.cat(keys + [torch.full_like(keys[0][:1], float("nan"))])
    value = torch.cat(values + [torch.full_like(values[0][:1], float("nan"))])
    slot_mapping = torch.cat(slots + [torch.tensor([-1], device="cuda")])
    impl.do_kv_cache_update(None, key, value, kv_cache, slot_mapping)
    n = case.q.shape[0]
    pad = 3
    query = torch.cat([case.q, torch.randn(pad, num_heads, head_dim, device="cuda").bfloat16()])
    out = torch.full_like(query, 5.0)
    dummy = torch.zeros(n + pad, num_kv_heads, head_dim, dtype=torch.bfloat16, device="cuda")
    impl.forward(None, query, dummy, dummy, kv_cache, _metadata(case), output=out)
    torch.cuda.synchronize()
    ref = _oracle(case, None)
    assert (out[:n].float().cpu() - ref).abs().max().item() <= OUT_TOL
    assert torch.all(out[n:] == 5.0)


@pytest.mark.gpu
def test_dump_and_replay_cuda_path(monkeypatch, tmp_path):
    monkeypatch.delenv("TOY_FLASH_ATTN_USE", raising=False)
    monkeypatch.setenv("TOY_FLASH_ATTN_DUMP_DIR", str(tmp_path))
    from toy_flash_attn import flash_attention_func as faf

    case = reference_case([1, 7, 40], [30, 64, 100], num_heads=8, num_kv_heads=2, causal=True, block_size=16,
                          seed=5).to("cuda")
    faf.flash_attn_varlen_func(**case.kwargs())
    torch.cuda.synchronize()
    files = sorted(tmp_path.glob("*.pt"))
    assert len(files) == 1 and re.fullmatch(r"\d{5}_with_block_cu\.pt", files[0].name)
    monkeypatch.delenv("TOY_FLASH_ATTN_DUMP_DIR")
    again, dumped = replay_mod.replay(files[0], device="cuda")
    torch.cuda.synchronize()
    assert torch.equal(again, dumped)  # same inputs, same plan: bit-identical
    ref = _oracle(case, None)
    assert (again.float().cpu() - ref).abs().max().item() <= OUT_TOL


# ------------------------------------------------------------------ vLLM e2e script (CPU parts)
def test_vllm_e2e_compare_and_prompts():
    from toy_flash_attn import vllm_e2e

    prompts = vllm_e2e._prompts(4, vllm_e2e.QWEN2_SMALL["vocab_size"])
    assert [len(p) for p in prompts] == [17, 54, 91, 128]
    assert all(0 <= t < vllm_e2e.QWEN2_SMALL["vocab_size"] for p in prompts for t in p)
    cfg = vllm_e2e.QWEN2_SMALL
    assert cfg["num_attention_heads"] % cfg["num_key_value_heads"] == 0
    assert cfg["hidden_size"] // cfg["num_attention_heads"] == 64  # a head size the kernels take
    a = {"sequences": [{"tokens": [1, 2, 3, 4], "logprobs": [-1.0, -2.0, -3.0, -4.0]},
                       {"tokens": [5, 6], "logprobs": [-0.5, -0.25]}]}
    b = {"sequences": [{"tokens": [1, 2, 9, 4], "logprobs": [-1.0, -2.5, -3.0, -4.0]},
                       {"tokens": [5, 6], "logprobs": [-0.5, -0.25]}]}
    res = vllm_e2e.compare(a, b)
    assert res["first_divergence"] == [2, 2]
    assert res["tokens_identical_prefix"] == 4 and res["tokens_total"] == 6
    assert res["max_logprob_gap_before_divergence"] == 0.5
