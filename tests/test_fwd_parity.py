"""Parity of the sm_100a forward with the CPU oracle and the reference's golden outputs.

Tolerances (bf16 inputs, fp32 math in the oracle): output max-abs error <= 2e-2,
natural-log LSE max-abs error <= 1e-3. Calls go through the public
``flash_attn_varlen_func`` (which calls the C ABI ``tfa_fwd``).
"""

from __future__ import annotations

import math

import pytest
import torch

from conftest import golden_files, load_golden
from oracle.paged_attention import paged_attention_oracle
from toy_flash_attn import flash_attention_func as faf
from toy_flash_attn.workloads import PagedCase, baseline_config, reference_case

OUT_TOL = 2e-2
LSE_TOL = 1e-3

pytestmark = pytest.mark.gpu


def run_cuda(case: PagedCase, **kw):
    c = case.to("cuda")
    out = torch.empty_like(c.q)
    lse = torch.empty(c.q.shape[0], c.q.shape[1], dtype=torch.float32, device="cuda")
    res = faf.flash_attn_varlen_func(**c.kwargs(), out=out, softmax_lse=lse, **kw)
    assert res.data_ptr() == out.data_ptr()
    torch.cuda.synchronize()
    assert faf.read_device_error() == 0
    return out.cpu(), lse.cpu()


def oracle(case: PagedCase):
    return paged_attention_oracle(case.q, case.k_cache, case.v_cache, case.cu_seqlens_q, case.seqused_k,
                                  case.block_table, case.causal, case.window_size)


def assert_parity(case: PagedCase, **kw):
    out, lse = run_cuda(case, **kw)
    ref_out, ref_lse = oracle(case)
    assert torch.isfinite(out.float()).all(), "non-finite output"
    err = (out.float() - ref_out).abs().max().item() if out.numel() else 0.0
    assert err <= OUT_TOL, f"{case.name}: out max-abs err {err}"
    fin = torch.isfinite(ref_lse)
    assert torch.equal(fin, torch.isfinite(lse)), f"{case.name}: LSE finiteness differs"
    if fin.any():
        lerr = (lse[fin] - ref_lse[fin]).abs().max().item()
        assert lerr <= LSE_TOL, f"{case.name}: lse max-abs err {lerr}"
    return out, lse


GOLDEN = [p for p in golden_files()]


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_golden_vs_reference_output(path):
    g = load_golden(path)
    case = PagedCase(g["name"], g["q"], g["k"], g["v"], g["cu_seqlens_q"], g["seqused_k"], g["block_table"],
                     g["max_seqlen_q"], g["max_seqlen_k"], g["causal"], g["window_size"])
    if case.q.shape[2] not in (64, 128):
        with pytest.raises(RuntimeError, match="TFA_ERR_HEAD_DIM"):
            run_cuda(case)
        return
    out, _ = assert_parity(case)
    err = (out.float() - g["out_ref_fp32"].float()).abs().max().item()
    assert err <= OUT_TOL, f"vs reference output: {err}"


@pytest.mark.parametrize("name", ["C1", "C2", "C3", "C4"])
def test_baseline_configs_full_size(name):
    assert_parity(baseline_config(name))


def test_long_prefill_d128_gqa():
    case = reference_case([1536], [1536], num_heads=8, num_kv_heads=2, head_dim=128, causal=True, block_size=16,
                          seed=21)
    assert_parity(case)


@pytest.mark.parametrize(
    "q_lens, hq, hkv, hd",
    [([1024] * 6, 14, 2, 64), ([512] * 7 + [300], 32, 8, 128), ([700, 1024, 33, 513] * 2, 16, 4, 128)],
    ids=["d64_g7", "d128_g4", "d128_g4_ragged"],
)
def test_two_tile_prefill_items(q_lens, hq, hkv, hd):
    """Large prefill batches use 256-row items (two q tiles per CTA)."""
    case = reference_case(q_lens, num_heads=hq, num_kv_heads=hkv, head_dim=hd, causal=True, block_size=16,
                          seed=len(q_lens) + hd)
    c = case.to("cuda")
    p = faf.plan(c.q, c.k_cache, c.v_cache, c.cu_seqlens_q, c.seqused_k, c.block_table, c.max_seqlen_q,
                 c.max_seqlen_k, True)
    assert p["kernel"] in (1, 2) and p["rows_per_tile"] == 256  # 2: >= 8 sequences also run the decode kernel
    assert_parity(case)


def test_c5_reduced_batch_full_lengths():
    case = baseline_config("C5", batch=12, num_blocks=40000)
    assert_parity(case)


@pytest.mark.parametrize("hq, hkv, hd, bs, q_lens", [
    (32, 8, 128, 16, [1, 1]),       # C5 heads: 16384 pages in one block-table row
    (14, 2, 64, 256, [1, 2]),       # the reference's heads, large pages, a 2-token chunk (14 rows)
])
def test_long_context_decode(hq, hkv, hd, bs, q_lens):
    """Decode against a 262144-token context (and a 100003-token one): tile, position and
    block-table index arithmetic well past the BASELINE lengths, splits at their cap."""
    case = reference_case(q_lens, [262144, 100003], num_heads=hq, num_kv_heads=hkv, head_dim=hd, causal=True,
                          block_size=bs, seed=21, name="long_context")
    p = faf.plan(case.q.cuda(), case.k_cache.cuda(), case.v_cache.cuda(), case.cu_seqlens_q.cuda(),
                 case.seqused_k.cuda(), case.block_table.cuda(), case.max_seqlen_q, case.max_seqlen_k, True)
    assert p["kernel"] == 0 and p["max_splits"] > 1
    assert_parity(case)


@pytest.mark.parametrize("q_len", [1, 3])
def test_wide_batch_decode(q_len):
    """4096 short sequences in one call (16384 work groups): the persistent scheduler, the
    split bookkeeping and the combine over far more groups than the in-kernel merge counts."""
    g = torch.Generator().manual_seed(33)
    k_lens = torch.randint(1, 300, (4096,), generator=g).tolist()
    case = reference_case([q_len] * 4096, [max(k, q_len) for k in k_lens], num_heads=16, num_kv_heads=4,
                          causal=True, block_size=16, seed=33, name="wide_batch")
    assert_parity(case)


def _page_decode_case(hd, group, window=None, seed=41, n_seqs=10):
    """One-token sequences with ragged lengths (every last page partial, one sequence of a
    single token), 8 kv heads, 16-slot pages, NaN in every slot past a sequence's end."""
    g = torch.Generator().manual_seed(seed)
    k_lens = [int(x) for x in torch.randint(5000, 8192, (n_seqs,), generator=g)]
    k_lens[3] = 1
    k_lens = [k if k % 16 else k + 5 for k in k_lens]
    case = reference_case([1] * n_seqs, k_lens, num_heads=8 * group, num_kv_heads=8, head_dim=hd, causal=True,
                          window_size=window, block_size=16, seed=seed, name=f"pages_d{hd}_g{group}")
    for b, n in enumerate(k_lens):
        last = int(case.block_table[b, (n - 1) // 16])
        case.k_cache[last, n % 16:] = float("nan")
        case.v_cache[last, n % 16:] = float("nan")
    return case


@pytest.mark.parametrize("hd, group", [(64, 1), (64, 2), (64, 4), (128, 1), (128, 2), (128, 4)])
def test_page_decode_kernel(hd, group):
    """Large one-token decode calls with 8 kv heads and 16-slot pages run the page kernel
    (one item = a sequence's split over all kv heads, one box per page)."""
    case = _page_decode_case(hd, group)
    c = case.to("cuda")
    p = faf.plan(c.q, c.k_cache, c.v_cache, c.cu_seqlens_q, c.seqused_k, c.block_table, 1, c.max_seqlen_k, True)
    assert p["pages"] == 1 and p["max_splits"] > 1
    assert_parity(case)


def test_page_decode_kernel_window():
    case = _page_decode_case(128, 4, window=(6000, 0), seed=43, n_seqs=16)
    c = case.to("cuda")
    p = faf.plan(c.q, c.k_cache, c.v_cache, c.cu_seqlens_q, c.seqused_k, c.block_table, 1, c.max_seqlen_k, True,
                 (6000, 0))
    assert p["pages"] == 1
    assert_parity(case)


def test_c5_full_size_sample_vs_oracle():
    """The headline call at full size: all 256 sequences, the 2^21-block pool (137 GB of
    K/V), one call. The 16 longest and 16 seeded-random sequences are checked against the
    oracle (the oracle on all 256 would take minutes on the CPU); the rest must be finite."""
    from toy_flash_attn.workloads import compact_sample, verify_sequences

    torch.cuda.empty_cache()
    free, _ = torch.cuda.mem_get_info()
    if free < 145e9:
        pytest.skip(f"full C5 needs ~140 GB of free device memory, {free / 1e9:.0f} GB free")
    case = baseline_config("C5", device="cuda")
    try:
        out = torch.empty_like(case.q)
        lse = torch.empty(case.q.shape[0], case.q.shape[1], dtype=torch.float32, device="cuda")
        faf.flash_attn_varlen_func(**case.kwargs(), out=out, softmax_lse=lse)
        torch.cuda.synchronize()
        assert faf.read_device_error() == 0
        assert torch.isfinite(out).all() and torch.isfinite(lse).all()
        seqs = verify_sequences(case.seqused_k.tolist())
        sub = compact_sample(case, seqs, device="cpu")
    finally:
        del case
        torch.cuda.empty_cache()
    ref, ref_lse = oracle(sub)
    err = (out[seqs].cpu().float() - ref).abs().max().item()
    lerr = (lse[seqs].cpu() - ref_lse).abs().max().item()
    assert err <= OUT_TOL, f"out max-abs err {err}"
    assert lerr <= LSE_TOL, f"lse max-abs err {lerr}"


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 16])
def test_forced_splits_decode(splits):
    assert_parity(baseline_config("C2"), num_splits=splits)


@pytest.mark.parametrize("splits", [1, 2, 5])
def test_forced_splits_prefill(splits):
    assert_parity(baseline_config("C3"), num_splits=splits)


@pytest.mark.parametrize("block_size", [1, 2, 4, 8, 16, 32, 64])
def test_block_sizes(block_size):
    case = reference_case([1, 3, 40], [300, 77, 129], num_heads=8, num_kv_heads=2, causal=True,
                          block_size=block_size, seed=block_size)
    assert_parity(case)


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("group", [1, 2, 4, 7, 8, 16])
@pytest.mark.parametrize("q_lens", [[1, 1, 1, 1], [1, 1, 5, 33]], ids=["decode", "mixed"])
def test_gqa_groups(hd, group, q_lens):
    hkv = 2
    case = reference_case(q_lens, [260, 1, 140, 200], num_heads=hkv * group, num_kv_heads=hkv, head_dim=hd,
                          causal=True, block_size=16, seed=group + hd)
    assert_parity(case)


def test_speculative_decode_rows_packed():
    # q_len * group <= 16 packs several q tokens into the decode kernel's 16 columns
    case = reference_case([4, 2, 1], [300, 17, 129], num_heads=8, num_kv_heads=2, causal=True, block_size=16)
    assert_parity(case)


@pytest.mark.parametrize("window", [(0, 0), (1, 0), (16, 0), (127, 0), (128, 0), (300, 0), (5, 3), (64, 64),
                                    (-1, 10), (10, -1)])
def test_windows_non_causal_and_causal(window):
    for causal in (False, True):
        case = reference_case([1, 7, 150], [500, 90, 150], num_heads=4, num_kv_heads=2, causal=causal,
                              window_size=window, block_size=16, seed=3)
        assert_parity(case)


def test_empty_and_ragged_sequences():
    # zero-length kv, zero-length q, kv shorter than q (fully masked causal rows -> 0 / -inf)
    case = reference_case([3, 0, 4, 1, 6], [0, 5, 2, 1, 130], num_heads=4, num_kv_heads=1, causal=True,
                          block_size=16, seed=5)
    case.block_table[case.block_table < 0] = 0  # entries past kv_len are never read
    out, lse = assert_parity(case)
    assert torch.all(out[:3] == 0)
    assert torch.all(torch.isneginf(lse[:3]))


def test_nan_slots_are_masked():
    case = baseline_config("C4", batch=4, kv_range=(17, 300))
    assert torch.isnan(case.k_cache).any()
    assert_parity(case)


def test_strided_q_and_out_views():
    case = reference_case([5, 70], [90, 70], num_heads=8, num_kv_heads=2, causal=True, block_size=16, seed=9)
    c = case.to("cuda")
    big_q = torch.randn(c.q.shape[0], c.q.shape[1] * 2, c.q.shape[2], device="cuda").to(torch.bfloat16)
    big_q[:, ::2] = c.q
    qv = big_q[:, ::2]
    big_out = torch.zeros(c.q.shape[0], c.q.shape[1], c.q.shape[2] * 2, dtype=torch.bfloat16, device="cuda")
    ov = big_out[:, :, : c.q.shape[2]]
    faf.flash_attn_varlen_func(qv, c.k_cache, c.v_cache, c.max_seqlen_q, c.cu_seqlens_q, c.max_seqlen_k, None,
                               c.seqused_k, c.causal, c.window_size, c.block_table, out=ov)
    ref, _ = oracle(case)
    assert (ov.float().cpu() - ref).abs().max().item() <= OUT_TOL
    assert torch.all(big_out[:, :, c.q.shape[2]:] == 0)


def test_repeat_calls_identical():
    case = baseline_config("C2")
    a, la = run_cuda(case)
    b, lb = run_cuda(case)
    assert torch.equal(a, b) and torch.equal(la, lb)


def test_block_permutation_invariance():
    """Moving pages to new physical ids (and updating the table) changes nothing."""
    case = baseline_config("C2", num_blocks=512)
    a, _ = run_cuda(case)
    perm = torch.randperm(512, generator=torch.Generator().manual_seed(1))
    moved = PagedCase(case.name, case.q, torch.empty_like(case.k_cache), torch.empty_like(case.v_cache),
                      case.cu_seqlens_q, case.seqused_k, perm[case.block_table.long()].to(torch.int32),
                      case.max_seqlen_q, case.max_seqlen_k, case.causal, case.window_size)
    moved.k_cache[perm] = case.k_cache
    moved.v_cache[perm] = case.v_cache
    b, _ = run_cuda(moved)
    assert torch.equal(a, b)


def test_softmax_scale_override():
    case = reference_case([1, 20], [100, 20], num_heads=4, num_kv_heads=2, causal=True, block_size=16, seed=2)
    out, lse = run_cuda(case, softmax_scale=0.3)
    ref, ref_lse = paged_attention_oracle(case.q, case.k_cache, case.v_cache, case.cu_seqlens_q, case.seqused_k,
                                          case.block_table, True, None, softmax_scale=0.3)
    assert (out.float() - ref).abs().max().item() <= OUT_TOL
    assert (lse - ref_lse).abs().max().item() <= LSE_TOL


def test_non_paged_varlen_path():
    """block_table=None: dense varlen K/V (flash_attention_func.py:411-457)."""
    g = torch.Generator().manual_seed(4)
    lens_q, lens_k = [3, 64], [40, 64]
    q = torch.randn(sum(lens_q), 4, 64, generator=g).to(torch.bfloat16)
    k = torch.randn(sum(lens_k), 2, 64, generator=g).to(torch.bfloat16)
    v = torch.randn(sum(lens_k), 2, 64, generator=g).to(torch.bfloat16)
    cq = torch.tensor([0, 3, 67], dtype=torch.int32)
    ck = torch.tensor([0, 40, 104], dtype=torch.int32)
    out = faf.flash_attn_varlen_func(q.cuda(), k.cuda(), v.cuda(), 64, cq.cuda(), 64, ck.cuda(), causal=True)
    # oracle on an equivalent paged layout (one token per block)
    bt = torch.stack([torch.arange(64) + 0, torch.arange(64) + 40]).to(torch.int32)
    bt[0, 40:] = 0
    ref, _ = paged_attention_oracle(q, k.unsqueeze(1), v.unsqueeze(1), cq, torch.tensor(lens_k, dtype=torch.int32),
                                    bt, True, None)
    assert (out.float().cpu() - ref).abs().max().item() <= OUT_TOL


def test_input_validation_errors():
    case = reference_case([2], [10], num_heads=4, num_kv_heads=2, block_size=16).to("cuda")
    with pytest.raises(TypeError):
        faf.flash_attn_varlen_func(case.q.float(), case.k_cache, case.v_cache, 2, case.cu_seqlens_q, 10, None,
                                   case.seqused_k, False, None, case.block_table)
    with pytest.raises(TypeError):
        faf.flash_attn_varlen_func(case.q, case.k_cache, case.v_cache, 2, case.cu_seqlens_q.long(), 10, None,
                                   case.seqused_k, False, None, case.block_table)
    with pytest.raises(ValueError):
        faf.flash_attn_varlen_func(case.q[:, :3], case.k_cache, case.v_cache, 2, case.cu_seqlens_q, 10, None,
                                   case.seqused_k, False, None, case.block_table)
    with pytest.raises(RuntimeError, match="TFA_ERR_HEAD_DIM"):
        q = torch.zeros(2, 4, 96, dtype=torch.bfloat16, device="cuda")
        kc = torch.zeros(4, 16, 2, 96, dtype=torch.bfloat16, device="cuda")
        faf.flash_attn_varlen_func(q, kc, kc, 2, case.cu_seqlens_q, 10, None, case.seqused_k, False, None,
                                   case.block_table)


def test_bad_block_id_reported_not_faulting():
    case = reference_case([1], [40], num_heads=2, num_kv_heads=1, block_size=16)
    case.block_table[0, 1] = 10_000  # outside the pool
    c = case.to("cuda")
    faf.flash_attn_varlen_func(**c.kwargs())
    torch.cuda.synchronize()
    assert faf.read_device_error() == 110
    assert faf.read_device_error() == 0  # cleared


def test_plan_decode_vs_prefill_selection():
    c2 = baseline_config("C2").to("cuda")
    p = faf.plan(c2.q, c2.k_cache, c2.v_cache, c2.cu_seqlens_q, c2.seqused_k, c2.block_table, c2.max_seqlen_q,
                 c2.max_seqlen_k, True)
    assert p["kernel"] == 0 and p["max_splits"] > 1 and p["combine"] == 2
    c3 = baseline_config("C3").to("cuda")
    p = faf.plan(c3.q, c3.k_cache, c3.v_cache, c3.cu_seqlens_q, c3.seqused_k, c3.block_table, c3.max_seqlen_q,
                 c3.max_seqlen_k, True)
    assert p["kernel"] == 1 and p["rows_per_tile"] in (128, 256)
    assert p["grid"] <= torch.cuda.get_device_properties(0).multi_processor_count
    assert math.isfinite(p["workspace_bytes"])


# Mixed batches (vLLM chunked prefill: decode tokens and prompt chunks in one call) run
# the decode kernel on decode-shaped sequences (q_len * group <= 16) and the prefill
# kernel on the rest.
MIXED = [
    # q lens: decode tokens, short speculative chunks (q_len * G == 16 is still decode-shaped), prompt chunks
    dict(q=[1, 1, 1, 4, 1, 2, 1, 40, 1, 300, 1, 3], k=[50, 700, 129, 260, 1, 33, 2048, 40, 900, 812, 16, 3],
         heads=16, kv=4, d=128, causal=True, window=None),
    dict(q=[1, 2, 1, 1, 17, 1, 1, 1, 1, 9], k=[300, 64, 1000, 5, 17, 128, 129, 2000, 77, 500],
         heads=8, kv=1, d=64, causal=True, window=(100, 0)),
    dict(q=[1] * 9 + [64], k=[33 * i + 1 for i in range(9)] + [200], heads=4, kv=4, d=64, causal=False,
         window=None),
    # group 16: one q token is exactly 16 rows (decode-shaped), two are prefill-shaped
    dict(q=[1, 2, 1, 1, 1, 1, 1, 3], k=[100, 300, 17, 2049, 64, 65, 1, 500], heads=32, kv=2, d=128, causal=True,
         window=None),
    # two-sided window, not causal
    dict(q=[1, 1, 30, 1, 1, 1, 1, 5], k=[400, 90, 260, 33, 1000, 128, 7, 77], heads=8, kv=2, d=64, causal=False,
         window=(48, 16)),
]


@pytest.mark.parametrize("cfg", MIXED, ids=["gqa4_d128", "gqa8_d64_window", "mha_d64_noncausal", "gqa16_d128",
                                         "two_sided_window"])
@pytest.mark.parametrize("splits", [0, 3])
def test_mixed_batch_both_kernels(cfg, splits):
    case = reference_case(cfg["q"], cfg["k"], num_heads=cfg["heads"], num_kv_heads=cfg["kv"], head_dim=cfg["d"],
                          causal=cfg["causal"], window_size=cfg["window"], block_size=cfg.get("bs", 16), seed=21)
    c = case.to("cuda")
    p = faf.plan(c.q, c.k_cache, c.v_cache, c.cu_seqlens_q, c.seqused_k, c.block_table, c.max_seqlen_q,
                 c.max_seqlen_k, c.causal, c.window_size, num_splits=splits)
    assert p["kernel"] == 2
    assert_parity(case, num_splits=splits)
    # the same call again on the same workspace (control words left zeroed)
    assert_parity(case, num_splits=splits)


def test_mixed_batch_all_prefill_rows():
    """A call that qualifies for both kernels but holds no decode-shaped sequence."""
    case = reference_case([20] * 8, [20 + 7 * i for i in range(8)], num_heads=4, num_kv_heads=2, head_dim=64,
                          causal=True, block_size=16, seed=22)
    assert_parity(case)


def _item_list_case():
    """Decode call shaped like a C5 shard at 8 GPUs (one kv head, long-tailed lengths): split
    slots to spare and a small work bound, so the decode kernel takes its items from the
    device-built list."""
    g = torch.Generator().manual_seed(31)
    k_lens = [int(x) for x in torch.exp(torch.empty(64).uniform_(0, math.log(8192), generator=g)).round().clamp(1, 8192)]
    k_lens[0] = 8192
    return reference_case([1] * 64, k_lens, num_heads=16, num_kv_heads=4, head_dim=128, causal=True, block_size=16,
                          seed=31)


@pytest.mark.parametrize("name", ["C2", "C1", "list", "pages"],
                         ids=["decode_split", "prefill", "decode_item_list", "decode_pages"])
def test_time_limit_reports_error_and_recovers(monkeypatch, name):
    """Every in-kernel wait is bounded. The test hook makes each CTA wait on a barrier
    nothing arrives on: after the wait's limit (about 1 s) the call must record a time-limit
    error (101-103: whichever warp's wait expired first), every warp must unwind (no hang,
    no fault), the error word must clear, and the next call on the same stream and workspace
    must be correct."""
    case = (_item_list_case() if name == "list" else _page_decode_case(128, 4) if name == "pages"
            else baseline_config(name))
    c = case.to("cuda")
    if name in ("list", "pages"):
        p = faf.plan(c.q, c.k_cache, c.v_cache, c.cu_seqlens_q, c.seqused_k, c.block_table, c.max_seqlen_q,
                     c.max_seqlen_k, True)
        assert p["item_list" if name == "list" else "pages"] == 1
    out = torch.empty_like(c.q)
    monkeypatch.setenv("TFA_DEBUG_STALL_WAIT", "1")
    faf.flash_attn_varlen_func(**c.kwargs(), out=out)
    torch.cuda.synchronize()
    # the first limit to expire wins the error word: the MMA warp's (102) or a warp waiting on it (101, 103)
    assert faf.read_device_error() in (101, 102, 103)
    assert faf.read_device_error() == 0
    monkeypatch.delenv("TFA_DEBUG_STALL_WAIT")
    assert_parity(case)


def test_mixed_batch_large_pages():
    """Mixed dispatch with 64-token pages (one page covers half a kv tile)."""
    case = reference_case([1, 1, 1, 1, 40, 1, 1, 2], [500, 64, 65, 1, 300, 129, 700, 90], num_heads=8,
                          num_kv_heads=2, head_dim=128, causal=True, block_size=64, seed=23)
    assert_parity(case)



@pytest.mark.parametrize("bs", [1, 4])
def test_mixed_batch_small_pages_and_empty_sequences(bs):
    """Mixed dispatch with empty queries, empty caches and sub-16-token pages."""
    case = reference_case([1, 0, 1, 12, 1, 1, 0, 2], [50, 30, 0, 70, 129, 1, 0, 19], num_heads=8, num_kv_heads=2,
                          head_dim=64, causal=True, block_size=bs, seed=24)
    out, _ = run_cuda(case)
    ref, _ = oracle(case)
    # rows of a sequence with an empty cache attend to nothing: the reference's softmax of an
    # all-masked row is NaN, this library writes zeros (and -inf LSE); compare the others
    q0 = case.cu_seqlens_q.tolist()
    keep = torch.ones(out.shape[0], dtype=torch.bool)
    for b, kv in enumerate(case.seqused_k.tolist()):
        if kv == 0:
            keep[q0[b]:q0[b + 1]] = False
    assert torch.isfinite(out.float()).all()
    assert (out.float()[keep] - ref[keep]).abs().max().item() <= OUT_TOL
    assert torch.all(out[~keep] == 0)


def test_decode_with_device_item_list():
    """A decode call with split slots to spare and a small work bound takes its items from a
    list built on the device, longest first; results must not depend on that order."""
    case = _item_list_case()
    c = case.to("cuda")
    p = faf.plan(c.q, c.k_cache, c.v_cache, c.cu_seqlens_q, c.seqused_k, c.block_table, c.max_seqlen_q,
                 c.max_seqlen_k, True)
    assert p["kernel"] == 0 and p["max_splits"] > 1 and p["num_items"] > 2 * p["grid"]
    assert p["item_list"] == 1  # the list instance of the decode kernel runs
    out, _ = assert_parity(case)
    out2, _ = run_cuda(case)
    assert torch.equal(out, out2)


def test_graph_replay_after_workspace_growth():
    """A CUDA graph captured with a small call keeps using that call's workspace; a later,
    larger call on the same stream grows the workspace, and replaying the graph afterwards
    must still give the right result (the old buffer stays allocated)."""
    small = baseline_config("C2").to("cuda")  # 16 splits: uses the workspace's split buffers
    big = baseline_config("C4").to("cuda")
    out = torch.empty_like(small.q)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        faf.flash_attn_varlen_func(**small.kwargs(), out=out)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            faf.flash_attn_varlen_func(**small.kwargs(), out=out)
        big_out = torch.empty_like(big.q)
        faf.flash_attn_varlen_func(**big.kwargs(), out=big_out, num_splits=16)  # needs a larger workspace
        out.zero_()
        g.replay()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        assert faf.read_device_error() == 0
    ref, _ = oracle(baseline_config("C2"))
    assert (out.cpu().float() - ref).abs().max().item() <= OUT_TOL


def test_call_cache_follows_new_buffers():
    """The C ABI keeps a per-thread cache of plans and tensor maps keyed by the argument
    struct: a call with other K/V/q buffers of the same shapes must use the new buffers."""
    a = baseline_config("C2", seed=41).to("cuda")
    b = baseline_config("C2", seed=42).to("cuda")  # same shapes and tables, other values
    assert not torch.equal(a.k_cache, b.k_cache)
    out_a1, _ = run_cuda(a)
    out_b, _ = run_cuda(b)
    out_a2, _ = run_cuda(a)
    assert torch.equal(out_a1, out_a2)
    ref_b, _ = oracle(baseline_config("C2", seed=42))
    assert (out_b.float() - ref_b).abs().max().item() <= OUT_TOL
    assert not torch.equal(out_a1, out_b)


def test_two_host_threads_on_their_own_streams():
    """Host threads driving their own streams concurrently (the library's caches are per
    thread or atomic, each stream has its own workspace) get correct results."""
    import threading

    cases = [baseline_config("C4", batch=6, seed=50 + i).to("cuda") for i in range(2)]
    results, errors = [None, None], []

    def worker(i):
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                outs = []
                for _ in range(20):
                    out = torch.empty_like(cases[i].q)
                    faf.flash_attn_varlen_func(**cases[i].kwargs(), out=out)
                    outs.append(out)
                s.synchronize()
                assert faf.read_device_error() == 0
            results[i] = [o.cpu() for o in outs]
        except Exception as e:  # reported below
            errors.append(e)

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not errors, errors
    for i in range(2):
        ref, _ = oracle(baseline_config("C4", batch=6, seed=50 + i))
        for o in results[i]:
            assert (o.float() - ref).abs().max().item() <= OUT_TOL
