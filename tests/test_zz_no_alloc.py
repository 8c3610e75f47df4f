"""The allocation-free entry point ``tfa_fwd_static_workspace``.

It exists for callers that cannot allocate device memory (a serving loop that must not
call cudaMalloc once running, or a foreign-language host that binds the C ABI without a
device allocator): it uses a fixed array in the library's device memory as its split-KV
workspace. This file runs last so a failure here never hides the other tests; it also
passes when run alone in a fresh process.

Check: two calls in a row through the C ABI must agree with the caller-workspace entry
point ``tfa_fwd`` and with the CPU oracle within the parity tolerance (2e-2 on the output,
1e-3 on the LSE); kernel errors of these calls are read back with
``tfa_read_static_workspace_error``.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from oracle.paged_attention import paged_attention_oracle
from toy_flash_attn import _lib
from toy_flash_attn import flash_attention_func as faf
from toy_flash_attn.workloads import baseline_config, reference_case

pytestmark = pytest.mark.gpu

OUT_TOL = 2e-2
LSE_TOL = 1e-3
STATIC_WS_BYTES = 32 * 1024 * 1024


def _params(c, out, lse, num_splits=0):
    return faf._fill_params(c.q, c.k_cache, c.v_cache, out, c.cu_seqlens_q, c.seqused_k, c.block_table,
                            c.max_seqlen_q, c.max_seqlen_k, c.causal, c.window_size, lse, None, num_splits)


def _static_error() -> int:
    err = ctypes.c_int(-1)
    _lib.check(_lib.load().tfa_read_static_workspace_error(torch.cuda.current_stream().cuda_stream,
                                                           ctypes.byref(err)), "tfa_read_static_workspace_error")
    return err.value


def _item_list_case():
    g = torch.Generator().manual_seed(31)
    k_lens = [int(x) for x in torch.exp(torch.empty(48).uniform_(0, 8.3, generator=g)).round().clamp(1, 4096)]
    k_lens[0] = 4096
    return reference_case([1] * 48, k_lens, num_heads=16, num_kv_heads=4, head_dim=128, causal=True, block_size=16,
                          seed=31)


def _large_page_case():
    """One-token decode, 8 kv heads, 16-slot pages, a 32768-token bound: the caller-workspace
    entry point runs the page kernel with ~37 splits per sequence (> 32 MiB of partials)."""
    g = torch.Generator().manual_seed(53)
    k_lens = [int(x) for x in torch.randint(100, 2000, (64,), generator=g)]
    k_lens[5] = 32768
    return reference_case([1] * 64, k_lens, num_heads=32, num_kv_heads=8, head_dim=128, causal=True,
                          block_size=16, seed=53)


def _static_call(c, num_splits=0):
    out = torch.full_like(c.q, float("nan"))
    lse = torch.full((c.q.shape[0], c.q.shape[1]), float("nan"), dtype=torch.float32, device=c.q.device)
    p = _params(c, out, lse, num_splits)
    stream = torch.cuda.current_stream().cuda_stream
    rc = _lib.load().tfa_fwd_static_workspace(ctypes.byref(p), stream)
    _lib.check(rc, "tfa_fwd_static_workspace")
    torch.cuda.synchronize()
    return out, lse


@pytest.mark.parametrize(
    "make, splits",
    [
        (lambda: baseline_config("C2"), 0),                 # decode kernel, 16 splits + combine
        (lambda: baseline_config("C3"), 3),                 # prefill kernel, forced splits + combine
        (lambda: baseline_config("C4", batch=8), 0),        # sliding window, NaN cache slots
        (lambda: reference_case([1, 9], [700, 90], num_heads=8, num_kv_heads=2, head_dim=128, causal=True,
                                block_size=16, seed=3), 0),
        (_item_list_case, 0),                                # decode kernel with the device-built item list
        (lambda: reference_case([1, 1, 1, 40, 1, 1, 1, 2], [900, 700, 1200, 300, 129, 800, 60, 90], num_heads=8,
                                num_kv_heads=2, head_dim=64, causal=True, block_size=16, seed=8), 0),
                                                             # both kernels in one call (chunked prefill)
        (_large_page_case, 0),                               # planned per head here (page plan too large)
    ],
    ids=["C2", "C3_split3", "C4_b8", "hd128_mixed", "item_list", "mixed_dispatch", "large_pages_plan"],
)
def test_static_workspace_matches_tfa_fwd_twice(make, splits):
    case = make()
    c = case.to("cuda")
    ref_out = torch.empty_like(c.q)
    ref_lse = torch.empty(c.q.shape[0], c.q.shape[1], dtype=torch.float32, device="cuda")
    faf.flash_attn_varlen_func(**c.kwargs(), out=ref_out, softmax_lse=ref_lse, num_splits=splits)
    torch.cuda.synchronize()
    cpu_out, cpu_lse = paged_attention_oracle(case.q, case.k_cache, case.v_cache, case.cu_seqlens_q,
                                              case.seqused_k, case.block_table, case.causal, case.window_size)
    for _ in range(2):  # the array keeps the previous call's contents; results must not depend on it
        out, lse = _static_call(c, splits)
        assert _static_error() == 0
        assert torch.isfinite(out.float()).all()
        for want_out, want_lse in ((ref_out.float(), ref_lse), (cpu_out.to("cuda"), cpu_lse.to("cuda"))):
            assert (out.float() - want_out).abs().max().item() <= OUT_TOL
            fin = torch.isfinite(want_lse)
            assert torch.equal(fin, torch.isfinite(lse))
            assert (lse[fin] - want_lse[fin]).abs().max().item() <= LSE_TOL


def test_static_workspace_keeps_large_decode_on_the_per_head_plan():
    """The page decode kernel's split partials of this call exceed the static array, so the
    allocation-free entry point plans it for the per-head kernel, which fits (the call itself
    is checked against tfa_fwd and the oracle by the parametrized test above)."""
    c = _large_page_case().to("cuda")
    out = torch.empty_like(c.q)
    p = _params(c, out, None)
    info = _lib.TfaPlanInfo()
    assert _lib.load().tfa_plan(ctypes.byref(p), torch.cuda.current_device(), ctypes.byref(info)) == 0
    assert info.pages == 1 and info.workspace_bytes > STATIC_WS_BYTES
    _static_call(c)
    assert _static_error() == 0


def test_static_workspace_reports_bad_block_id():
    case = reference_case([1], [40], num_heads=2, num_kv_heads=1, block_size=16)
    case.block_table[0, 1] = 10_000  # outside the pool: read as zeros and reported as error 110
    c = case.to("cuda")
    _static_call(c)
    assert _static_error() == 110
    assert _static_error() == 0  # cleared


def test_static_workspace_rejects_oversized_call():
    # 64 sequences x 32 q heads x 32 splits x 128 dims of fp32 partials = 32 MiB, plus the LSEs and
    # the control block: more than the static array holds
    c = reference_case([1] * 64, [4096] * 64, num_heads=32, num_kv_heads=8, head_dim=128, causal=True,
                       block_size=16).to("cuda")
    out = torch.empty_like(c.q)
    p = _params(c, out, None, num_splits=32)
    dev = torch.cuda.current_device()
    need = _lib.load().tfa_workspace_size(ctypes.byref(p), dev)
    assert need > STATIC_WS_BYTES
    rc = _lib.load().tfa_fwd_static_workspace(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
    assert _lib.STATUS_NAMES[rc] == "TFA_ERR_STATIC_WORKSPACE_LIMIT"
