"""Host-side checks that need no GPU: the C ABI library loads, exports every symbol
declared in include/tfa.h, and rejects invalid arguments with the documented codes
before touching the device. Also the Python-level argument checks."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from toy_flash_attn import _lib
from toy_flash_attn import flash_attention_func as faf

HEADER = Path(__file__).resolve().parent.parent / "include" / "tfa.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"TFA_API\s+[\w\s\*]+?\b(tfa_\w+)\s*\(", text))


def test_header_declares_expected_symbols():
    assert declared_symbols() == set(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_library_exports_nothing_else():
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.lib_path())], capture_output=True, text=True).stdout
    funcs = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert funcs == declared_symbols()


def test_status_strings():
    lib = _lib.load()
    for code in _lib.STATUS_NAMES:
        assert lib.tfa_status_string(code).decode()
    assert lib.tfa_status_string(12345) == b"unknown status"


def _params(**over):
    p = _lib.TfaFwdParams()
    buf = ctypes.create_string_buffer(1 << 16)
    base = (ctypes.addressof(buf) + 255) // 256 * 256
    p.q = p.k = p.v = p.out = base
    p.cu_seqlens_q = p.seqused_k = p.block_table = base
    p.q_stride[:] = [256, 64, 1]
    p.out_stride[:] = [256, 64, 1]
    p.k_stride[:] = [16 * 2 * 64, 2 * 64, 64, 1]
    p.v_stride[:] = [16 * 2 * 64, 2 * 64, 64, 1]
    p.block_table_stride0 = 8
    p.batch, p.total_q, p.num_q_heads, p.num_kv_heads = 1, 1, 4, 2
    p.head_dim, p.block_size, p.num_blocks = 64, 16, 8
    p.max_seqlen_q, p.max_seqlen_k = 1, 16
    p.window_left = p.window_right = -1
    for k, v in over.items():
        setattr(p, k, v)
    return p, buf


@pytest.mark.parametrize(
    "over, code",
    [
        (dict(head_dim=96), -2),
        (dict(head_dim=32), -2),
        (dict(num_q_heads=5), -3),
        (dict(block_size=24), -4),
        (dict(block_size=3), -4),
        (dict(window_left=-2), -6),
        (dict(num_blocks=0), -6),
        (dict(q=None), -1),
        (dict(block_table=None), -1),
    ],
)
def test_fwd_rejects_invalid_arguments(over, code):
    p, _buf = _params(**over)
    assert _lib.load().tfa_fwd(ctypes.byref(p), None, 0, None) == code


def test_fwd_rejects_misaligned_pointer_and_strides():
    p, _buf = _params()
    p.q = p.q + 2
    assert _lib.load().tfa_fwd(ctypes.byref(p), None, 0, None) == -5
    p, _buf = _params()
    p.k_stride[3] = 2
    assert _lib.load().tfa_fwd(ctypes.byref(p), None, 0, None) == -5
    p, _buf = _params()
    p.k_stride[1] = 36  # 72 bytes: not a multiple of 16
    assert _lib.load().tfa_fwd(ctypes.byref(p), None, 0, None) == -5


def test_empty_batch_is_a_no_op():
    p, _buf = _params(batch=0)
    assert _lib.load().tfa_fwd(ctypes.byref(p), None, 0, None) == 0
    p, _buf = _params(total_q=0)
    assert _lib.load().tfa_fwd(ctypes.byref(p), None, 0, None) == 0


def test_plan_without_gpu_uses_b200_sm_count():
    p, _buf = _params(max_seqlen_k=2048, num_q_heads=14, num_kv_heads=2)
    info = _lib.TfaPlanInfo()
    assert _lib.load().tfa_plan(ctypes.byref(p), -1, ctypes.byref(info)) == 0
    assert info.kernel == 0 and info.rows_per_tile == 16
    assert info.max_splits == 16 and info.split_cap == 1 and info.combine == 2  # merged in the decode kernel
    assert info.grid == min(info.num_items, 148)
    p.max_seqlen_q = 128
    assert _lib.load().tfa_plan(ctypes.byref(p), -1, ctypes.byref(info)) == 0
    assert info.kernel == 1 and info.rows_per_tile == 128 and info.q_tiles == 7  # few items: 128-row items
    p.batch, p.total_q, p.max_seqlen_q = 64, 64 * 4096, 4096
    assert _lib.load().tfa_plan(ctypes.byref(p), -1, ctypes.byref(info)) == 0
    assert info.rows_per_tile == 256 and info.q_tiles == 112


def test_workspace_size_grows_with_splits():
    p, _buf = _params(max_seqlen_k=32768, batch=4, total_q=4)
    lib = _lib.load()
    p.num_splits = 1
    one = lib.tfa_workspace_size(ctypes.byref(p), -1)
    p.num_splits = 8
    eight = lib.tfa_workspace_size(ctypes.byref(p), -1)
    assert one == 256 and eight > one
    # control block and the fixed 64 KB region of the decode kernel's split counters, then
    # split LSEs and split outputs
    assert eight == 65536 + ((8 * 4 * 4 * 4 + 255) // 256) * 256 + 8 * 4 * 4 * 64 * 4


def test_python_wrapper_rejects_cpu_tensors():
    q = torch.zeros(1, 4, 64, dtype=torch.bfloat16)
    kc = torch.zeros(2, 16, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="expects CUDA tensors"):
        faf.flash_attn_varlen_func(q, kc, kc, 1, torch.tensor([0, 1], dtype=torch.int32), 16, None,
                                   torch.tensor([16], dtype=torch.int32), True, None,
                                   torch.zeros(1, 1, dtype=torch.int32))


def test_unsupported_modes_raise(monkeypatch):
    monkeypatch.setenv("TOY_FLASH_ATTN_USE", "fp32")
    with pytest.raises(NotImplementedError):
        faf.flash_attn_varlen_func(None, None, None, 1, None, 1, None, None, False, None, block_table=object())


def test_reference_mode_matches_oracle_on_cpu(monkeypatch):
    """TOY_FLASH_ATTN_USE=reference is the explicitly selected PyTorch path."""
    from oracle.paged_attention import paged_attention_oracle
    from toy_flash_attn.workloads import reference_case

    monkeypatch.setenv("TOY_FLASH_ATTN_USE", "reference")
    case = reference_case([2, 6], [8, 8], causal=True, window_size=(2, 0), dtype=torch.float32)
    out = faf.flash_attn_varlen_func(**case.kwargs())
    ref, _ = paged_attention_oracle(case.q, case.k_cache, case.v_cache, case.cu_seqlens_q, case.seqused_k,
                                    case.block_table, True, (2, 0))
    torch.testing.assert_close(out, ref, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("kv_heads, q_heads, splits, cap, pages", [
    (8, 32, 32, 8, 1),  # C5 on one GPU: page decode, items of 8 tiles x 8 kv heads
    (1, 4, 10, 28, 0),  # C5 shard of one kv head per GPU (8 GPUs): finer splits for the tail
])
def test_plan_split_rule_large_decode(kv_heads, q_heads, splits, cap, pages):
    """Large decode calls get items of at least 16 tiles and ~16 items per SM of the
    max-length work bound (per kv head; the page kernel's items carry all 8 kv heads of a
    sequence, so its cap is that divided by 8); the split count never exceeds what the
    longest sequence needs."""
    p, _buf = _params(batch=256, total_q=256, num_q_heads=q_heads, num_kv_heads=kv_heads, head_dim=128,
                      max_seqlen_q=1, max_seqlen_k=32768, causal=1)
    p.q_stride[:] = [q_heads * 128, 128, 1]
    p.out_stride[:] = [q_heads * 128, 128, 1]
    p.k_stride[:] = [16 * kv_heads * 128, kv_heads * 128, 128, 1]
    p.v_stride[:] = [16 * kv_heads * 128, kv_heads * 128, 128, 1]
    p.num_blocks, p.block_table_stride0 = 1 << 21, 2048
    info = _lib.TfaPlanInfo()
    assert _lib.load().tfa_plan(ctypes.byref(p), -1, ctypes.byref(info)) == 0
    assert info.kernel == 0 and info.grid == 148 and info.pages == pages
    assert (info.max_splits, info.split_cap) == (splits, cap)


def test_plan_small_decode_keeps_coarse_splits():
    """C4-sized calls: 128 (sequence, kv head) groups already fill one wave of 148 SMs, so
    the latency-bound rule drops the split (a second wave and the combine cost more), and
    the per-head kernel runs (the page kernel would need splits to fill the grid)."""
    p, _buf = _params(batch=16, total_q=16, num_q_heads=32, num_kv_heads=8, head_dim=64,
                      max_seqlen_q=1, max_seqlen_k=8192, causal=1, window_left=1024, window_right=0)
    p.q_stride[:] = [32 * 64, 64, 1]
    p.out_stride[:] = [32 * 64, 64, 1]
    p.k_stride[:] = [16 * 8 * 64, 8 * 64, 64, 1]
    p.v_stride[:] = [16 * 8 * 64, 8 * 64, 64, 1]
    p.num_blocks, p.block_table_stride0 = 8192, 512
    info = _lib.TfaPlanInfo()
    assert _lib.load().tfa_plan(ctypes.byref(p), -1, ctypes.byref(info)) == 0
    assert info.kernel == 0 and info.pages == 0 and info.max_splits == 1 and info.combine == 0


@pytest.mark.parametrize("batch, heads, kv_heads, max_q, kernel", [
    (8, 16, 4, 64, 2),    # prefill-shaped call with several sequences: both kernels
    (4, 16, 4, 64, 1),    # few sequences: prefill kernel alone
    (8, 34, 1, 64, 1),    # group > 16: no decode-shaped sequence can exist
    (8, 16, 4, 4, 0),     # every sequence decode-shaped: decode kernel alone
])
def test_plan_mixed_dispatch(batch, heads, kv_heads, max_q, kernel):
    p, _buf = _params(batch=batch, total_q=batch * max_q, num_q_heads=heads, num_kv_heads=kv_heads, head_dim=64,
                      max_seqlen_q=max_q, max_seqlen_k=4096, causal=1)
    p.q_stride[:] = [heads * 64, 64, 1]
    p.out_stride[:] = [heads * 64, 64, 1]
    p.k_stride[:] = [16 * kv_heads * 64, kv_heads * 64, 64, 1]
    p.v_stride[:] = [16 * kv_heads * 64, kv_heads * 64, 64, 1]
    p.num_blocks, p.block_table_stride0 = 4096, 256
    lib = _lib.load()
    info = _lib.TfaPlanInfo()
    assert lib.tfa_plan(ctypes.byref(p), -1, ctypes.byref(info)) == 0
    assert info.kernel == kernel
    assert lib.tfa_workspace_size(ctypes.byref(p), -1) == info.workspace_bytes


def _decode_params(batch=256, hq=32, hkv=8, hd=128, bs=16, max_q=1, max_k=32768, num_splits=0):
    p, buf = _params(batch=batch, total_q=batch * max_q, num_q_heads=hq, num_kv_heads=hkv, head_dim=hd,
                     block_size=bs, max_seqlen_q=max_q, max_seqlen_k=max_k, causal=1)
    p.q_stride[:] = [hq * hd, hd, 1]
    p.out_stride[:] = [hq * hd, hd, 1]
    p.k_stride[:] = [bs * hkv * hd, hkv * hd, hd, 1]
    p.v_stride[:] = [bs * hkv * hd, hkv * hd, hd, 1]
    p.num_blocks, p.block_table_stride0 = 1 << 21, (max_k + bs - 1) // bs
    p.num_splits = num_splits
    return p, buf


@pytest.mark.parametrize("over, pages", [
    (dict(), 1),                          # C5: 8 kv heads, 16-slot pages, one token, a large call
    (dict(hd=64), 1),
    (dict(hq=8), 1),                      # GQA group 1
    (dict(hkv=4, hq=16), 0),              # 4 kv heads: a page is 64 rows
    (dict(bs=32), 0),                     # 32-slot pages
    (dict(max_q=2), 0),                   # two tokens per sequence
    (dict(hq=64, hd=64), 0),              # GQA group 8
    (dict(num_splits=4), 0),              # forced split count
    (dict(batch=2, max_k=4096), 0),       # latency-bound
])
def test_plan_page_decode_selection(over, pages):
    """The page decode kernel is planned only for large one-token decode calls with 8 kv
    heads, 16-slot pages and a GQA group of 1, 2 or 4; its items count per sequence."""
    p, _buf = _decode_params(**over)
    info = _lib.TfaPlanInfo()
    assert _lib.load().tfa_plan(ctypes.byref(p), -1, ctypes.byref(info)) == 0
    assert info.kernel == 0 and info.pages == pages
    per_group = p.batch * (1 if pages else p.num_kv_heads)
    assert info.num_items == info.max_splits * per_group
    if pages:
        assert info.combine == 1 and info.item_list == 0


def test_plan_info_mirror_covers_the_c_struct():
    """tfa_plan writes nothing past the ctypes mirror of tfa_plan_info (a field added to the
    C struct but not to the mirror would overwrite the caller's memory)."""
    size = ctypes.sizeof(_lib.TfaPlanInfo)
    buf = (ctypes.c_ubyte * (size + 64))(*([0xA5] * (size + 64)))
    p, _b = _decode_params()
    info = _lib.TfaPlanInfo.from_buffer(buf)
    assert _lib.load().tfa_plan(ctypes.byref(p), -1, ctypes.byref(info)) == 0
    assert bytes(buf[size:]) == bytes([0xA5] * 64)
    assert info.pages == 1 and info.workspace_bytes > 0
