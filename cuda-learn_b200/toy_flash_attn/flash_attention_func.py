"""Paged-KV attention entry points (the ``toy_flash_attn.flash_attention_func`` surface).

Mirrors ``flash_attention_backend/toy_flash_attn/flash_attention_func.py`` of the
reference: ``flash_attn_varlen_func`` (``:245-291``) dispatches on the environment key
``TOY_FLASH_ATTN_USE``:

* ``bf16`` (default): :func:`flash_attn_varlen_with_block_cu_bf16`, the sm_100a kernels
  behind the C ABI of ``include/tfa.h`` (replaces ``:518-600`` + the v8 op);
* ``reference``: :func:`flash_attn_varlen_with_block`, a plain PyTorch restatement of the
  reference's paged path (``:314-408``), selected explicitly and never used as a fallback;
* ``fp32`` / ``official_paged``: not provided (the reference's v4-only fp32 debug op and
  its monkey-patch to vLLM FA2, ``:275-282,294-312``); they raise ``NotImplementedError``.

The argument checks raise the same exception types as the reference
(``ValueError`` for device / shape problems, ``TypeError`` for dtypes, ``:111-144``).
"""

from __future__ import annotations

import ctypes
import os
import struct
import threading
from itertools import count
from pathlib import Path

import torch

from . import _lib

_CUDA_VALUE_DTYPE = torch.bfloat16
_CUDA_INDEX_DTYPE = torch.int32
_TFA_ERR_WORKSPACE = -7
_DUMP_COUNTER = count()

__all__ = [
    "flash_attn_varlen_func",
    "flash_attn_varlen_with_block",
    "flash_attn_varlen_with_block_cu_bf16",
    "flash_attn_varlen_without_block",
    "kv_cache_update_cu",
    "plan",
]


# ---------------------------------------------------------------------------
# debug hooks kept from the reference (same environment variables, same payload keys)
# ---------------------------------------------------------------------------
def _tensor_debug_str(name: str, tensor: torch.Tensor | None) -> str:
    if tensor is None:
        return f"{name}=None"
    return (
        f"{name}(shape={tuple(tensor.shape)}, dtype={tensor.dtype}, "
        f"device={tensor.device}, contiguous={tensor.is_contiguous()})"
    )


def _maybe_log_cuda_inputs(**tensors) -> None:
    if os.environ.get("TOY_FLASH_ATTN_DEBUG", "0") != "1":
        return
    print(
        "[toy_flash_attn] flash_attn_varlen_with_block_cu inputs:",
        ", ".join(_tensor_debug_str(n, t) for n, t in tensors.items()),
        flush=True,
    )


def _clone_for_dump(value):
    if isinstance(value, torch.Tensor):
        return value.detach().cpu().clone()
    if isinstance(value, (tuple, list)):
        return type(value)(_clone_for_dump(v) for v in value)
    if isinstance(value, dict):
        return {k: _clone_for_dump(v) for k, v in value.items()}
    return value


def _maybe_dump_flash_attn_context(op_name: str, **payload) -> None:
    """Saves the call as ``NNNNN_<op_name>.pt`` under ``TOY_FLASH_ATTN_DUMP_DIR``
    (same file naming and payload keys as ``flash_attention_func.py:89-99``)."""
    dump_dir = os.environ.get("TOY_FLASH_ATTN_DUMP_DIR")
    if not dump_dir:
        return
    path = Path(dump_dir).expanduser().resolve()
    path.mkdir(parents=True, exist_ok=True)
    file_path = path / f"{next(_DUMP_COUNTER):05d}_{op_name}.pt"
    torch.save(_clone_for_dump(payload), file_path)
    print(f"[toy_flash_attn] dumped {op_name} context to {file_path}", flush=True)


def _layer_debug_meta(layer) -> dict:
    if layer is None:
        return {}
    return {"layer_name": type(layer).__name__, "layer_idx": getattr(layer, "layer_idx", None)}


# ---------------------------------------------------------------------------
# argument checks (flash_attention_func.py:111-144)
# ---------------------------------------------------------------------------
def _check_cuda_tensor(name: str, tensor: torch.Tensor, *, expected_device, expected_dtype) -> None:
    if tensor.device != expected_device:
        raise ValueError(f"{name}.device={tensor.device} does not match q.device={expected_device}")
    if tensor.dtype != expected_dtype:
        raise TypeError(f"{name}.dtype={tensor.dtype} does not match CUDA op requirement {expected_dtype}")


def _check_gqa_heads(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor) -> None:
    q_heads = q.shape[1]
    kv_heads = k.shape[2]
    if v.shape[2] != kv_heads:
        raise ValueError(f"k/v head count mismatch, got k_heads={kv_heads}, v_heads={v.shape[2]}")
    if out.shape[1] != q_heads:
        raise ValueError(f"out head count must match q, got q_heads={q_heads}, out_heads={out.shape[1]}")
    if q_heads % kv_heads != 0:
        raise ValueError(
            f"GQA requires q_heads to be divisible by kv_heads, got q_heads={q_heads}, kv_heads={kv_heads}"
        )


# ---------------------------------------------------------------------------
# dispatcher (flash_attention_func.py:245-291)
# ---------------------------------------------------------------------------
def flash_attn_varlen_func(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    max_seqlen_q: int | None,
    cu_seqlens_q: torch.Tensor,
    max_seqlen_k: int | None,
    cu_seqlens_k: torch.Tensor | None,
    seqused_k: torch.Tensor | None = None,
    causal=False,
    window_size: tuple[int, int] | None = None,
    block_table=None,
    layer=None,
    out: torch.Tensor | None = None,
    *,
    softmax_lse: torch.Tensor | None = None,
    softmax_scale: float | None = None,
    num_splits: int = 0,
) -> torch.Tensor:
    """Decoder attention over a paged KV cache; q and kv are tail aligned.

    Same positional signature as the reference. Keyword-only extras: ``softmax_lse``
    (optional fp32 ``[total_q, num_q_heads]`` output, natural log), ``softmax_scale``
    (default ``1/sqrt(head_dim)`` as the reference) and ``num_splits`` (0 = automatic).
    """
    use = os.getenv("TOY_FLASH_ATTN_USE", "bf16")
    if block_table is None:
        return flash_attn_varlen_without_block(
            q, k, v, max_seqlen_q, cu_seqlens_q, max_seqlen_k, cu_seqlens_k, causal, window_size, out
        )
    if use == "reference":
        return flash_attn_varlen_with_block(
            q, k, v, max_seqlen_q, cu_seqlens_q, max_seqlen_k, seqused_k, causal, window_size, block_table, out,
            layer=layer,
        )
    if use in ("fp32", "official_paged"):
        raise NotImplementedError(
            f"TOY_FLASH_ATTN_USE={use!r} is not provided by the sm_100a backend; use 'bf16' or 'reference'"
        )
    return flash_attn_varlen_with_block_cu_bf16(
        q, k, v, max_seqlen_q, cu_seqlens_q, max_seqlen_k, seqused_k, causal, window_size, block_table, out,
        layer=layer, softmax_lse=softmax_lse, softmax_scale=softmax_scale, num_splits=num_splits,
    )


# ---------------------------------------------------------------------------
# sm_100a path
# ---------------------------------------------------------------------------
_workspaces: dict[tuple[int, int], torch.Tensor] = {}
# Workspaces replaced by a larger one stay allocated: a CUDA graph captured with an earlier
# call (vLLM captures one per batch size) keeps using the old buffer's address on replay,
# and freed memory could be handed to another tensor.
_retired_workspaces: list[torch.Tensor] = []


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """Zero-filled per (device, stream) workspace, grown on demand. The library keeps its
    control words zeroed between calls, so the buffer is only cleared when created."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        if ws is not None:
            _retired_workspaces.append(ws)
        ws = torch.zeros(max(nbytes, 4096), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


# struct tfa_fwd_params packed in one call (the fields in declaration order, native 64-bit
# layout; the trailing 4 bytes are the struct's padding)
_PARAM_FMT = "=Q3qQ4qQ4qQ3qQQQQ10q3ifi4x"
assert struct.calcsize(_PARAM_FMT) == ctypes.sizeof(_lib.TfaFwdParams)
_tls = threading.local()


def _current_raw_stream(device_index: int) -> int:
    """The current CUDA stream of a device as an integer handle."""
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return raw(device_index)
    return torch.cuda.current_stream(device_index).cuda_stream


def _fill_params(
    q, k, v, out, cu_seqlens_q, seqused_k, block_table, max_seqlen_q, max_seqlen_k, causal, window_size,
    softmax_lse, softmax_scale, num_splits, reuse: bool = False,
) -> _lib.TfaFwdParams:
    """Argument struct of one call. With ``reuse`` the struct object is this thread's
    scratch copy, overwritten by its next call (the hot path packs it in one step)."""
    if reuse:
        p = getattr(_tls, "params", None)
        if p is None:
            p = _tls.params = _lib.TfaFwdParams()
        wl, wr = (-1, -1) if window_size is None else (int(window_size[0]), int(window_size[1]))
        qs, ks, vs, os_ = q.stride(), k.stride(), v.stride(), out.stride()
        struct.pack_into(
            _PARAM_FMT, p, 0,
            q.data_ptr(), *qs, k.data_ptr(), *ks, v.data_ptr(), *vs, out.data_ptr(), *os_,
            softmax_lse.data_ptr() if softmax_lse is not None else 0,
            cu_seqlens_q.data_ptr(), seqused_k.data_ptr(), block_table.data_ptr(), block_table.stride(0),
            seqused_k.numel(), q.shape[0], q.shape[1], k.shape[2], q.shape[2], k.shape[1], k.shape[0],
            int(max_seqlen_q), int(max_seqlen_k), 1 if causal else 0, wl, wr,
            float(softmax_scale) if softmax_scale is not None else 0.0, int(num_splits))
        return p
    p = _lib.TfaFwdParams()
    p.q = q.data_ptr()
    p.q_stride[:] = list(q.stride())
    p.k = k.data_ptr()
    p.k_stride[:] = list(k.stride())
    p.v = v.data_ptr()
    p.v_stride[:] = list(v.stride())
    p.out = out.data_ptr()
    p.out_stride[:] = list(out.stride())
    p.softmax_lse = softmax_lse.data_ptr() if softmax_lse is not None else None
    p.cu_seqlens_q = cu_seqlens_q.data_ptr()
    p.seqused_k = seqused_k.data_ptr()
    p.block_table = block_table.data_ptr()
    p.block_table_stride0 = block_table.stride(0)
    p.batch = seqused_k.numel()
    p.total_q = q.shape[0]
    p.num_q_heads = q.shape[1]
    p.num_kv_heads = k.shape[2]
    p.head_dim = q.shape[2]
    p.block_size = k.shape[1]
    p.num_blocks = k.shape[0]
    p.max_seqlen_q = int(max_seqlen_q)
    p.max_seqlen_k = int(max_seqlen_k)
    wl, wr = (-1, -1) if window_size is None else (int(window_size[0]), int(window_size[1]))
    p.causal = 1 if causal else 0
    p.window_left = wl
    p.window_right = wr
    p.softmax_scale = float(softmax_scale) if softmax_scale is not None else 0.0
    p.num_splits = int(num_splits)
    return p


def plan(q, k, v, cu_seqlens_q, seqused_k, block_table, max_seqlen_q, max_seqlen_k, causal=False,
         window_size=None, num_splits=0) -> dict:
    """What the C ABI would launch for this call (``tfa_plan``), as a dict."""
    lib = _lib.load()
    out = torch.empty_like(q) if q.numel() else q
    p = _fill_params(q, k, v, out, cu_seqlens_q, seqused_k, block_table, max_seqlen_q, max_seqlen_k, causal,
                     window_size, None, None, num_splits)
    info = _lib.TfaPlanInfo()
    dev = q.device.index if q.device.type == "cuda" and q.device.index is not None else 0
    _lib.check(lib.tfa_plan(ctypes.byref(p), dev, ctypes.byref(info)), "tfa_plan")
    return {name: getattr(info, name) for name, _ in info._fields_}


def flash_attn_varlen_with_block_cu_bf16(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    max_seqlen_q: int,
    cu_seqlens_q: torch.Tensor,
    max_seqlen_k: int,
    seqused_k: torch.Tensor,
    causal=False,
    window_size: tuple[int, int] | None = None,
    block_table=None,
    out: torch.Tensor | None = None,
    layer=None,
    *,
    softmax_lse: torch.Tensor | None = None,
    softmax_scale: float | None = None,
    num_splits: int = 0,
    main_events: tuple[torch.cuda.Event, torch.cuda.Event] | None = None,
) -> torch.Tensor:
    """sm_100a paged attention forward; same checks and in-place ``out`` contract as the
    reference wrapper (``flash_attention_func.py:518-600``). ``main_events`` (two
    ``torch.cuda.Event``) are recorded around the attention kernel alone (``tfa_fwd_timed``)."""
    if out is None:
        out = torch.empty_like(q)
    if window_size is None:
        window_size = (-1, -1)
    if block_table is None:
        raise ValueError("block_table must not be None for flash_attn_varlen_with_block_cu")
    if not q.is_cuda:
        raise ValueError("flash_attn_varlen_with_block_cu expects CUDA tensors")
    _maybe_log_cuda_inputs(q=q, k=k, v=v, cu_seqlens_q=cu_seqlens_q, seqused_k=seqused_k,
                           block_table=block_table, out=out)
    dev = q.device
    di = q.get_device()
    for name, t, dt in (("q", q, _CUDA_VALUE_DTYPE), ("k", k, _CUDA_VALUE_DTYPE), ("v", v, _CUDA_VALUE_DTYPE),
                        ("cu_seqlens_q", cu_seqlens_q, _CUDA_INDEX_DTYPE), ("seqused_k", seqused_k, _CUDA_INDEX_DTYPE),
                        ("block_table", block_table, _CUDA_INDEX_DTYPE), ("out", out, _CUDA_VALUE_DTYPE)):
        if t.get_device() != di or t.dtype is not dt:
            _check_cuda_tensor(name, t, expected_device=dev, expected_dtype=dt)  # raises with the reference's message
    _check_gqa_heads(q, k, v, out)
    if q.shape != out.shape:
        raise ValueError(f"q and out must have the same shape, got {tuple(q.shape)} and {tuple(out.shape)}")
    if k.shape != v.shape or k.dim() != 4:
        raise ValueError("k/v must be [num_blocks, block_size, num_kv_heads, head_dim] with equal shapes")
    if block_table.dim() != 2 or block_table.stride(1) != 1:
        raise ValueError("block_table must be a 2-D tensor with a contiguous last dimension")
    if softmax_lse is not None:
        _check_cuda_tensor("softmax_lse", softmax_lse, expected_device=dev, expected_dtype=torch.float32)
        if tuple(softmax_lse.shape) != (q.shape[0], q.shape[1]) or not softmax_lse.is_contiguous():
            raise ValueError("softmax_lse must be a contiguous [total_q, num_q_heads] fp32 tensor")
    if not cu_seqlens_q.is_contiguous() or not seqused_k.is_contiguous():
        raise ValueError("cu_seqlens_q and seqused_k must be contiguous")
    if cu_seqlens_q.numel() != seqused_k.numel() + 1:
        raise ValueError("cu_seqlens_q must have batch + 1 entries")

    lib = _lib.load()
    p = _fill_params(q, k, v, out, cu_seqlens_q, seqused_k, block_table, max_seqlen_q, max_seqlen_k, causal,
                     window_size, softmax_lse, softmax_scale, num_splits, reuse=True)
    prev = torch.cuda.current_device()
    if prev != di:
        torch.cuda.set_device(di)
    try:
        stream = _current_raw_stream(di)
        ws = _workspace(dev, stream, 0)
        if main_events is None:
            rc = lib.tfa_fwd(ctypes.byref(p), ws.data_ptr(), ws.numel(), stream)
            if rc == _TFA_ERR_WORKSPACE:  # first call of a larger shape on this stream: grow and retry
                ws = _workspace(dev, stream, max(lib.tfa_workspace_size(ctypes.byref(p), di), 4096))
                rc = lib.tfa_fwd(ctypes.byref(p), ws.data_ptr(), ws.numel(), stream)
            _lib.check(rc, "tfa_fwd")
        else:
            ws = _workspace(dev, stream, max(lib.tfa_workspace_size(ctypes.byref(p), di), 4096))
            ev0, ev1 = main_events
            for ev in (ev0, ev1):
                if not ev.cuda_event:  # torch creates the event on its first record
                    ev.record()
            _lib.check(lib.tfa_fwd_timed(ctypes.byref(p), ws.data_ptr(), ws.numel(), stream, ev0.cuda_event,
                                         ev1.cuda_event), "tfa_fwd_timed")
    finally:
        if prev != di:
            torch.cuda.set_device(prev)
    _maybe_dump_flash_attn_context(
        "with_block_cu",
        q=q, k=k, v=v, max_seqlen_q=max_seqlen_q, cu_seqlens_q=cu_seqlens_q, max_seqlen_k=max_seqlen_k,
        seqused_k=seqused_k, causal=causal, window_size=window_size, block_table=block_table,
        debug_meta=_layer_debug_meta(layer), result=out,
    )
    return out


def read_device_error(device: torch.device | None = None) -> int:
    """Synchronises the current stream and returns (and clears) the kernels' error word
    of this stream's workspace; 0 means no error was recorded."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev).cuda_stream
    ws = _workspace(dev, stream, 4096)
    err = ctypes.c_int(0)
    _lib.check(_lib.load().tfa_read_device_error(ws.data_ptr(), stream, ctypes.byref(err)), "tfa_read_device_error")
    if err.value >= 100 and err.value < 110:
        ws.zero_()  # a kernel unwound on a time limit: its scheduler words may be stale
    return err.value


def gather_kv_cu(k: torch.Tensor, v: torch.Tensor, seqused_k: torch.Tensor, block_table: torch.Tensor,
                 max_seqlen_k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Dense ``[sum(kv_len), Hkv, d]`` copies of K and V staged through the kernels' TMA
    gather path (``tfa_gather_kv``); used to check the gather bit-exactly."""
    lib = _lib.load()
    dev = k.device
    kv_off = torch.zeros(seqused_k.numel() + 1, dtype=torch.int64, device=dev)
    kv_off[1:] = torch.cumsum(seqused_k.to(torch.int64), 0)
    total = int(kv_off[-1].item())
    k_out = torch.empty(max(total, 1), k.shape[2], k.shape[3], dtype=k.dtype, device=dev)
    v_out = torch.empty_like(k_out)
    dummy_q = torch.empty(1, k.shape[2], k.shape[3], dtype=k.dtype, device=dev)
    cu = torch.zeros(seqused_k.numel() + 1, dtype=torch.int32, device=dev)
    p = _fill_params(dummy_q, k, v, dummy_q, cu, seqused_k, block_table, 1, max_seqlen_k, False, None, None, None, 0)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        ws = _workspace(dev, stream, 4096)
        _lib.check(lib.tfa_gather_kv(ctypes.byref(p), kv_off.data_ptr(), k_out.data_ptr(), v_out.data_ptr(),
                                     ws.data_ptr(), stream), "tfa_gather_kv")
    return k_out[:total], v_out[:total]


def kv_cache_update_cu(key: torch.Tensor, value: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                       slot_mapping: torch.Tensor) -> None:
    """Scatter new K/V rows into the paged cache (``tfa_kv_cache_update``); slots < 0 are
    skipped, as in ``ToyFlashAttentionImpl.do_kv_cache_update`` (``impl.py:121-144``)."""
    lib = _lib.load()
    if slot_mapping.dtype != torch.int64:
        slot_mapping = slot_mapping.to(torch.int64)
    slot_mapping = slot_mapping.contiguous()
    n = min(key.shape[0], slot_mapping.numel())
    dev = key.device

    def arr(t, n_):
        return (ctypes.c_int64 * n_)(*t.stride()[:n_])

    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        ws = _workspace(dev, stream, 4096)
        _lib.check(
            lib.tfa_kv_cache_update(
                key.data_ptr(), arr(key, 2), value.data_ptr(), arr(value, 2), key_cache.data_ptr(),
                arr(key_cache, 3), value_cache.data_ptr(), arr(value_cache, 3), slot_mapping.data_ptr(), n,
                key.shape[1], key.shape[2], key_cache.shape[1], key_cache.shape[0], ws.data_ptr(), stream,
            ),
            "tfa_kv_cache_update",
        )


# ---------------------------------------------------------------------------
# TOY_FLASH_ATTN_USE=reference: plain PyTorch restatement of the reference's paged path
# ---------------------------------------------------------------------------
def flash_attn_varlen_with_block(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    max_seqlen_q: int,
    cu_seqlens_q: torch.Tensor,
    max_seqlen_k: int,
    seqused_k: torch.Tensor,
    causal=False,
    window_size: tuple[int, int] | None = None,
    block_table=None,
    out: torch.Tensor | None = None,
    layer=None,
) -> torch.Tensor:
    """Explicitly selected PyTorch path of ``flash_attention_func.py:314-408`` (math in the
    input dtype, masks built per row), vectorised over tokens."""
    assert block_table is not None
    if out is None:
        out = torch.empty_like(q)
    bs = k.shape[1]
    cu = cu_seqlens_q.tolist()
    used = seqused_k.tolist()
    for b, kv_len in enumerate(used):
        q0, q1 = cu[b], cu[b + 1]
        Q = q[q0:q1]
        t = torch.arange(kv_len, device=q.device)
        pages = block_table[b].long()[t // bs]
        K, V = k[pages, t % bs], v[pages, t % bs]
        hq, hkv = Q.shape[1], K.shape[1]
        if hq % hkv != 0:
            raise ValueError(f"GQA requires q_heads to be divisible by kv_heads, got q_heads={hq}, kv_heads={hkv}")
        if hq != hkv:
            idx = torch.arange(hq, device=q.device) // (hq // hkv)
            K, V = K[:, idx], V[:, idx]
        S = Q.transpose(0, 1).matmul(K.permute(1, 2, 0)) / float(q.shape[2] ** 0.5)
        win = window_size
        if win is None or tuple(win) == (-1, -1):
            win = (kv_len, kv_len)
        if causal:
            win = (win[0], 0)
        off = kv_len - Q.shape[0]
        i = torch.arange(Q.shape[0], device=q.device).unsqueeze(1)
        j = t.unsqueeze(0)
        hidden = (j < i + off - win[0]) | (j >= i + off + 1 + win[1])
        P = S.masked_fill(hidden, float("-inf")).softmax(2)
        out[q0:q1] = P.matmul(V.transpose(0, 1)).transpose(0, 1)
    _maybe_dump_flash_attn_context(
        "with_block",
        q=q, k=k, v=v, max_seqlen_q=max_seqlen_q, cu_seqlens_q=cu_seqlens_q, max_seqlen_k=max_seqlen_k,
        seqused_k=seqused_k, causal=causal, window_size=window_size, block_table=block_table,
        debug_meta=_layer_debug_meta(layer), result=out,
    )
    return out


def flash_attn_varlen_without_block(
    q, k, v, max_seqlen_q, cu_seqlens_q, max_seqlen_k, cu_seqlens_k, causal=False, window_size=None, out=None
):
    """Non-paged varlen path (``flash_attention_func.py:411-457``) on the sm_100a kernels:
    the dense ``[total_k, Hkv, d]`` K/V are viewed as a cache of one-token blocks and a
    block table ``block_table[b, t] = cu_seqlens_k[b] + t`` is built on the device."""
    if cu_seqlens_k is None:
        raise ValueError("cu_seqlens_k is required when block_table is None")
    if out is None:
        out = torch.empty_like(q)
    batch = cu_seqlens_k.numel() - 1
    lens = (cu_seqlens_k[1:] - cu_seqlens_k[:-1]).to(torch.int32)
    mk = int(max_seqlen_k) if max_seqlen_k is not None else int(lens.max().item()) if batch else 0
    bt = (cu_seqlens_k[:-1].to(torch.int32).unsqueeze(1) +
          torch.arange(max(mk, 1), dtype=torch.int32, device=q.device).unsqueeze(0)).contiguous()
    k_pages = k.unsqueeze(1)
    v_pages = v.unsqueeze(1)
    mq = int(max_seqlen_q) if max_seqlen_q is not None else int((cu_seqlens_q[1:] - cu_seqlens_q[:-1]).max().item())
    return flash_attn_varlen_with_block_cu_bf16(
        q, k_pages, v_pages, mq, cu_seqlens_q, mk, lens.contiguous(), causal, window_size, bt, out,
    )
