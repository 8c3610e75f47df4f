"""Side-by-side on one GPU: the reference's own CUDA op (v8, built by build_ref_v8.py into
oracle/_ref/) against this repository's sm_100a kernels, on the BASELINE configurations it
supports (C1-C4: head_dim 64, block_size 16; v8 has no head_dim-128 instantiation, so C5
is out). Benchmark infrastructure only; nothing here is used by the product path.

Both ops get identical inputs; each call is timed alone with CUDA events after a 256 MB
L2 flush (plain calls, no CUDA graph, since v8 allocates its split buffers per call), and
both outputs are checked against the CPU oracle (fp32 math on the bf16 inputs).

    python oracle/compare_ref_v8.py          # prints one JSON line per configuration
"""

from __future__ import annotations

import importlib.util
import json
import statistics
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
for p in (REPO, REPO / "cuda-learn_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

from oracle.paged_attention import paged_attention_oracle  # noqa: E402
from toy_flash_attn import flash_attention_func as faf  # noqa: E402
from toy_flash_attn.workloads import baseline_config  # noqa: E402

L2_FLUSH_BYTES = 256 * 1024 * 1024


def load_v8():
    so = HERE / "_ref" / "toy_ref_v8.so"
    if not so.exists():
        raise SystemExit(f"{so} is not built: run oracle/build_ref_v8.py where the reference tree is mounted")
    spec = importlib.util.spec_from_file_location("toy_ref_v8", so)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def time_cold(fn, iters: int = 30) -> float:
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    t = []
    for _ in range(iters):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        t.append(e0.elapsed_time(e1))
    return statistics.median(t) * 1e3  # us


def main() -> None:
    v8 = load_v8()
    for name in ("C1", "C2", "C3", "C4"):
        case = baseline_config(name)
        ref, _ = paged_attention_oracle(case.q, case.k_cache, case.v_cache, case.cu_seqlens_q, case.seqused_k,
                                        case.block_table, case.causal, case.window_size)
        c = case.to("cuda")
        wl, wr = c.window_size if c.window_size is not None else (-1, -1)
        out_v8 = torch.empty_like(c.q)
        out_ours = torch.empty_like(c.q)

        def run_v8():
            v8.flash_attn_varlen_with_block_v8_64(c.q, c.k_cache, c.v_cache, c.max_seqlen_q, c.cu_seqlens_q,
                                                  c.max_seqlen_k, c.seqused_k, c.causal, wl, wr, c.block_table,
                                                  out_v8)

        def run_ours():
            faf.flash_attn_varlen_with_block_cu_bf16(c.q, c.k_cache, c.v_cache, c.max_seqlen_q, c.cu_seqlens_q,
                                                     c.max_seqlen_k, c.seqused_k, c.causal, c.window_size,
                                                     c.block_table, out_ours)

        us_v8, us_ours = time_cold(run_v8), time_cold(run_ours)
        err_v8 = (out_v8.float().cpu() - ref).abs().max().item()
        err_ours = (out_ours.float().cpu() - ref).abs().max().item()
        print(json.dumps({"config": name, "v8_us": round(us_v8, 2), "ours_us": round(us_ours, 2),
                          "speedup": round(us_v8 / us_ours, 2), "v8_max_abs_err": err_v8,
                          "ours_max_abs_err": err_ours, "timing": "plain calls, L2 flushed before each"}),
              flush=True)


if __name__ == "__main__":
    main()
