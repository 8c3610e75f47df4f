"""Generates the golden fixtures ``tests/golden/*.pt`` from the reference itself.

Run here (where the reference tree is mounted), never on the GPU box::

    python tests/golden/make_golden.py <path of the reference tree>

The reference module ``flash_attention_backend/toy_flash_attn/flash_attention_func.py``
cannot be imported in this container (it imports vLLM's FA2 CUDA extension and JIT-builds
CUDA at import, ``:9-12,147-242``). Its pure-PyTorch paged path
``flash_attn_varlen_with_block`` (``:314-408``) and the debug helpers it calls are taken
out of the file with ``ast`` and executed as they are. Each case is run twice on the CPU:
on fp32 copies of the bf16 inputs ("fp32 math on bf16 inputs", the oracle's contract)
and on the native bf16 inputs (what ``TOY_FLASH_ATTN_USE=reference`` computes). Inputs,
both outputs and the case parameters are saved; no reference source is stored.

The cases are the reference's own test cases (``tests/correctness/test_cuda_regression.py``,
``toy_flash_attn/flash_attention_func_test.py:881-929``, ``tests/correctness/test_paged_kv_parity.py``,
``bench/op/cases_op.py``) plus reduced versions of the five benchmark configurations.
"""

from __future__ import annotations

import ast
import sys
from itertools import count
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "cuda-learn_b200"))

from toy_flash_attn.workloads import baseline_config, reference_case  # noqa: E402

REF_FILE = "flash_attention_backend/toy_flash_attn/flash_attention_func.py"
WANTED = {
    "flash_attn_varlen_with_block",
    "_maybe_log_with_block_dtypes",
    "_maybe_dump_flash_attn_context",
    "_layer_debug_meta",
    "_clone_for_dump",
}


def load_reference_fn(ref_root: Path):
    src_path = ref_root / REF_FILE
    tree = ast.parse(src_path.read_text())
    body = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in WANTED]
    missing = WANTED - {n.name for n in body}
    if missing:
        raise RuntimeError(f"functions not found in {src_path}: {missing}")
    mod = ast.Module(body=body, type_ignores=[])
    import os

    ns = {"torch": torch, "os": os, "Path": Path, "count": count, "_DUMP_COUNTER": count()}
    ns["__builtins__"] = __builtins__
    exec(compile(mod, str(src_path), "exec"), ns)
    return ns["flash_attn_varlen_with_block"]


def cases():
    rc = reference_case
    yield rc([3, 5], head_dim=16, name="regression_full_q35_hd16")
    yield rc([2, 6], [8, 8], causal=True, window_size=(2, 0), name="regression_hd64_finite_q26_k88_causal_w20")
    yield rc([2, 6], name="regression_hd64_q26_full")
    yield rc([1, 1], name="regression_hd64_q11_full")
    yield rc([2, 6], causal=True, name="matrix_hd64_q26_causal")
    yield rc([2, 6], causal=True, window_size=(2, 0), name="matrix_hd64_q26_causal_w20")
    yield rc([1, 7], seed=1, name="matrix_hd64_q17_full_seed1")
    yield rc([3, 5], [6, 9], causal=True, name="matrix_hd64_q35_k69_causal")
    yield rc([4, 4], seed=423, name="matrix_hd64_q44_seed423")
    yield rc([4, 9], [8, 12], causal=True, window_size=(3, 0), name="tail_aligned_q49_k812_causal_w30")
    yield rc([2, 3], [5, 7], causal=True, name="tail_aligned_q23_k57_causal")
    yield rc([5, 5], [8, 12], causal=True, head_dim=16, name="paged_q55_k812_causal_hd16")
    yield rc([5, 5], causal=True, window_size=(3, 0), head_dim=16, name="paged_local_causal_w30_hd16")
    yield rc([1], [128], num_heads=8, num_kv_heads=2, causal=True, window_size=(64, 0), seed=7, block_size=16,
             name="op_gqa_case_b1_s128")
    yield rc([1, 1, 1, 1], [512, 384, 512, 256], num_heads=8, num_kv_heads=2, causal=True, seed=9, block_size=16,
             name="op_gqa_case_b4_s512")
    yield rc([1], [2048], num_heads=14, num_kv_heads=2, causal=True, seed=1, block_size=16,
             name="op_qwen_like_b1_s2048_h64")
    yield rc([3, 17], [40, 150], num_heads=4, num_kv_heads=1, head_dim=128, causal=True, seed=11, block_size=16,
             name="hd128_gqa4_q3_17_k40_150_causal")
    yield rc([200], [200], num_heads=6, num_kv_heads=2, causal=True, seed=12, block_size=32,
             name="prefill_q200_gqa3_bs32_causal")
    # reduced benchmark configurations (full C1 and C2 are small enough to keep as is)
    yield baseline_config("C1")
    yield baseline_config("C2", num_blocks=256)
    yield baseline_config("C4", batch=3, kv_range=(100, 400))
    yield baseline_config("C5", batch=3, kv_range=(17, 700), num_blocks=256)


def compact(case):
    """Keeps only the cache blocks the table references (fixtures stay small)."""
    bt = case.block_table
    used = sorted({int(x) for x in bt.flatten().tolist() if x >= 0})
    remap = {old: new for new, old in enumerate(used)}
    nbt = bt.clone()
    for i in range(bt.shape[0]):
        for j in range(bt.shape[1]):
            v = int(bt[i, j])
            nbt[i, j] = remap[v] if v >= 0 else -1
    idx = torch.tensor(used, dtype=torch.long)
    case.k_cache = case.k_cache[idx].clone()
    case.v_cache = case.v_cache[idx].clone()
    case.block_table = nbt
    return case


def main(ref_root: str) -> None:
    ref_fn = load_reference_fn(Path(ref_root))
    torch.set_num_threads(8)
    for case in cases():
        case = compact(case.to("cpu"))
        args = dict(
            max_seqlen_q=case.max_seqlen_q, cu_seqlens_q=case.cu_seqlens_q, max_seqlen_k=case.max_seqlen_k,
            seqused_k=case.seqused_k, causal=case.causal, window_size=case.window_size,
            block_table=case.block_table,
        )
        out32 = ref_fn(case.q.float(), case.k_cache.float(), case.v_cache.float(), **args, out=None)
        out16 = ref_fn(case.q, case.k_cache, case.v_cache, **args, out=None)
        payload = {
            "name": case.name,
            "q": case.q, "k": case.k_cache, "v": case.v_cache,
            "cu_seqlens_q": case.cu_seqlens_q, "seqused_k": case.seqused_k, "block_table": case.block_table,
            "max_seqlen_q": case.max_seqlen_q, "max_seqlen_k": case.max_seqlen_k,
            "causal": case.causal, "window_size": case.window_size,
            "out_ref_fp32": out32, "out_ref_bf16": out16,
            "generator": "reference flash_attn_varlen_with_block (flash_attention_func.py:314-408)",
        }
        torch.save(payload, HERE / f"{case.name}.pt")
        print(f"{case.name}: q{tuple(case.q.shape)} cache{tuple(case.k_cache.shape)} finite={bool(out32.isfinite().all())}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <path of the reference tree>")
    main(sys.argv[1])
