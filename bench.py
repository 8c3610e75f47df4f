#!/usr/bin/env python
"""Benchmark of the sm_100a paged-KV attention forward.

Headline: configuration C5 (large-batch decode: batch 256, kv lengths log-uniform in
[1024, 32768], 32 q / 8 kv heads, head_dim 128, block_size 16, a 2^21-block pool per GPU),
metric = KV bytes read per second (TB/s, every attended K/V byte counted once per kv head).
With N GPUs (one process per GPU, torchrun) the kv heads are sharded: each rank holds
8/N kv heads (and their q heads) of every sequence in its own pool; no collective runs in
the timed region. Total work is fixed, so scaling is "strong".

Per step: one forward call over the whole batch. Inputs are larger than L2 (8.60 GB of
K/V per step at one GPU), so no L2 flush is needed for the headline. C1-C4 (N=1 only)
are timed one call at a time from a CUDA graph with a 256 MB L2 flush between calls.

``--impl reference`` times the reference's own CPU algorithm (the oracle port of
``flash_attn_varlen_with_block``) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "cuda-learn_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "decode attn KV-read HBM TB/s (C5 large-batch decode)"
UNIT = "TB/s"
L2_BYTES = 126 * 1024 * 1024
# DRAM bytes (read + write) of one attention-kernel launch per algorithmic K/V byte, from
# ncu captures on a reduced C5 (traffic grows with the K/V bytes read): the page decode
# kernel (one GPU: 8 kv heads) and the per-head decode kernel (kv-head shards)
TRAFFIC_PER_KV_BYTE = {True: (471.88e6 + 5.79e6) / 471.49e6, False: (471.91e6 + 4.19e6) / 471.49e6}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-configs", action="store_true", help="skip the C1-C4 side table")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None, help="override C5 batch (debug only)")
    ap.add_argument("--num-blocks", type=int, default=None, help="override C5 pool size (debug only)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="target CPU baseline sample time")
    ap.add_argument("--profile-configs", default=None,
                    help="comma-separated configurations (C1..C5, P1, P2) to run --calls times each through "
                         "flash_attn_varlen_with_block_cu_bf16 and exit (a driver for ncu captures; no timing)")
    ap.add_argument("--calls", type=int, default=3)
    return ap.parse_args()


def run_profile_configs(args):
    from toy_flash_attn import flash_attention_func as faf
    from toy_flash_attn.workloads import baseline_config

    torch.cuda.set_device(0)
    for name in args.profile_configs.split(","):
        case = baseline_config(name, device="cuda")
        out = torch.empty_like(case.q)
        for _ in range(args.calls):
            call(case, out)
        torch.cuda.synchronize()
        if faf.read_device_error() != 0:
            raise SystemExit(f"{name}: kernel reported an error")
        print(f"ran {name} x{args.calls}", flush=True)
        del case, out
        torch.cuda.empty_cache()


def peaks() -> dict:
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# --------------------------------------------------------------------------------------
# clocks
# --------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------------------
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def allreduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------------------
# workloads
# --------------------------------------------------------------------------------------
def c5_shard(world: int, rank: int, args):
    """This rank's part of C5: a group of kv heads (with their q heads) of every sequence,
    in the rank's own pool. Only the shard is generated on the device."""
    from toy_flash_attn.sharding import plan_shards
    from toy_flash_attn.workloads import baseline_config, c5_kv_lengths

    if 8 % world:
        raise SystemExit("C5 shards its 8 kv heads: --gpus must divide 8")
    lens = c5_kv_lengths(args.batch or 256)
    shard = plan_shards(lens, 32, 8, world)[rank]
    assert shard.sequences == tuple(range(len(lens)))  # heads only: every rank keeps the whole batch
    hkv = shard.kv_heads[1] - shard.kv_heads[0]
    # same lengths and block tables on every rank, different q/K/V values per shard
    return baseline_config("C5", device="cuda", seed=5, batch=args.batch, num_blocks=args.num_blocks,
                           kv_heads=hkv, q_heads=shard.q_heads[1] - shard.q_heads[0], value_seed=5 + 7919 * rank)


def verify_c5(case, world: int, rank: int) -> dict:
    """Checks the call's output and LSE on a sample of sequences (the 16 longest and 16
    seeded-random others) against the CPU oracle, after timing. With N ranks every rank
    contributes its kv-head shard of the sample (q rows, live K/V pages, output, LSE),
    NCCL all-gathers them, and rank 0 reassembles all 32 q / 8 kv heads and checks the
    whole. Returns the errors (rank 0) against the tolerances of the parity tests."""
    from toy_flash_attn.workloads import compact_sample, verify_sequences

    out = torch.empty_like(case.q)
    lse = torch.empty(case.q.shape[0], case.q.shape[1], dtype=torch.float32, device=case.q.device)
    call(case, out, lse)
    torch.cuda.synchronize()
    seqs = verify_sequences(case.seqused_k.tolist())
    sub = compact_sample(case, seqs)
    cu = case.cu_seqlens_q.tolist()
    rows = torch.cat([torch.arange(cu[b], cu[b + 1], device=out.device) for b in seqs])
    parts = [sub.q, sub.k_cache, sub.v_cache, out[rows], lse[rows]]
    if world > 1:
        import torch.distributed as dist

        gathered = []
        for t in parts:
            t = t.contiguous()
            buf = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(buf, t)
            # rank r holds q heads [r*Hq/N, (r+1)*Hq/N) and kv heads [r*8/N, (r+1)*8/N):
            # concatenating along the head axis in rank order restores the full head order
            head_axis = 2 if t.dim() == 4 else 1
            gathered.append(torch.cat(list(buf.unbind(0)), dim=head_axis))
        parts = gathered
    res = {"gathered": True, "sequences": len(seqs), "world": world}
    if rank == 0:
        from oracle.paged_attention import paged_attention_oracle  # the checker, outside timing

        q, k, v, o, l = (t.cpu() for t in parts)
        ref, ref_lse = paged_attention_oracle(q, k, v, sub.cu_seqlens_q, sub.seqused_k, sub.block_table,
                                              case.causal, case.window_size)
        err = (o.float() - ref).abs().max().item()
        finite = torch.isfinite(ref_lse)
        lerr = (l[finite] - ref_lse[finite]).abs().max().item()
        lse_inf_match = bool(torch.equal(torch.isfinite(l), finite))
        res.update({"heads": [int(q.shape[1]), int(k.shape[2])], "kv_tokens": int(sub.seqused_k.sum()),
                    "max_abs_out": err, "max_abs_lse": lerr, "tol_out": 2e-2, "tol_lse": 1e-3,
                    "pass": bool(err <= 2e-2 and lerr <= 1e-3 and lse_inf_match),
                    "checker": "oracle.paged_attention.paged_attention_oracle (fp32 on the bf16 inputs)"})
    return res


def call(case, out, lse=None, events=None, num_splits=0):
    from toy_flash_attn import flash_attention_func as faf

    return faf.flash_attn_varlen_with_block_cu_bf16(
        case.q, case.k_cache, case.v_cache, case.max_seqlen_q, case.cu_seqlens_q, case.max_seqlen_k,
        case.seqused_k, case.causal, case.window_size, case.block_table, out, softmax_lse=lse,
        num_splits=num_splits, main_events=events)


def plan_of(case):
    from toy_flash_attn import flash_attention_func as faf

    return faf.plan(case.q, case.k_cache, case.v_cache, case.cu_seqlens_q, case.seqused_k, case.block_table,
                    case.max_seqlen_q, case.max_seqlen_k, case.causal, case.window_size)


# --------------------------------------------------------------------------------------
# CPU baseline: the reference's algorithm (oracle port) on a bounded sample
# --------------------------------------------------------------------------------------
def cpu_sample(case, target_bytes: int | None, max_seqs: int):
    """Compacted CPU copy of the first sequences of `case` (only their live blocks)."""
    from toy_flash_attn.workloads import PagedCase, kv_bytes

    used = case.seqused_k.tolist()
    bs = case.k_cache.shape[1]
    hkv, d = case.k_cache.shape[2], case.k_cache.shape[3]
    n, acc = 0, 0
    while n < min(len(used), max_seqs):
        acc += used[n] * hkv * d * 4
        n += 1
        if target_bytes is not None and acc >= target_bytes:
            break
    need = [(used[b] + bs - 1) // bs for b in range(n)]
    rows = [case.block_table[b, :need[b]].long() for b in range(n)]
    ids = torch.cat(rows)
    k = case.k_cache[ids].cpu()
    v = case.v_cache[ids].cpu()
    table = torch.full((n, max(need)), -1, dtype=torch.int32)
    o = 0
    for b in range(n):
        table[b, :need[b]] = torch.arange(o, o + need[b], dtype=torch.int32)
        o += need[b]
    cu = case.cu_seqlens_q[: n + 1].cpu()
    q = case.q[: int(cu[-1])].cpu()
    sub = PagedCase(case.name + f"[:{n}]", q, k, v, cu, case.seqused_k[:n].cpu(), table, case.max_seqlen_q,
                    max(used[:n]), case.causal, case.window_size)
    return sub, kv_bytes(sub)


def time_reference_port(sub, reps: int = 1) -> float:
    from oracle.paged_attention import reference_port

    t0 = time.perf_counter()
    for _ in range(reps):
        reference_port(sub.q, sub.k_cache, sub.v_cache, sub.max_seqlen_q, sub.cu_seqlens_q, sub.max_seqlen_k,
                       sub.seqused_k, sub.causal, sub.window_size, sub.block_table)
    return (time.perf_counter() - t0) / reps


def cpu_baseline(case, seconds: float) -> dict:
    torch.set_num_threads(os.cpu_count() or 1)
    probe, probe_bytes = cpu_sample(case, None, 2)
    time_reference_port(probe)  # warm-up
    t = time_reference_port(probe)
    rate = probe_bytes / max(t, 1e-9)
    sub, sub_bytes = cpu_sample(case, int(rate * seconds), 64)
    t = time_reference_port(sub)
    return {
        "value": sub_bytes / t / 1e12,
        "unit": UNIT,
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": f"first {sub.batch} of {case.batch} sequences ({sub_bytes / 1e9:.2f} GB of K/V, "
                  f"{t:.1f} s), bf16 math as TOY_FLASH_ATTN_USE=reference",
        "seconds": t,
    }


# --------------------------------------------------------------------------------------
# side table: C1-C4 on one GPU, per call from a CUDA graph, L2 flushed between calls
# --------------------------------------------------------------------------------------
def time_graph_cold(case, iters: int = 20) -> float:
    out = torch.empty_like(case.q)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            call(case, out)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        call(case, out)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")
    times = []
    for i in range(iters + 3):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        if i >= 3:
            times.append(e0.elapsed_time(e1))
    return statistics.median(times) * 1e3  # us


def time_graph_marginal(case, n: int = 20, reps: int = 7) -> float:
    """Per-call time inside a stream of calls: graph replays of [L2 flush, call] x n minus
    replays of [L2 flush] x n, divided by n (us). Every call still starts with a cold L2,
    but the cost of recording events around one isolated replay (about 4 us on B200, an
    empty graph measures 6 us that way) is not counted."""
    out = torch.empty_like(case.q)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")

    def graph_of(body):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            body()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            body()
        return g

    def with_calls():
        for _ in range(n):
            flush.zero_()
            call(case, out)

    def flush_only():
        for _ in range(n):
            flush.zero_()

    g1, g0 = graph_of(with_calls), graph_of(flush_only)

    def t(g):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3

    d = []
    for _ in range(reps):
        d.append(t(g1) - t(g0))
    return max(statistics.median(d[1:]) / n, 0.0)


def time_graph_loop(case, seconds: float = 0.6) -> float:
    """Per-call time of back-to-back graph replays for about `seconds` (no L2 flush): the
    sustained rate of a long compute-bound call, with the clocks the power cap allows."""
    out = torch.empty_like(case.q)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            call(case, out)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        call(case, out)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    n = max(10, int(seconds / max(e0.elapsed_time(e1) * 1e-3, 1e-6)))
    e0.record()
    for _ in range(n):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n * 1e3  # us


def op_cases(warmup: int = 10, iters: int = 30) -> dict:
    """The reference's op metric on its own ten op cases: host wall-clock per call of
    flash_attn_varlen_with_block_cu_bf16 (out allocated by the call, as there), timed with
    perf_counter around the call and a synchronize (bench_attention_op.py:198-210), 10
    warm-up and 30 timed calls; mean and median in ms. The reference's published numbers
    for these cases are RTX 2050 timings of its v8 op (context only)."""
    from toy_flash_attn import flash_attention_func as faf
    from toy_flash_attn.workloads import REFERENCE_OP_CASES, reference_op_case

    res = {}
    for name in REFERENCE_OP_CASES:
        c = reference_op_case(name).to("cuda")

        def run():
            return faf.flash_attn_varlen_with_block_cu_bf16(
                q=c.q, k=c.k_cache, v=c.v_cache, max_seqlen_q=c.max_seqlen_q, cu_seqlens_q=c.cu_seqlens_q,
                max_seqlen_k=c.max_seqlen_k, seqused_k=c.seqused_k, causal=c.causal, window_size=c.window_size,
                block_table=c.block_table)

        for _ in range(warmup):
            run()
        torch.cuda.synchronize()
        ts = []
        for _ in range(iters):
            t0 = time.perf_counter()
            run()
            torch.cuda.synchronize()
            ts.append((time.perf_counter() - t0) * 1e3)
        res[name] = {"ms_mean": round(statistics.mean(ts), 4), "ms_median": round(statistics.median(ts), 4)}
    return res


def side_configs(pk: dict) -> dict:
    from toy_flash_attn.workloads import baseline_config, kv_bytes, prefill_flops

    res = {}
    for name in ("C1", "C2", "C3", "C4", "P1", "P2"):
        case = baseline_config(name, device="cuda")
        us_iso = time_graph_cold(case)
        us = time_graph_marginal(case) if not name.startswith("P") else us_iso
        p = plan_of(case)
        entry = {"us_per_call": round(us, 2), "us_per_call_isolated": round(us_iso, 2),
                 "kernel": ("decode pages" if p.get("pages") else "decode") if p["kernel"] == 0 else "prefill",
                 "splits": p["max_splits"], "tokens_per_s": round(case.q.shape[0] / (us * 1e-6), 1),
                 "timing": ("marginal cost per call in a stream of calls, each after an L2 flush (graph of "
                            "[flush, call] x 20 minus graph of [flush] x 20); us_per_call_isolated = CUDA events "
                            "around one graph replay after a flush") if not name.startswith("P")
                 else "CUDA events around one graph replay after an L2 flush"}
        if p["kernel"] == 0:
            gbs = kv_bytes(case) / (us * 1e-6) / 1e9
            entry.update({"kv_GBps": round(gbs, 1), "hbm_frac": round(gbs / pk["hbm_gbs"], 4)})
        else:
            tf = prefill_flops(case) / (us * 1e-6) / 1e12
            entry.update({"TFLOPs": round(tf, 2), "tensor_frac": round(tf / pk["bf16_tflops"], 4)})
        if name.startswith("P"):
            entry["scaled"] = "not a BASELINE configuration: long-prompt prefill to show tensor-pipe use"
            with ClockSampler(torch.cuda.current_device()) as clk:
                us_loop = time_graph_loop(case)
            tf_loop = prefill_flops(case) / (us_loop * 1e-6) / 1e12
            entry["sustained"] = {"us_per_call": round(us_loop, 2), "TFLOPs": round(tf_loop, 2),
                                  "frac_of_sustained_peak": round(tf_loop / pk["bf16_tflops_sustained"], 4),
                                  "clocks": clk.summary(),
                                  "note": "back-to-back calls for ~0.6 s, no L2 flush"}
        res[name] = entry
        del case
        torch.cuda.empty_cache()
    return res


# --------------------------------------------------------------------------------------
# main arms
# --------------------------------------------------------------------------------------
def run_reference(args):
    """Reference arm: the reference's CPU algorithm (oracle port) on the host cores, rank 0
    only, each step a bounded sample (the first sequences) of C5."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    case = _c5_cpu_case(64)
    per_step = max(0.5, args.cpu_seconds / max(1, args.steps + args.warmup))
    probe, probe_bytes = cpu_sample(case, None, 1)
    time_reference_port(probe)
    rate = probe_bytes / max(time_reference_port(probe), 1e-9)
    sub, sub_bytes = cpu_sample(case, int(rate * per_step), 64)
    for _ in range(args.warmup):
        time_reference_port(sub)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        time_reference_port(sub)
    dt = (time.perf_counter() - t0) / args.steps
    value = sub_bytes / dt / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": _config_desc(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"first {sub.batch} of 256 C5 sequences per step ({sub_bytes / 1e9:.3f} GB K/V), "
                                   "bf16 math as TOY_FLASH_ATTN_USE=reference"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _c5_cpu_case(n_seqs: int):
    """The first `n_seqs` sequences of C5 (same kv lengths as the GPU workload) with a CPU
    pool holding just their blocks; pool size does not change the reference's work."""
    from toy_flash_attn.workloads import PagedCase, c5_kv_lengths

    kv = c5_kv_lengths()[:n_seqs]
    bs = 16
    need = [(n + bs - 1) // bs for n in kv]
    g = torch.Generator().manual_seed(1005)
    q = torch.randn(n_seqs, 32, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(sum(need), bs, 8, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(sum(need), bs, 8, 128, generator=g).to(torch.bfloat16)
    perm = torch.randperm(sum(need), generator=g).to(torch.int32)
    table = torch.full((n_seqs, max(need)), -1, dtype=torch.int32)
    o = 0
    for b, n in enumerate(need):
        table[b, :n] = perm[o:o + n]
        o += n
    return PagedCase("C5-cpu", q, k, v, torch.arange(n_seqs + 1, dtype=torch.int32),
                     torch.tensor(kv, dtype=torch.int32), table, 1, max(kv), True, None)


def _config_desc(world: int) -> dict:
    return {
        "workload": "C5 large-batch decode",
        "batch": 256, "q_heads": 32, "kv_heads": 8, "head_dim": 128, "block_size": 16,
        "kv_lengths": "log-uniform [1024, 32768], seed 5", "pool_blocks_per_gpu": 1 << 21,
        "parallelism": f"kv-head shards x{world} (8/{world} kv heads per GPU), no collective in the timed region",
        "l2": "inputs larger than L2 (~9.6 GB K/V per step); no flush needed",
    }


def run_ours(args):
    world, rank, local = dist_setup(args.gpus)
    from toy_flash_attn import flash_attention_func as faf
    from toy_flash_attn.workloads import kv_bytes

    pk = peaks()
    case = c5_shard(world, rank, args)
    torch.cuda.synchronize()
    kvb_local = kv_bytes(case)
    kvb_total = kvb_local * world
    out = torch.empty_like(case.q)
    p = plan_of(case)
    # the attention kernel, the combine kernel where the plan uses it (combine == 1) and the
    # item-list kernel where the plan builds one
    launches_per_step = 1 + int(p["combine"] == 1) + int(p["item_list"])

    for _ in range(max(args.warmup, 3)):
        call(case, out)
    torch.cuda.synchronize()
    assert faf.read_device_error() == 0

    # the headline: K plain calls, events only around the whole loop (an event between the
    # attention kernel and the combine would stop their programmatic-dependent overlap)
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t_start.record()
        for i in range(args.steps):
            call(case, out)
        t_end.record()
        torch.cuda.synchronize()
    barrier(world)
    ms_local = t_start.elapsed_time(t_end) / args.steps
    ms = allreduce_max(ms_local, world)
    # the roofline: the attention kernel alone, CUDA events on its stream around it
    # (tfa_fwd_timed), over another K calls
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    for i in range(args.steps):
        call(case, out, events=evs[i])
    torch.cuda.synchronize()
    main_ms_local = statistics.mean(a.elapsed_time(b) for a, b in evs)
    main_ms = allreduce_max(main_ms_local, world)
    assert faf.read_device_error() == 0

    # sustained: about one second of back-to-back calls with its own clock record
    n_sus = max(10, int(1.0 / max(ms * 1e-3, 1e-6)))
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk_sus:
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(n_sus):
            call(case, out)
        s1.record()
        torch.cuda.synchronize()
    sus_ms = allreduce_max(s0.elapsed_time(s1) / n_sus, world)
    assert faf.read_device_error() == 0

    # end to end through the public API with host buffers: every step copies its inputs
    # (q, block table, lengths) from pinned host memory, calls flash_attn_varlen_func and
    # reads its output back into pinned host memory. As in a serving loop, the inputs and
    # outputs are double-buffered and the copies run on their own streams, so the h2d of
    # step i+1 and the d2h of step i-1 overlap the attention of step i; the timed region
    # still holds all of them (the first h2d and the last d2h included).
    host_in = {n: getattr(case, n).cpu().pin_memory() for n in ("q", "block_table", "seqused_k", "cu_seqlens_q")}
    host_out = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True) for _ in range(2)]
    dev_in = [{n: torch.empty_like(getattr(case, n)) for n in host_in} for _ in range(2)]
    dev_out = [out, torch.empty_like(out)]
    h2d = sum(t.numel() * t.element_size() for t in host_in.values())
    d2h = host_out[0].numel() * host_out[0].element_size()
    main = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    out_ready = [torch.cuda.Event() for _ in range(2)]
    out_free = [torch.cuda.Event() for _ in range(2)]

    def e2e_run(n_steps):
        def upload(i):
            j = i % 2
            with torch.cuda.stream(up):
                if i >= 2:
                    up.wait_event(in_free[j])  # the call of step i-2 has read buffer j
                for name, t in host_in.items():
                    dev_in[j][name].copy_(t, non_blocking=True)
                in_ready[j].record(up)

        up.wait_stream(main)
        down.wait_stream(main)
        upload(0)
        for i in range(n_steps):
            j = i % 2
            if i + 1 < n_steps:
                upload(i + 1)
            main.wait_event(in_ready[j])
            if i >= 2:
                main.wait_event(out_free[j])  # the d2h of step i-2 has read output j
            d = dev_in[j]
            faf.flash_attn_varlen_func(d["q"], case.k_cache, case.v_cache, case.max_seqlen_q, d["cu_seqlens_q"],
                                       case.max_seqlen_k, None, d["seqused_k"], case.causal, case.window_size,
                                       d["block_table"], out=dev_out[j])
            in_free[j].record(main)
            out_ready[j].record(main)
            with torch.cuda.stream(down):
                down.wait_event(out_ready[j])
                host_out[j].copy_(dev_out[j], non_blocking=True)
                out_free[j].record(down)
        main.wait_stream(up)
        main.wait_stream(down)

    e2e_run(max(args.warmup, 3))
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    e2e_run(args.steps)
    e1.record()
    torch.cuda.synchronize()
    ref_out = out.cpu()  # every step has the same inputs; the kernels are deterministic
    assert all(torch.equal(h, ref_out) for h in host_out), "e2e output read back differs"
    e2e_ms = allreduce_max(e0.elapsed_time(e1) / args.steps, world)

    # verification, outside timing: the whole output gathered to rank 0 (NCCL) must be
    # finite, and a sample of sequences must match the CPU oracle (verify_c5)
    if world > 1:
        import torch.distributed as dist

        gathered = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device="cuda")
        dist.all_gather_into_tensor(gathered, out.contiguous())
        finite = bool(torch.isfinite(gathered).all())
        del gathered
    else:
        finite = bool(torch.isfinite(out).all())
    verify = verify_c5(case, world, rank)
    verify["finite"] = finite

    if rank == 0:
        value = kvb_total / (ms * 1e-3) / 1e12
        achieved_gbs = kvb_local / (main_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "us_per_call": ms * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded N(0,1) bf16 q/K/V, random non-identity block tables",
            "config": _config_desc(world),
            "kv_bytes_per_step": kvb_total,
            "tokens_per_s": case.q.shape[0] / (ms * 1e-3),
            "roofline": {
                "kernel": ("decode_page_kernel (tfa_decode_pages.cu)" if p.get("pages")
                           else "decode_kernel (tfa_decode.cu)"), "bound": "hbm", "achieved": achieved_gbs,
                "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved_gbs / pk["hbm_gbs"],
                "peak_source": pk["source"], "traffic": kvb_local * TRAFFIC_PER_KV_BYTE[bool(p.get("pages"))],
                "traffic_unit": "bytes per launch (ncu, scaled from reduced C5)",
                "note": "achieved = algorithmic K/V bytes per launch / mean CUDA-event duration of the attention "
                        "kernel alone (tfa_fwd_timed), max over ranks",
            },
            "e2e": {"value": kvb_total / (e2e_ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                    "api": "toy_flash_attn.flash_attention_func.flash_attn_varlen_func",
                    "pipeline": "pinned host buffers; inputs and outputs double-buffered, h2d and d2h on "
                                "their own streams overlapping the neighbouring steps' attention"},
            "sustained": {"calls": n_sus, "ms_per_call": sus_ms, "value": kvb_total / (sus_ms * 1e-3) / 1e12,
                          "unit": UNIT, "clocks": clk_sus.summary(),
                          "note": "back-to-back calls for about one second (max over ranks)"},
            "gpu_launches": launches_per_step * args.steps,
            "plan": p,
            "clocks": clk.summary(),
            "verify": verify,
        }
        if world == 1 and not args.no_configs:
            del case
            torch.cuda.empty_cache()
            line["configs"] = side_configs(pk)
            line["op_cases"] = {"metric": "host wall-clock ms per call (perf_counter + synchronize), the "
                                          "reference's op benchmark method and cases",
                                "cases": op_cases()}
            case = c5_shard(world, rank, args)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(case, args.cpu_seconds)
        print(json.dumps(line), flush=True)
    barrier(world)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.profile_configs:
        run_profile_configs(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
