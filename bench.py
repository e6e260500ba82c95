#!/usr/bin/env python3
"""Benchmark of the B200 attention hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Default (no --workload): one JSON line whose headline is the long-context
paged decode, bf16, GQA 32 q / 8 kv heads x 128: 256 sequences with context
~ U[4096, 32768] (seed 2027), 16-token blocks, sequences sharded across the
ranks by a longest-first greedy split of their lengths (no collective; the
256 sequences are the whole job at every N, "scaling": "strong"). A step is
one decode launch over the rank's sequences. Metric: decode KV-bytes GB/s =
algorithmic bytes / kernel time, algorithmic bytes = sum(ctx) * kv_heads *
head_dim * 2 * element bytes + fp32 queries and outputs + table entries and
context lengths; value = all ranks' bytes / the slowest rank's time. Beside it,
each timed in the same run, are the other halves of the metric:
prefill_f16 (causal prefill 8 x 1024 tokens, 16 heads x 128, f16; TFLOP/s per
rank, one batch per rank), decode_fp32 (64 sequences x U[64, 2048], 8 heads x
64, fp32; one batch per rank), longseq_split (one 131,072-token sequence
split across the ranks by contiguous block ranges, partials all-gathered over
NCCL and merged in rank order), mixed_bf16 (one continuous-batching step per
rank: its decode launch and its chunked-prefill launch) and single_seq_fp32
(the drop-in C entry on the reference's own 129 x 4 x 32 case, microseconds
per prefill + decode call pair). Every object carries its roofline, per-rank
step times and clocks; at N = 1 the CPU baseline legs time the reference's
own kernel (oracle/_ref/libref.so, built from kernels/attention_cpu.cpp) on a
bounded sample of the same data and record how its outputs compare with ours.

--workload NAME prints that workload's line alone: longctx_bf16,
decode_fp32, prefill_f16, longseq_split, mixed_bf16 (one continuous-batching
step: 32 decode sequences with context Zipf(1.1) clipped to [32, 8192] + 4 x
512-token prefill chunks, GQA 32/8 x 128 bf16), single_seq_fp32 (the drop-in
C entry inferlab_attention_forward with host buffers on one 129 x 4 x 32
sequence: prefill of 128 queries plus one decode query), qkv_append_bf16 and
outproj_bf16 (the projections either side of attention on the mixed step's
chunk tokens).

--impl reference times the reference's own CPU kernel on the host cores for
the same workload (rank 0 only; other ranks exit): per sequence the page
gather plus one inferlab_attention_forward call per q-head, as the reference
worker's paged decode does, on a bounded sample of the workload per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2
L2_NOTE = ("flushed between steps: 256 MB write then 256 MB read of a second buffer, outside "
           "the step events")


def load_peaks() -> tuple[dict, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as handle:
            return json.load(handle), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def read_traffic(name: str):
    """DRAM bytes per launch from a committed ncu summary (profiles/<name>.md,
    line 'traffic_bytes_per_launch: N'), or None. The summary records the
    kernel version it was captured on; the bench does not re-measure it."""
    path = os.path.join(ROOT, "profiles", f"{name}.md")
    if not os.path.exists(path):
        return None
    with open(path) as handle:
        for line in handle:
            if line.strip().startswith("traffic_bytes_per_launch:"):
                try:
                    return int(float(line.split(":", 1)[1].strip()))
                except ValueError:
                    return None
    return None


def traffic_fields(name: str) -> dict:
    value = read_traffic(name)
    return {"traffic": value,
            "traffic_source": (f"profiles/{name}.md (ncu dram__bytes_read.sum + "
                               "dram__bytes_write.sum per launch, committed summary; not "
                               "measured in this run)") if value is not None else None}


class L2Flush:
    """Evicts the previous step's data from the 126 MB L2 between timed steps:
    writes one 256 MB buffer, then reads a second 256 MB buffer, so the written
    lines are themselves evicted (written back) before the next step's events
    start and the timed kernel pays for neither hits nor write-backs."""

    def __init__(self, device: int):
        import torch

        self.write = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{device}")
        self.read = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{device}")

    def fill_(self, value: float) -> None:
        self.write.fill_(value)
        self.read.sum()


class ClockSampler:
    """nvidia-smi samples (SM clock, throttle reasons) while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_id = str(device_index)
        try:  # name the GPU by UUID so CUDA_VISIBLE_DEVICES remapping does not matter
            import torch

            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            self.device_id = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            pass
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_id}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.reader.join(timeout=2)
            self.proc = None

    def summary(self) -> dict:
        sms, maxes, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes),
                "power_w_max": max(power) if power else None,
                "reasons": sorted(reasons), "samples": len(sms)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world: int, local: int):
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local}"))
    return dist if world > 1 else None


def barrier(dist):
    if dist is not None:
        dist.barrier()


def max_over_ranks(dist, value: float) -> float:
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(dist, value: float) -> float:
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def per_rank(dist, **values) -> list[dict]:
    """Every rank's named numbers (None allowed), gathered in rank order."""
    keys = sorted(values)
    row = [float("nan") if values[k] is None else float(values[k]) for k in keys]
    if dist is None:
        rows = [row]
    else:
        import torch

        t = torch.tensor(row, dtype=torch.float64, device="cuda")
        parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
        dist.all_gather(parts, t)
        rows = [p.tolist() for p in parts]
    out = []
    for rank, r in enumerate(rows):
        entry = {"rank": rank}
        for k, v in zip(keys, r):
            entry[k] = None if v != v else round(v, 5)
        out.append(entry)
    return out


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as handle:
            for line in handle:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def timed_region(args, dist, device, stream, flush, parts):
    """Untimed pre-roll of about 0.5 s of the step (so the clock samples see
    the GPU under this load), then exactly args.steps steps, each part
    bracketed by its own CUDA events on `stream`, with the L2 flushed before
    every step; a barrier and a device synchronize on both sides. Every rank
    runs the same number of pre-roll steps (sized from the slowest rank's
    first step), since a step may hold collectives or peer exchanges that pair
    up across ranks. Returns each part's total milliseconds on this rank."""
    import torch

    def one_step():
        flush.fill_(0.0)
        for part in parts:
            part()
        stream.synchronize()

    start = time.perf_counter()
    one_step()
    first = max_over_ranks(dist, time.perf_counter() - start)
    for _ in range(max(0, min(int(0.5 / max(first, 1e-6)), 20000) - 1)):
        one_step()
    events = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in parts] for _ in range(args.steps)]
    barrier(dist)
    torch.cuda.synchronize(device)
    # Keep the GPU busy while the host enqueues every timed step, so the step
    # events time the kernels and not the host's launch latency.
    torch.cuda._sleep(int(2e6 + 3e5 * args.steps))
    for i in range(args.steps):
        flush.fill_(float(i))  # evict the previous step's data from L2
        for (start, end), part in zip(events[i], parts):
            start.record(stream)
            part()
            end.record(stream)
    torch.cuda.synchronize(device)
    barrier(dist)
    return [sum(events[i][k][0].elapsed_time(events[i][k][1]) for i in range(args.steps))
            for k in range(len(parts))]


# ---------------------------------------------------------------------------
# decode (long-context headline and fp32 sub-line)
# ---------------------------------------------------------------------------
LONGCTX_SEED = 2027
LONGCTX_SAMPLE = 4  # sequences the CPU baseline leg takes


def build_decode(workload: str, rank: int, world: int, device: int, longctx_seqs: int = 256):
    from inferlab_b200 import distributed
    from inferlab_b200 import workloads as wl

    if workload == "decode_fp32":
        batch = wl.decode_fp32(device=device, seed=2026 + rank)
        desc = {"workload": "paged decode fp32: 64 seqs x ctx U[64,2048], 8 heads x 64 (MHA), "
                            "block 16, 8192-block pool, random permutation tables",
                "num_seqs": 64, "q_heads": 8, "kv_heads": 8, "head_dim": 64,
                "block_tokens": 16, "pool_blocks": 8192, "seed": 2026 + rank,
                "per_rank": "independent batch per rank"}
        return batch, desc, "f32", "weak"
    if workload == "longctx_bf16":
        contexts = wl.longctx_contexts(LONGCTX_SEED)[:longctx_seqs]
        owner = distributed.shard_sequences(contexts, world)
        mine = contexts[owner == rank]
        batch = wl.longctx_bf16(device=device, seed=LONGCTX_SEED + rank, contexts=mine)
        desc = {"workload": f"paged decode bf16: {len(contexts)} seqs x ctx U[4096,32768], "
                            "GQA 32q/8kv x 128, block 16, sequences sharded across GPUs",
                "num_seqs_total": int(len(contexts)), "num_seqs_this_rank": int(len(mine)),
                "q_heads": 32, "kv_heads": 8, "head_dim": 128, "block_tokens": 16,
                "seed": LONGCTX_SEED, "sum_context_total": int(contexts.sum()),
                "sharding": "longest-first greedy over context lengths, no collective"}
        return batch, desc, "bf16", "strong"
    raise SystemExit(f"unknown decode workload {workload}")


def host_sample(pool, tables_host, contexts, seqs):
    """Host copies of the blocks of sequences `seqs` (compacted) and their
    tables renumbered into the copy."""
    import torch

    need = (np.asarray(contexts)[seqs] + 15) // 16
    ids = np.unique(np.concatenate([tables_host[s, :n] for s, n in zip(seqs, need)]))
    index = torch.from_numpy(ids.astype(np.int64)).to(f"cuda:{pool.device}")

    def grab(arena):
        part = arena.index_select(0, index)
        if part.dtype == torch.float32:
            return part.cpu().numpy()
        return part.view(torch.int16).cpu().numpy().view(np.uint16)

    remap = np.zeros(pool.num_blocks, np.int64)
    remap[ids] = np.arange(len(ids))
    width = int(need.max())
    tables = np.zeros((len(seqs), width), np.int32)
    for i, (s, n) in enumerate(zip(seqs, need)):
        tables[i, :n] = remap[tables_host[s, :n]]
    return grab(pool.key_arena), grab(pool.value_arena), tables


def compare(got, ref, rtol, atol=0.0, row_atol=0.0) -> dict:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref)
    row = np.max(np.abs(ref), axis=-1, keepdims=True)
    big = np.abs(ref) > 1e-2
    bound = atol + rtol * np.abs(ref) + row_atol * row
    return {"max_abs": float(err.max()),
            "max_rel_ref_gt_1e-2": float((err[big] / np.abs(ref[big])).max()) if big.any() else 0.0,
            "max_err_over_rowmax": float(np.max(err / np.maximum(row, 1e-30))),
            "within_tolerance": bool(np.all(err <= bound)),
            "elements": int(err.size)}


def cpu_baseline_decode(sample, bytes_per_step_sample, q_heads, dtype, seconds, what):
    """The reference CPU kernel (page gather + one inferlab_attention_forward
    per q-head, OnlineTiled tile 16) on a host sample of the timed workload,
    on all host threads, repeated for about `seconds`; plus one single-thread
    pass over its first sequence, and how its outputs compare with ours."""
    from oracle import oracle

    k_host, v_host, tables, contexts, q, ours = sample
    threads = host_threads()
    steps = 0
    ref = None
    t0 = time.perf_counter()
    while True:
        ref = oracle.reference_paged_decode_timed(k_host, v_host, dtype, tables, contexts, q,
                                                  q_heads, threads)
        steps += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= seconds:
            break
    kind = "reference" if oracle.ref_lib() is not None else "port"
    first = np.array([contexts[0]])
    one_bytes = bytes_per_step_sample * float(contexts[0]) / float(np.sum(contexts))
    t1 = time.perf_counter()
    oracle.reference_paged_decode_timed(k_host, v_host, dtype, tables[:1], first, q[:1], q_heads, 1)
    single = one_bytes / (time.perf_counter() - t1) / 1e9
    parity = compare(ours, ref, rtol=1e-5, atol=1e-6)
    parity["tolerance"] = "|ours - reference| <= 1e-6 + 1e-5 |reference| (fp32 arithmetic)"
    return {"value": round(bytes_per_step_sample * steps / elapsed / 1e9, 4), "unit": "GB/s",
            "cores": threads, "kind": kind, "cpu_model": cpu_model(),
            "single_thread_value": round(single, 4),
            "sample": f"{what}: {steps} passes in {elapsed:.1f} s; page gather + "
                      "inferlab_attention_forward (OnlineTiled, tile 16) per q-head from "
                      "oracle/_ref/libref.so, sequences (or (sequence, q-head) calls) spread "
                      "over the host threads",
            "parity_sample": parity}


def measure_decode(args, dist, world, rank, device, peaks, peak_kind, workload):
    import torch

    batch, desc, dtype_name, scaling = build_decode(workload, rank, world, device,
                                                    args.longctx_seqs)
    pool = batch.pool
    stream = torch.cuda.current_stream(device)
    num_seqs = len(batch.contexts)
    workspace = pool.make_workspace(num_seqs, batch.q_heads, batch.max_context_len)
    out = torch.empty_like(batch.queries)
    flush = L2Flush(device)
    bytes_per_step = batch.decode_bytes()

    def step():
        pool.decode(batch.queries, batch.block_tables, batch.context_lens,
                    batch.max_context_len, out=out, workspace=workspace)

    for i in range(args.warmup):
        flush.fill_(float(i))
        step()
    pool.synchronize()
    clocks = ClockSampler(device).__enter__()
    (kernel_ms,) = timed_region(args, dist, device, stream, flush, [step])
    pool.synchronize()
    total_ms = max_over_ranks(dist, kernel_ms)
    all_bytes = sum_over_ranks(dist, float(bytes_per_step) * args.steps)
    value = all_bytes / (total_ms * 1e-3) / 1e9
    achieved = bytes_per_step / (kernel_ms / args.steps * 1e-3) / 1e9
    peak = float(peaks["hbm_gbs"])

    # CPU baseline sample (rank 0, one GPU): copied before the end-to-end steps
    # append new rows to the pool.
    sample = None
    want_cpu = rank == 0 and world == 1 and not args.no_cpu_baseline
    if want_cpu:
        from inferlab_b200 import workloads as wl

        seqs = (list(range(num_seqs)) if workload == "decode_fp32"
                else list(range(min(LONGCTX_SAMPLE, num_seqs))))
        k_host, v_host, tables = host_sample(pool, batch.tables_host, batch.contexts, seqs)
        q = wl.round_queries(batch.queries, pool.dtype)[seqs]
        sample = (k_host, v_host, tables, batch.contexts[seqs], q, out.cpu().numpy()[seqs])
        ctx = batch.contexts[seqs].astype(np.int64)
        sample_bytes = (int(ctx.sum()) * batch.kv_heads * batch.head_dim * 2 * pool.element_bytes
                        + 2 * len(seqs) * batch.q_heads * batch.head_dim * 4
                        + int(((ctx + 15) // 16).sum()) * 4 + len(seqs) * 4)

    e2e = run_decode_e2e(args, batch, pool, flush, device, dist, bytes_per_step)
    clocks.__exit__(None, None, None)
    clock = clocks.summary()
    clock["window"] = "0.5 s pre-roll of the same step + timed steps + e2e steps"
    ranks = per_rank(dist, ms_per_step=kernel_ms / args.steps, sm_mhz=clock["sm_mhz"],
                     e2e_ms_per_step=e2e["rank_ms_per_step"], gbs=achieved)
    e2e.pop("rank_ms_per_step")
    profile = f"paged_decode_{workload}"
    line = {
        "metric": "decode attn KV-bytes GB/s",
        "value": round(value, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 5),
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": dtype_name,
        "data": "synthetic (seeded N(0,1) Q/K/V, seeded contexts and block tables)",
        "config": dict(desc, l2=L2_NOTE, parallelism=f"sequence-sharded x{world}, no collective"),
        "roofline": dict({"bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                          "unit": "GB/s", "frac": round(achieved / peak, 4),
                          "peak_kind": f"{peak_kind} hbm_gbs",
                          "algorithmic_bytes_per_launch": int(bytes_per_step),
                          "rank": rank}, **traffic_fields(profile)),
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clock,
        "per_rank": ranks,
    }
    pool.close()
    del workspace, out, flush
    torch.cuda.empty_cache()
    if sample is not None:
        what = ("the whole 64-sequence batch" if workload == "decode_fp32" else
                f"{len(sample[3])} of the 256 sequences (contexts "
                + ", ".join(str(int(c)) for c in sample[3]) + ")")
        line["cpu_baseline"] = cpu_baseline_decode(sample, sample_bytes, batch.q_heads,
                                                   batch.pool.dtype, args.cpu_seconds, what)
    return line


def run_decode_e2e(args, batch, pool, flush, device, dist, bytes_per_step):
    """The same decode step through the C ABI with HOST buffers: one
    inferlab_cuda_decode_step_host call per step takes the step's queries,
    the new token's K/V rows, the block tables and context lengths from host
    memory (page-locked and mapped, so a prologue kernel reads them over the
    bus), appends the new rows at position ctx - 1, decodes every sequence and
    writes the output into the host array (synchronous). Host wall clock around
    each call."""
    import torch

    num_seqs, q_heads, head_dim = batch.queries.shape
    kvh = batch.kv_heads
    gen = np.random.Generator(np.random.PCG64(99))

    def pinned(a):
        # page-locked host memory, as a serving loop keeps its step buffers
        t = torch.empty(a.shape, dtype=getattr(torch, str(a.dtype)), pin_memory=True)
        t.numpy()[...] = a
        return t.numpy()

    h_q = pinned(gen.standard_normal((num_seqs, q_heads, head_dim), dtype=np.float32))
    h_k = pinned(gen.standard_normal((num_seqs, kvh, head_dim), dtype=np.float32))
    h_v = pinned(gen.standard_normal((num_seqs, kvh, head_dim), dtype=np.float32))
    h_tables = pinned(np.ascontiguousarray(batch.tables_host, dtype=np.int32))
    h_lens = pinned(batch.contexts.astype(np.int32))
    h_out = pinned(np.zeros((num_seqs, q_heads, head_dim), dtype=np.float32))
    # payload crossing the bus each step: inputs (+ positions and sequence ids
    # derived on the host) down, output + error word up
    h2d = (h_q.nbytes + h_k.nbytes + h_v.nbytes + h_tables.nbytes + 3 * h_lens.nbytes)
    d2h = h_out.nbytes + 4
    stream = torch.cuda.current_stream(device)

    def step():
        pool.decode_step_host(h_q, h_tables, h_lens, h_k, h_v, out=h_out, stream=stream)

    for i in range(args.warmup):
        flush.fill_(float(i))
        step()
    pool.synchronize()
    total = 0.0
    barrier(dist)
    for i in range(args.steps):
        flush.fill_(float(i))
        stream.synchronize()
        t0 = time.perf_counter()
        step()
        total += time.perf_counter() - t0
    pool.synchronize()
    barrier(dist)
    mine = total
    total = max_over_ranks(dist, total)
    all_bytes = sum_over_ranks(dist, float(bytes_per_step) * args.steps)
    return {"value": round(all_bytes / total / 1e9, 3), "unit": "GB/s",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "ms_per_step": round(total / args.steps * 1e3, 5),
            "rank_ms_per_step": mine / args.steps * 1e3,
            "gpu_launches_per_step": 2,
            "path": "inferlab_cuda_decode_step_host with page-locked host arrays: a prologue "
                    "kernel reads them over the bus (appends the new K/V rows, stages q, "
                    "tables and lengths in HBM), the paged decode writes the output straight "
                    "into the host array, a 4-byte copy returns the error word; host wall "
                    "clock per call, max over ranks"}


# ---------------------------------------------------------------------------
# prefill
# ---------------------------------------------------------------------------
def cpu_baseline_prefill(pool, batch, ours, seconds):
    """The reference's causal prefill on the host on segment 0 of the timed
    batch (1024 tokens, all 16 heads): inferlab_attention_forward (OnlineTiled,
    tile 16, Fp16 storage mode, causal) from oracle/_ref/libref.so, one call
    per head (heads = 1 on that head's slice of the pool's f16 K/V and the
    f16 queries), the heads spread over the host threads; repeated for about
    `seconds`. Also how the reference's outputs compare with ours."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle

    tokens = int(batch.counts[0])
    heads, dim = batch.q_heads, batch.head_dim
    k_host, v_host, tables = host_sample(pool, batch.prefill_tables_host,
                                         batch.starts + batch.counts, [0])
    nblk = (tokens + 15) // 16
    ids = tables[0, :nblk]

    def widen(bits):  # [nblk][kvh][16][dim] f16 bits -> [kvh][tokens][dim] fp32
        x = bits[ids].view(np.float16).astype(np.float32)
        return x.transpose(1, 0, 2, 3).reshape(x.shape[1], nblk * 16, dim)[:, :tokens]

    kk, vv = widen(k_host), widen(v_host)
    q = batch.prefill_queries[:tokens].float().cpu().numpy()  # [tokens][heads][dim]
    group = heads // kk.shape[0]
    per_head = [(np.ascontiguousarray(q[:, h]), np.ascontiguousarray(kk[h // group]),
                 np.ascontiguousarray(vv[h // group])) for h in range(heads)]
    ref = np.zeros((tokens, heads, dim), np.float32)

    def head(h):
        qh, kh, vh = per_head[h]
        o, _ = oracle.attention_forward(qh, kh, vh, tokens, tokens, 1, dim, 0,
                                        oracle.ONLINE_TILED, oracle.FP16, 16, True,
                                        impl="reference")
        ref[:, h] = o.reshape(tokens, dim)

    threads = host_threads()
    flops = 4 * dim * heads * tokens * (tokens + 1) // 2
    passes = 0
    with ThreadPoolExecutor(max_workers=threads) as ex:
        t0 = time.perf_counter()
        while True:
            list(ex.map(head, range(heads)))
            passes += 1
            elapsed = time.perf_counter() - t0
            if elapsed >= seconds:
                break
    parity = compare(ours[:tokens], ref, rtol=2e-3, row_atol=1e-3)
    parity["tolerance"] = ("|ours - reference| <= 2e-3 |reference| + 1e-3 max|reference row| "
                           "(fp16 probabilities on the tensor cores); reference in its Fp16 "
                           "storage mode")
    return {"value": round(flops * passes / elapsed / 1e12, 6), "unit": "TFLOP/s",
            "cores": threads, "kind": "reference", "cpu_model": cpu_model(),
            "sample": f"segment 0 of the batch (1024 tokens, 16 heads): {passes} passes in "
                      f"{elapsed:.1f} s, one inferlab_attention_forward call per head "
                      "(OnlineTiled, tile 16, Fp16 mode) from oracle/_ref/libref.so",
            "parity_sample": parity}


def measure_prefill(args, dist, world, rank, device, peaks, peak_kind):
    import torch

    from inferlab_b200 import workloads as wl

    batch = wl.prefill_f16(device=device, seed=2028 + rank)
    pool = batch.pool
    stream = torch.cuda.current_stream(device)
    flops = batch.prefill_flops()
    out = torch.empty((batch.prefill_queries.shape[0], batch.q_heads, batch.head_dim),
                      dtype=torch.float32, device=f"cuda:{device}")
    flush = L2Flush(device)

    def step():
        pool.prefill(batch.prefill_queries, batch.prefill_tables, batch.starts_dev,
                     batch.counts_dev, batch.offsets_dev, int(batch.counts.max()), out=out)

    for i in range(args.warmup):
        flush.fill_(float(i))
        step()
    pool.synchronize()
    with ClockSampler(device) as clocks:
        (kernel_ms,) = timed_region(args, dist, device, stream, flush, [step])
    pool.synchronize()
    total_ms = max_over_ranks(dist, kernel_ms)
    all_flops = sum_over_ranks(dist, float(flops) * args.steps)
    value = all_flops / (total_ms * 1e-3) / 1e12
    achieved = flops / (kernel_ms / args.steps * 1e-3) / 1e12
    peak = float(peaks["bf16_tflops"])
    clock = clocks.summary()
    line = {
        "metric": "prefill attn TFLOP/s", "value": round(value, 3), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0, 0.5^2))",
        "config": {"workload": "causal prefill f16: 8 x 1024 tokens, 16 heads x 128, paged "
                               "block 16 (one batch per rank)", "flops_per_step": int(flops),
                   "flops_counted": "4 * head_dim * score elements (the reference's causal "
                                    "count, kernels/attention_cpu.cpp:149-168)",
                   "l2": L2_NOTE},
        "roofline": dict({"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                          "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                          "peak_kind": f"{peak_kind} bf16_tflops (burst; dense f16 = bf16 rate)",
                          "frac_of_sustained": round(achieved / float(
                              peaks.get("bf16_tflops_sustained", peak)), 4),
                          "rank": rank}, **traffic_fields("paged_prefill_prefill_f16")),
        "gpu_launches": args.steps, "clocks": clock,
        "per_rank": per_rank(dist, ms_per_step=kernel_ms / args.steps, sm_mhz=clock["sm_mhz"],
                             tflops=achieved),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_prefill(pool, batch, out.cpu().numpy(),
                                                    min(args.cpu_seconds, 8.0))
    pool.close()
    return line


# ---------------------------------------------------------------------------
# one long sequence split across the ranks
# ---------------------------------------------------------------------------
def measure_long_sequence(args, dist, world, rank, device, peaks, peak_kind):
    """One 131072-token sequence split across the ranks: per step (at N > 1)
    ONE kernel decodes the local blocks, and the CTA that finishes each
    kv-head stores its rows' (m, l, o) into every peer's receive buffer over
    NVLink, waits for those rows from all ranks and merges them in rank order
    (distributed.PeerExchange.decode). The NCCL all-gather + merge of the same
    partials is timed beside it. Timed per rank with events, max over ranks."""
    import torch

    from inferlab_b200 import distributed, workloads as wl

    batch = wl.long_sequence_shard(device, rank, world)
    pool = batch.pool
    stream = torch.cuda.current_stream(device)
    flush = L2Flush(device)
    local = int(batch.contexts[0])
    workspace = pool.make_workspace(1, 32, local)

    exchange, exchange_error = None, None
    if world > 1:
        try:
            exchange = distributed.PeerExchange(32, 128)
        except (RuntimeError, ValueError) as caught:  # every rank takes this branch together
            exchange_error = str(caught)

    def step():
        return distributed.decode_split_sequence(pool, batch.queries, batch.block_tables, local,
                                                 workspace=workspace, exchange=exchange)

    def step_nccl():
        return distributed.decode_split_sequence(pool, batch.queries, batch.block_tables, local,
                                                 workspace=workspace)

    for i in range(args.warmup):
        flush.fill_(float(i))
        step()
        if exchange is not None:
            step_nccl()
    pool.synchronize()
    with ClockSampler(device) as clocks:
        (ms,) = timed_region(args, dist, device, stream, flush, [step])
    pool.synchronize()
    nccl = None
    if exchange is not None:
        exchange.synchronize(timeout_ms=20000)  # raises if a peer's block never arrived
        (nccl_ms,) = timed_region(args, dist, device, stream, flush, [step_nccl])
        pool.synchronize()
        nccl_total = max_over_ranks(dist, nccl_ms)
        nccl = {"ms_per_step": round(nccl_total / args.steps, 5),
                "value": round(131072 * 8 * 128 * 2 * 2 * args.steps / (nccl_total * 1e-3) / 1e9, 3),
                "unit": "GB/s",
                "path": "the same partials exchanged by all_gather_into_tensor over NCCL, "
                        "then inferlab_cuda_lse_combine_packed"}
        exchange.close()
    total_ms = max_over_ranks(dist, ms)
    kv_bytes = 131072 * 8 * 128 * 2 * 2
    value = kv_bytes * args.steps / (total_ms * 1e-3) / 1e9
    clock = clocks.summary()
    comm = None
    if dist is not None:
        comm = dist.get_world_size()
    line = {
        "metric": "long-sequence decode KV-bytes GB/s", "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 5), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": {"workload": "one 131072-token sequence, GQA 32/8 x 128 bf16, blocks split "
                               "across GPUs, (m, l, o) partials exchanged and merged in rank order"
                               + (", decode and exchange in one kernel over NVLink peer memory"
                                  if exchange is not None else ""),
                   "tokens_this_rank": local, "comm_nranks": comm,
                   "collective": ("peer stores over NVLink inside the decode kernel "
                                  "(inferlab_cuda_paged_decode_exchange): each kv-head's rows "
                                  "of (m, l, o) from every rank to every peer as step-tagged "
                                  "8-byte words"
                                  if exchange is not None else
                                  f"all_gather_into_tensor over NCCL ({exchange_error})"
                                  if comm and comm > 1 else "none (one GPU)"),
                   "l2": L2_NOTE},
        "roofline": {"bound": "hbm", "achieved_per_gpu": round(value / world, 2),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(value / world / peaks["hbm_gbs"], 4),
                     "peak_kind": f"{peak_kind} hbm_gbs"},
        "gpu_launches": (1 if exchange is not None else 2) * args.steps, "clocks": clock,
        "per_rank": per_rank(dist, ms_per_step=ms / args.steps, sm_mhz=clock["sm_mhz"]),
    }
    if nccl is not None:
        line["nccl_all_gather"] = nccl
    pool.close()
    return line


# ---------------------------------------------------------------------------
# default line and dispatch
# ---------------------------------------------------------------------------
def run_default(args, dist, world, rank, device, peaks, peak_kind):
    """The headline long-context decode plus the other halves of the metric,
    each measured in this run (the same collective steps on every rank)."""
    line = measure_decode(args, dist, world, rank, device, peaks, peak_kind, "longctx_bf16")
    line["prefill_f16"] = measure_prefill(args, dist, world, rank, device, peaks, peak_kind)
    line["decode_fp32"] = measure_decode(args, dist, world, rank, device, peaks, peak_kind,
                                         "decode_fp32")
    line["longseq_split"] = measure_long_sequence(args, dist, world, rank, device, peaks,
                                                  peak_kind)
    line["mixed_bf16"] = run_mixed(args, dist, world, rank, device, peaks, peak_kind)
    line["single_seq_fp32"] = run_single_sequence(args, dist, world, rank, device)
    return line


def run_ours(args):
    import torch

    from inferlab_b200 import _lib

    world, rank, local = dist_env()
    dist = init_dist(world, local)
    device = local
    peaks, peak_kind = load_peaks()
    _lib.lib()  # fails loudly if the CUDA library is missing
    try:
        if args.workload == "default":
            line = run_default(args, dist, world, rank, device, peaks, peak_kind)
        elif args.workload in ("longctx_bf16", "decode_fp32"):
            line = measure_decode(args, dist, world, rank, device, peaks, peak_kind,
                                  args.workload)
        elif args.workload == "prefill_f16":
            line = measure_prefill(args, dist, world, rank, device, peaks, peak_kind)
        elif args.workload == "longseq_split":
            line = measure_long_sequence(args, dist, world, rank, device, peaks, peak_kind)
        elif args.workload == "mixed_bf16":
            line = run_mixed(args, dist, world, rank, device, peaks, peak_kind)
        elif args.workload in ("qkv_append_bf16", "outproj_bf16"):
            line = run_projection(args, dist, world, rank, device, peaks, peak_kind)
        elif args.workload == "single_seq_fp32":
            line = run_single_sequence(args, dist, world, rank, device)
        else:
            raise SystemExit(f"unknown workload {args.workload}")
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            torch.cuda.synchronize(device)
            dist.destroy_process_group()


def run_single_sequence(args, dist, world, rank, device):
    """The reference's own CPU-runnable case through the drop-in C entry:
    Q/K/V ~ N(0, 1) [129][4][32] fp32; prefill of the first 128 queries
    (start 0, causal, OnlineTiled tile 16) and decode of query 128 against all
    129 keys (start 128). A step is both calls, host buffers in and out (each
    call copies its inputs to the device, runs one kernel and copies the
    output back). Timed on the host clock around each call pair; the reference
    CPU kernel (oracle/_ref/libref.so) runs the same calls for cpu_baseline."""
    import inferlab_b200 as il
    from oracle import oracle

    rng = np.random.Generator(np.random.PCG64(20261201))
    t, h, d = 129, 4, 32
    q = rng.standard_normal(t * h * d, dtype=np.float32)
    k = rng.standard_normal(t * h * d, dtype=np.float32)
    v = rng.standard_normal(t * h * d, dtype=np.float32)
    cfg = il.AttentionConfig(il.AttentionAlgorithm.ONLINE_TILED)
    width = h * d

    def ours():
        il.run_attention(q[:128 * width], k[:128 * width], v[:128 * width], 128, 128, h, d, 0, cfg)
        il.run_attention(q[128 * width:], k, v, 1, 129, h, d, 128, cfg)

    def reference():
        oracle.attention_forward(q[:128 * width], k[:128 * width], v[:128 * width], 128, 128, h,
                                 d, 0, oracle.ONLINE_TILED, oracle.FP32, 16, impl="reference")
        oracle.attention_forward(q[128 * width:], k, v, 1, 129, h, d, 128, oracle.ONLINE_TILED,
                                 oracle.FP32, 16, impl="reference")

    for _ in range(args.warmup):
        ours()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ours()
        times.append(time.perf_counter() - t0)
    us = statistics.median(times) * 1e6
    line = {
        "metric": "drop-in attention_forward us per call pair", "value": round(us, 2),
        "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(us / 1e3, 4), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": "single sequence 129 x 4 heads x 32, fp32: prefill 128 + decode 1 "
                               "through inferlab_attention_forward (host buffers)",
                   "timing": "host clock, median of steps; launch-bound, no roofline claim"},
        "gpu_launches": 2 * args.steps,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline and oracle.ref_lib() is not None:
        for _ in range(3):
            reference()
        ref_times = []
        for _ in range(max(args.steps, 20)):
            t0 = time.perf_counter()
            reference()
            ref_times.append(time.perf_counter() - t0)
        line["cpu_baseline"] = {"value": round(statistics.median(ref_times) * 1e6, 2), "unit": "us",
                                "cores": 1, "kind": "reference", "cpu_model": cpu_model(),
                                "sample": "the same two calls on oracle/_ref/libref.so "
                                          "(kernels/attention_cpu.cpp), one thread"}
    return line



def cpu_projection_baseline(batch, seconds: float):
    """The reference's own fp32 linear (oracle/_ref/libref_linear.so, built
    from worker/cpp/inferlab_runtime.cpp:1266-1285; one thread, as the
    reference runs it) over a bounded sample of the step's tokens; falls back
    to the oracle's restatement of the same loop."""
    from oracle import projection

    w = batch.weights.float().cpu().numpy()
    rows = 8
    x = batch.hidden[:rows].float().cpu().numpy()
    kind, fn = "reference", projection.ref_linear
    if projection.ref_linear(x[:1], w[:64]) is None:
        kind, fn = "port", projection.linear
    done, t0 = 0, time.perf_counter()
    while True:
        fn(x, w)
        done += 1
        if time.perf_counter() - t0 >= seconds:
            break
    elapsed = time.perf_counter() - t0
    flops = 2.0 * rows * w.shape[0] * w.shape[1] * done
    return {"value": round(flops / elapsed / 1e12, 6), "unit": "TFLOP/s", "cores": 1, "kind": kind,
            "cpu_model": cpu_model(),
            "sample": f"{done} x {rows} tokens of the step through linear() "
                      f"({w.shape[0]} x {w.shape[1]} fp32 weights) in {elapsed:.1f} s, one thread"}


def run_projection(args, dist, world, rank, device, peaks, peak_kind):
    """qkv_append_bf16: Q/K/V projection + paged K/V append of the mixed
    step's 4 x 512 chunk tokens (inferlab_cuda_qkv_project_append).
    outproj_bf16: the output projection + residual add of the same tokens
    from the fp32 attention output (inferlab_cuda_output_project, which
    rounds its input to bf16 in the step). TFLOP/s of the GEMM."""
    import torch

    from inferlab_b200 import workloads as wl

    batch = wl.qkv_append_bf16(device=device, seed=2030 + rank)
    pool = batch.pool
    stream = torch.cuda.current_stream(device)
    dev = f"cuda:{device}"
    tokens, model_dim = batch.hidden.shape
    outproj = args.workload == "outproj_bf16"
    if outproj:
        gen = torch.Generator(device=dev).manual_seed(2040 + rank)
        attn = torch.randn((tokens, 32 * 128), generator=gen, device=dev)
        w_o = (torch.randn((model_dim, 32 * 128), generator=gen, device=dev) /
               (32 * 128) ** 0.5).to(torch.bfloat16)
        residual = torch.randn((tokens, model_dim), generator=gen, device=dev)
        out = torch.empty_like(residual)
        flops = 2 * tokens * model_dim * 32 * 128
    else:
        flops = batch.flops()
        q_out = torch.empty((tokens, batch.q_heads, 128), dtype=torch.bfloat16, device=dev)
    flush = L2Flush(device)

    def step():
        if outproj:
            pool.output_project(attn, w_o, residual, out=out)
        else:
            pool.project_append(batch.hidden, batch.weights, batch.q_heads, batch.row_sequences,
                                batch.positions, batch.block_tables, q_out=q_out)

    for i in range(args.warmup):
        flush.fill_(float(i))
        step()
    pool.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier(dist)
    torch.cuda.synchronize(device)
    with ClockSampler(device) as clocks:
        preroll_end = time.perf_counter() + 0.5
        while time.perf_counter() < preroll_end:
            flush.fill_(0.0)
            step()
            stream.synchronize()
        torch.cuda._sleep(int(2e6 + 3e5 * args.steps))
        for i in range(args.steps):
            flush.fill_(float(i))
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize(device)
        barrier(dist)
    pool.synchronize()
    kernel_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    total_ms = max_over_ranks(dist, kernel_ms)
    value = sum_over_ranks(dist, float(flops) * args.steps) / (total_ms * 1e-3) / 1e12
    achieved = flops / (kernel_ms / args.steps * 1e-3) / 1e12
    peak = float(peaks["bf16_tflops"])
    if outproj:
        metric = "output projection + residual TFLOP/s"
        workload = ("output projection of 4 x 512 chunk tokens: fp32 attention output "
                    "[2048][4096] rounded to bf16 in the step, W_o [4096][4096] bf16, fp32 "
                    "residual add")
        profile = "qkv_append_outproj_bf16"
    else:
        metric = "qkv projection + paged append TFLOP/s"
        workload = ("Q/K/V projection of 4 x 512 chunk tokens, model_dim 4096, GQA 32/8 x 128 "
                    "(N = 6144), K/V rows appended to a bf16 pool")
        profile = "qkv_append_qkv_append_bf16"
    line = {
        "metric": metric, "value": round(value, 3),
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,1)/sqrt(in) weights)",
        "config": {"workload": workload,
                   "flops_per_step": int(flops),
                   "l2": "flushed between steps: 256 MB write then 256 MB read of a second "
                         "buffer, outside the step events"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "peak_kind": f"{peak_kind} bf16_tflops",
                     "traffic": read_traffic(profile)},
        "gpu_launches": args.steps * (2 if outproj else 1), "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if outproj:
            batch.hidden, batch.weights = attn.to(torch.bfloat16), w_o
        line["cpu_baseline"] = cpu_projection_baseline(batch, min(args.cpu_seconds, 10.0))
    pool.close()
    return line



# ---------------------------------------------------------------------------
# other workloads
# ---------------------------------------------------------------------------
def run_mixed(args, dist, world, rank, device, peaks, peak_kind):
    """Continuous-batching step: one decode launch over the decode sequences
    and one prefill launch over the chunks, back to back on one stream."""
    import torch

    from inferlab_b200 import workloads as wl

    batch = wl.mixed_bf16(device=device, seed=2029 + rank)
    pool = batch.pool
    stream = torch.cuda.current_stream(device)
    flush = L2Flush(device)
    workspace = pool.make_workspace(len(batch.contexts), batch.q_heads, batch.max_context_len)
    out_d = torch.empty_like(batch.queries)
    out_p = torch.empty((batch.prefill_queries.shape[0], 32, 128), dtype=torch.float32,
                        device=f"cuda:{device}")

    def decode():
        pool.decode(batch.queries, batch.block_tables, batch.context_lens, batch.max_context_len,
                    out=out_d, workspace=workspace)

    def prefill():
        pool.prefill(batch.prefill_queries, batch.prefill_tables, batch.starts_dev,
                     batch.counts_dev, batch.offsets_dev, int(batch.counts.max()), out=out_p)

    for i in range(args.warmup):
        flush.fill_(float(i))
        decode()
        prefill()
    pool.synchronize()
    with ClockSampler(device) as clocks:
        ms_d, ms_p = timed_region(args, dist, device, stream, flush, [decode, prefill])
    pool.synchronize()
    step_ms = max_over_ranks(dist, (ms_d + ms_p) / args.steps)
    dbytes = batch.decode_bytes()
    flops = batch.prefill_flops()
    tokens = len(batch.contexts) + int(batch.counts.sum())
    line = {
        "metric": "continuous-batching step ms", "value": round(step_ms, 5), "unit": "ms",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_ms, 5), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": {"workload": "32 decode seqs ctx Zipf(1.1) clip [32,8192] + 4 x 512-token "
                               "chunked prefill, GQA 32/8 x 128 bf16, 65536-block pool",
                   "decode_contexts": [int(c) for c in batch.contexts],
                   "chunk_priors": [int(c) for c in batch.starts], "query_tokens": tokens},
        "decode": {"ms": round(ms_d / args.steps, 5), "GB/s": round(dbytes / (ms_d / args.steps) / 1e6, 2),
                   "frac_hbm": round(dbytes / (ms_d / args.steps) / 1e6 / peaks["hbm_gbs"], 4)},
        "prefill": {"ms": round(ms_p / args.steps, 5),
                    "TFLOP/s": round(flops / (ms_p / args.steps) / 1e9, 2),
                    "frac_tensor": round(flops / (ms_p / args.steps) / 1e9 / peaks["bf16_tflops"], 4)},
        "gpu_launches": 2 * args.steps, "clocks": clocks.summary(),
        "per_rank": per_rank(dist, ms_per_step=(ms_d + ms_p) / args.steps,
                             decode_ms=ms_d / args.steps, prefill_ms=ms_p / args.steps),
    }
    pool.close()
    return line



# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from oracle import oracle

    if oracle.ref_lib() is None:
        print(json.dumps({"impl": "reference",
                          "unavailable": "oracle/_ref/libref.so was not built (reference sources "
                                         "absent when the tree was prepared)"}), flush=True)
        return
    if args.workload == "prefill_f16":
        return run_reference_prefill(args, world)
    if args.workload in ("qkv_append_bf16", "outproj_bf16"):
        return run_reference_projection(args, world)
    if args.workload == "mixed_bf16":
        return run_reference_mixed(args, world)
    if args.workload in ("default", "longctx_bf16", "longseq_split"):
        return run_reference_long(args, world)
    if args.workload != "decode_fp32":
        print(json.dumps({"impl": "reference",
                          "unavailable": "reference arm implemented for every workload except "
                                         "single_seq_fp32, whose line times the reference "
                                         "itself"}),
              flush=True)
        return
    # Host-side copy of the same workload shape (seeded numpy; no GPU on this path).
    rng = np.random.Generator(np.random.PCG64(2026))
    num_seqs, heads, head_dim, blocks = 64, 8, 64, 8192
    contexts = rng.integers(64, 2048, size=num_seqs, endpoint=True)
    need = (contexts + 15) // 16
    perm = rng.permutation(blocks).astype(np.int32)
    tables = np.zeros((num_seqs, 128), np.int32)
    used = 0
    for i, n in enumerate(need):
        tables[i, :n] = perm[used:used + n]
        used += n
    k_arena = rng.standard_normal((blocks, heads, 16, head_dim), dtype=np.float32)
    v_arena = rng.standard_normal((blocks, heads, 16, head_dim), dtype=np.float32)
    q = rng.standard_normal((num_seqs, heads, head_dim), dtype=np.float32)
    ctx = contexts.astype(np.int64)
    bytes_per_step = (int(ctx.sum()) * heads * head_dim * 2 * 4 + 2 * num_seqs * heads * head_dim * 4
                      + int(need.sum()) * 4 + num_seqs * 4)
    threads = host_threads()
    for _ in range(args.warmup):
        oracle.reference_paged_decode_timed(k_arena, v_arena, 0, tables, contexts, q, heads,
                                            threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.reference_paged_decode_timed(k_arena, v_arena, 0, tables, contexts, q, heads,
                                            threads)
    elapsed = time.perf_counter() - t0
    value = bytes_per_step * args.steps / elapsed / 1e9
    line = {
        "impl": "reference", "metric": "decode attn KV-bytes GB/s", "value": round(value, 4),
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(elapsed / args.steps * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1))",
        "config": {"workload": "paged decode fp32: 64 seqs x ctx U[64,2048], 8 heads x 64 (MHA), "
                               "block 16, 8192-block pool, random permutation tables",
                   "num_seqs": num_seqs, "q_heads": heads, "kv_heads": heads,
                   "head_dim": head_dim, "block_tokens": 16, "pool_blocks": blocks},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads,
                         "kind": "reference",
                         "sample": "each step = the whole 64-sequence batch: page gather + "
                                   "inferlab_attention_forward (OnlineTiled, tile 16) per q-head "
                                   "from oracle/_ref/libref.so"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _reference_line(args, world, metric, value, unit, workload, threads, sample, dtype):
    return {
        "impl": "reference", "metric": metric, "value": round(value, 6), "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic (seeded)", "config": {"workload": workload},
        "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": threads,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_reference_prefill(args, world):
    """The reference's causal prefill on the host: inferlab_attention_forward
    (OnlineTiled, tile 16, Fp16 storage mode, causal) from oracle/_ref/libref.so,
    one call per head (heads = 1 on that head's slice) spread over the host
    threads. Each step is a bounded sample of the 8 x 1024 workload: one
    sequence, all 16 heads; TFLOP/s counts the same causal FLOPs as our arm."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle

    rng = np.random.Generator(np.random.PCG64(2028))
    tokens, heads, dim = 1024, 16, 128
    q = (rng.standard_normal((tokens, heads, dim), dtype=np.float32) * 0.5)
    k = (rng.standard_normal((tokens, heads, dim), dtype=np.float32) * 0.5)
    v = (rng.standard_normal((tokens, heads, dim), dtype=np.float32) * 0.5)
    per_head = [(np.ascontiguousarray(q[:, h]), np.ascontiguousarray(k[:, h]),
                 np.ascontiguousarray(v[:, h])) for h in range(heads)]
    threads = host_threads()

    def head(h):
        qh, kh, vh = per_head[h]
        oracle.attention_forward(qh, kh, vh, tokens, tokens, 1, dim, 0, oracle.ONLINE_TILED,
                                 oracle.FP16, 16, True, impl="reference")

    flops = 4 * dim * heads * tokens * (tokens + 1) // 2
    with ThreadPoolExecutor(max_workers=threads) as pool:
        for _ in range(args.warmup):
            list(pool.map(head, range(heads)))
        t0 = time.perf_counter()
        for _ in range(args.steps):
            list(pool.map(head, range(heads)))
        elapsed = time.perf_counter() - t0
    value = flops * args.steps / elapsed / 1e12
    line = _reference_line(
        args, world, "prefill attn TFLOP/s", value, "TFLOP/s",
        "causal prefill f16: 8 x 1024 tokens, 16 heads x 128 (reference: one sequence per step)",
        threads, "each step = one 1024-token sequence, 16 heads, one inferlab_attention_forward "
                 "call per head (OnlineTiled, tile 16, Fp16 mode) from oracle/_ref/libref.so",
        "f16")
    line["ms_per_step"] = round(elapsed / args.steps * 1e3, 4)
    print(json.dumps(line), flush=True)


def run_reference_mixed(args, world):
    """The reference's continuous-batching step on the host, as its worker runs
    it: one inferlab_attention_forward call per (sequence, q-head) - the 32
    decode sequences (contexts from the same seeded clipped Zipf as our arm)
    in full, and the 4 x 512-token chunks on a sample of 4 of their 32 q-heads,
    scaled by 8 (their cost is the same for every head). Bf16 storage mode,
    OnlineTiled, tile 16, causal; calls spread over the host threads. K/V
    values come from one shared random slice per call (the reference's cost
    does not depend on them)."""
    from concurrent.futures import ThreadPoolExecutor

    from inferlab_b200.workloads import zipf_contexts
    from oracle import oracle

    rng = np.random.Generator(np.random.PCG64(2029))
    contexts = zipf_contexts(rng, 32)
    priors = zipf_contexts(rng, 4)
    chunk, dim, q_heads, sample_heads = 512, 128, 32, 4
    data = np.random.Generator(np.random.PCG64(7))
    kmax = int(max(contexts.max(), (priors + chunk).max()))
    keys = data.standard_normal((kmax, dim), dtype=np.float32)
    values = data.standard_normal((kmax, dim), dtype=np.float32)
    q_dec = data.standard_normal((dim,), dtype=np.float32)
    q_pre = data.standard_normal((chunk, dim), dtype=np.float32)
    threads = host_threads()

    def decode_call(task):
        ctx = int(contexts[task // q_heads])
        oracle.attention_forward(q_dec, keys[:ctx], values[:ctx], 1, ctx, 1, dim, ctx - 1,
                                 oracle.ONLINE_TILED, oracle.BF16, 16, True, impl="reference")

    def prefill_call(task):
        prior = int(priors[task // sample_heads])
        kv = prior + chunk
        oracle.attention_forward(q_pre, keys[:kv], values[:kv], chunk, kv, 1, dim, prior,
                                 oracle.ONLINE_TILED, oracle.BF16, 16, True, impl="reference")

    dec_tasks = range(len(contexts) * q_heads)
    pre_tasks = range(len(priors) * sample_heads)
    with ThreadPoolExecutor(max_workers=threads) as pool:
        for _ in range(args.warmup):
            list(pool.map(decode_call, dec_tasks))
            list(pool.map(prefill_call, pre_tasks))
        t_dec = t_pre = 0.0
        for _ in range(args.steps):
            t0 = time.perf_counter()
            list(pool.map(decode_call, dec_tasks))
            t1 = time.perf_counter()
            list(pool.map(prefill_call, pre_tasks))
            t2 = time.perf_counter()
            t_dec += t1 - t0
            t_pre += t2 - t1
    scale = q_heads // sample_heads
    step_ms = (t_dec + scale * t_pre) / args.steps * 1e3
    line = _reference_line(
        args, world, "continuous-batching step ms", step_ms, "ms",
        "32 decode seqs ctx Zipf(1.1) clip [32,8192] + 4 x 512-token chunked prefill, GQA 32/8 "
        "x 128 bf16", threads,
        f"each step = the 32 decode sequences x 32 q-heads in full ({t_dec / args.steps * 1e3:.1f} "
        f"ms) + the 4 chunks on {sample_heads} of 32 q-heads ({t_pre / args.steps * 1e3:.1f} ms, "
        f"scaled x{scale}); one inferlab_attention_forward call per (sequence, q-head), Bf16 mode",
        "bf16")
    line["higher_is_better"] = False
    line["ms_per_step"] = round(step_ms, 4)
    print(json.dumps(line), flush=True)


def run_reference_long(args, world):
    """The reference's paged decode on the host for the long-context lines
    (GQA 32/8 x 128, bf16 storage): per sequence the page gather plus one
    inferlab_attention_forward call per q-head (Bf16 mode), the sequences in
    parallel over the host threads. Bounded samples: longctx_bf16 takes 4 of
    its 256 sequences per step, longseq_split the first 32,768 of the 131,072
    tokens (its whole step would hold ~2 GB of widened pages); GB/s counts the
    same algorithmic bytes as our arm."""
    from inferlab_b200.workloads import longctx_contexts
    from oracle import oracle

    longseq = args.workload == "longseq_split"
    contexts = np.array([32768], np.int64) if longseq else longctx_contexts(2027)[:4]
    kvh, q_heads, dim = 8, 32, 128
    need = (contexts + 15) // 16
    blocks = int(need.sum())
    rng = np.random.Generator(np.random.PCG64(2031))

    def arena():
        # bf16 storage bits of values with |x| in [2^-15, 1), random signs
        bits = rng.integers(0x3800, 0x3F80, size=(blocks, kvh, 16, dim), dtype=np.uint16)
        return bits | (rng.integers(0, 2, size=bits.shape, dtype=np.uint16) << 15)

    k_arena, v_arena = arena(), arena()
    perm = rng.permutation(blocks).astype(np.int32)
    tables = np.zeros((len(contexts), int(need.max())), np.int32)
    used = 0
    for i, n in enumerate(need):
        tables[i, :n] = perm[used:used + n]
        used += int(n)
    q = rng.standard_normal((len(contexts), q_heads, dim), dtype=np.float32)
    bytes_per_step = (int(contexts.sum()) * kvh * dim * 2 * 2 + 2 * len(contexts) * q_heads * dim * 4
                      + blocks * 4 + len(contexts) * 4)
    threads = host_threads()
    for _ in range(args.warmup):
        oracle.reference_paged_decode_timed(k_arena, v_arena, oracle.BF16, tables, contexts, q,
                                            q_heads, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.reference_paged_decode_timed(k_arena, v_arena, oracle.BF16, tables, contexts, q,
                                            q_heads, threads)
    elapsed = time.perf_counter() - t0
    value = bytes_per_step * args.steps / elapsed / 1e9
    sample = ("the first 32,768 tokens of the one 131,072-token sequence" if longseq
              else "4 of the 256 sequences (contexts " + ", ".join(str(int(c)) for c in contexts)
              + ")")
    line = _reference_line(
        args, world, "long-sequence decode KV-bytes GB/s" if longseq else "decode attn KV-bytes GB/s",
        value, "GB/s",
        ("one 131072-token sequence, GQA 32/8 x 128 bf16, blocks split across GPUs, NCCL "
         "all-gather of (m, l, o) + rank-order merge" if longseq
         else "paged decode bf16: 256 seqs x ctx U[4096,32768], GQA 32q/8kv x 128, block 16, "
              "sequences sharded across GPUs"), threads,
        f"each step = {sample}: page gather + one inferlab_attention_forward call per q-head "
        "(OnlineTiled, tile 16, Bf16 mode) from oracle/_ref/libref.so, on the host cores of "
        "one node whatever the GPU count", "bf16")
    if not longseq:
        line["config"].update({"num_seqs_total": 256, "q_heads": 32, "kv_heads": 8,
                               "head_dim": 128, "block_tokens": 16, "seed": 2027})
    line["scaling"] = "strong"
    line["ms_per_step"] = round(elapsed / args.steps * 1e3, 4)
    print(json.dumps(line), flush=True)


def run_reference_projection(args, world):
    """The reference's fp32 linear (worker/cpp/inferlab_runtime.cpp:1266-1285,
    oracle/_ref/libref_linear.so) over a bounded sample of the projection's
    tokens: 4 tokens per host thread per step, threads on disjoint rows."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle import projection

    rng = np.random.Generator(np.random.PCG64(2030))
    model_dim = 4096
    outproj = args.workload == "outproj_bf16"
    in_dim = 32 * 128 if outproj else model_dim
    out_dim = model_dim if outproj else (32 + 16) * 128
    w = (rng.standard_normal((out_dim, in_dim), dtype=np.float32) / np.float32(in_dim ** 0.5))
    threads = host_threads()
    rows = 4
    xs = [rng.standard_normal((rows, in_dim), dtype=np.float32) for _ in range(threads)]
    if projection.ref_linear(xs[0][:1], w[:32]) is None:
        print(json.dumps({"impl": "reference",
                          "unavailable": "oracle/_ref/libref_linear.so was not built (reference "
                                         "sources absent when the tree was prepared)"}), flush=True)
        return

    def part(i):
        projection.ref_linear(xs[i], w)

    with ThreadPoolExecutor(max_workers=threads) as pool:
        for _ in range(args.warmup):
            list(pool.map(part, range(threads)))
        t0 = time.perf_counter()
        for _ in range(args.steps):
            list(pool.map(part, range(threads)))
        elapsed = time.perf_counter() - t0
    flops = 2.0 * rows * threads * out_dim * in_dim * args.steps
    value = flops / elapsed / 1e12
    metric = ("output projection + residual TFLOP/s" if outproj
              else "qkv projection + paged append TFLOP/s")
    line = _reference_line(
        args, world, metric, value, "TFLOP/s",
        f"{'output' if outproj else 'Q/K/V'} projection {in_dim} -> {out_dim} (reference: "
        f"{rows * threads} tokens per step)",
        threads, f"each step = {rows} tokens on each of {threads} threads through the "
                 f"reference's linear() ({out_dim} x {in_dim} fp32 weights)", "f32")
    line["ms_per_step"] = round(elapsed / args.steps * 1e3, 4)
    print(json.dumps(line), flush=True)


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", default="default",
                        choices=["default", "longctx_bf16", "decode_fp32", "prefill_f16",
                                 "mixed_bf16", "longseq_split", "single_seq_fp32",
                                 "qkv_append_bf16", "outproj_bf16"])
    parser.add_argument("--longctx-seqs", type=int, default=256,
                        help="take the first N of the 256 long-context sequences (small "
                             "profiling cases)")
    parser.add_argument("--cpu-seconds", type=float, default=8.0)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)  # at least three untimed warm-up steps
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
