"""Benchmark: the per-decode-step KG constraint engine (sync/advance + mask + apply).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--config 3]

Workload (default: config 3, "paths-100k"): a seeded KG of 100,000 entities with 1-3
labels each, 100 relations and 1,000,000 uniform triples, a seeded 128,256-id byte-level
BPE, path mode with committed paths; 256 request rows per GPU with stream lengths
uniform in [64, 1024], replenished continuously (a finished request's slot is re-begun
with the next stream, as a serving batch does); bf16 logits [256, 128256] ~ N(0, 2).
The token streams are constrained decodes sampled on the GPU under the engine's own
masks (xgraph_b200.synthetic.sample_streams), then replayed the way the reference's
bench replays outputs (src/xgraph/bench.py:82-139): per step `sync` over the token
history in place, then `apply_mask` on the logits.

One timed step = begin(restarted slots) + sync + apply_mask, on one stream, bracketed by
CUDA events; L2 is flushed (a 512 MiB write) between steps outside the events.  The
stream is held by a bounded device spin before the timed steps while the host queues
them, so host launch latency never lands between a step's events.  value =
rows x steps / time (rows.steps/s), whole job over all ranks (max time over ranks).
roofline: the apply kernel (its own events) against the measured HBM copy bandwidth,
algorithmic bytes = sum over rows of 4*words (mask read) + 2*disallowed columns
(the -inf stores).  e2e: the same step through the public API with host buffers
(tokens and logits copied in from pinned memory, masked logits copied back, the uploads
and downloads of neighbouring steps overlapped on two copy streams).
cpu_baseline / --impl reference: the oracle (oracle/oracle.py, a restatement of the
reference's CPU Oracle) on the host cores, per row-step allowed set + masked logits +
advance, on a bounded sample of the same streams; its masks are also checked against
the engine's at the sampled steps.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "mask+advance rows.steps/s at B=256, V=128,256 (bf16 logits)"
UNIT = "rows.steps/s"


HOLD_CYCLES_PER_STEP = 1_000_000  # ~0.5 ms of device time per queued step: far above the host's launch time


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=512)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", choices=("engine", "reference"), default="engine")
    p.add_argument("--config", type=int, default=3)
    p.add_argument("--seed", type=int, default=3)
    p.add_argument("--cpu-seconds", type=float, default=25.0, help="CPU baseline budget per worker")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    p.add_argument("--e2e-steps", type=int, default=32)
    p.add_argument("--profile", action="store_true", help="short run for a profiler (no CPU leg, no e2e)")
    p.add_argument("--max-len", type=int, default=0, help="cap stream lengths (profiling runs)")
    return p.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# ---------------------------------------------------------------------------------------
# workload

def make_workload(config: int, seed: int):
    from xgraph_b200.synthetic import build_workload

    return build_workload(config, seed)


def schedule(lengths: list[int], rows: int, steps: int):
    """Per slot, the streams it replays back to back (stream ids) and, per step, the
    slots that start a new stream (replenishment)."""
    assigned = [[] for _ in range(rows)]
    restarts = [[] for _ in range(steps)]
    next_stream = 0
    for slot in range(rows):
        at = 0
        while at < steps:
            sid = next_stream % len(lengths)
            next_stream += 1
            assigned[slot].append((sid, at))
            restarts[at].append(slot)
            at += lengths[sid]
    return assigned, restarts


class Clocks:
    """nvidia-smi clock/throttle sampling during the timed region."""

    def __init__(self, device: int):
        self.path = Path(tempfile.mkstemp(suffix=".csv")[1])
        query = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={device}", f"--query-gpu={query}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.path.open("w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, value in zip(names, parts[5:9]):
                if value.lower() == "active":
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------------------
# CPU baseline: the oracle port on the host cores (spawned workers).

def _cpu_worker(args):
    index, served, options, jobs, budget = args
    from oracle.oracle import Oracle
    from xgraph_b200.syntax import SpanSyntax

    oracle = Oracle(index, served, SpanSyntax(), **options)
    vocab = served.vocab_size
    rng = np.random.default_rng(len(jobs))
    logits_src = rng.normal(0.0, 2.0, size=vocab).astype(np.float32)
    done, spent, mismatches = 0, 0.0, 0
    started = time.perf_counter()
    for tokens, sampled, masks in jobs:
        state = oracle.initial_state()
        for step, token in enumerate(tokens):
            if step in sampled:
                t0 = time.perf_counter()
                allowed = oracle.allowed(state)
                mask = np.zeros(vocab, dtype=bool)
                mask[list(allowed)] = True
                logits = logits_src.copy()
                logits[~mask] = -np.inf
                state = oracle.advance(state, token)
                spent += time.perf_counter() - t0
                done += 1
                words = masks[step]
                bits = np.unpackbits(words.view(np.uint8), bitorder="little")[:vocab].astype(bool)
                mismatches += int((bits != mask).any())
            else:
                state = oracle.advance(state, token)
            if time.perf_counter() - started > budget:
                break
        if time.perf_counter() - started > budget:
            break
    return done, spent, mismatches


def cpu_baseline(workload, streams, recorded, budget: float, workers: int | None = None) -> dict:
    import multiprocessing as mp

    cores = os.cpu_count() or 1
    workers = workers or max(1, min(cores, 32))
    jobs = [[] for _ in range(workers)]
    by_row: dict[int, list[int]] = {}
    for (row, step) in recorded:
        by_row.setdefault(row, []).append(step)
    for k, (row, steps) in enumerate(sorted(by_row.items())):
        last = max(steps)
        jobs[k % workers].append((streams[row][: last + 1], set(steps), {s: recorded[(row, s)] for s in steps}))
    options = dict(workload.config.options)
    ctx = mp.get_context("spawn")
    t0 = time.perf_counter()
    with ctx.Pool(workers) as pool:
        results = pool.map(_cpu_worker, [(workload.index, workload.served, options, j, budget) for j in jobs])
    wall = time.perf_counter() - t0
    done = sum(r[0] for r in results)
    spent = sum(r[1] for r in results)
    mismatches = sum(r[2] for r in results)
    per_core = done / spent if spent else 0.0
    return {
        "value": per_core * workers,
        "unit": UNIT,
        "cores": workers,
        "kind": "port",
        "sample": (f"{done} row-steps (oracle allowed set + masked logits + advance, V={workload.served.vocab_size}) "
                   f"at sampled positions of {len(by_row)} engine streams; {workers} spawned workers, "
                   f"value = per-core throughput x workers; wall {wall:.0f} s incl. oracle build"),
        "parity_sample": {"row_steps": done, "mask_mismatches": mismatches},
    }


# ---------------------------------------------------------------------------------------
# engine arm

def engine_arm(args) -> None:
    import torch
    import torch.distributed as dist

    from xgraph_b200.engine import Engine
    from xgraph_b200.synthetic import sample_streams
    from xgraph_b200.tables import pack_tables

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=device)
    # -- index: built once on rank 0, device tables broadcast over NCCL --------------------
    build_s = 0.0
    workload = packed = None
    if rank == 0:
        t0 = time.perf_counter()
        workload = make_workload(args.config, args.seed)
        packed = pack_tables(workload.index, workload.served, workload.syntax, escapes=True)
        build_s = time.perf_counter() - t0
    if world > 1:
        from xgraph_b200.replicas import broadcast_index

        replica = broadcast_index(workload, packed, device)
        workload, blob, meta = replica.payload, replica.blob, replica.packed
    else:
        blob, meta = torch.from_numpy(packed.blob).to(device), packed
    cfg = workload.config
    options = dict(cfg.options)
    rows = cfg.rows
    pool = 2 * rows
    gen_engine = Engine(workload.index, workload.served, workload.syntax, pool, device_blob=(blob, meta), **options)
    lo, hi = cfg.lengths
    if args.max_len:
        lo, hi = min(lo, args.max_len), min(hi, args.max_len)
    max_len = hi
    rng = np.random.default_rng(args.seed + 100 + rank)
    lengths = rng.integers(lo, hi + 1, size=pool).tolist()
    record = set()
    if rank == 0 and world == 1 and not args.no_cpu and not args.profile:
        for row in range(min(48, pool)):
            for s in sorted(set(rng.integers(0, lengths[row], size=4).tolist())):
                record.add((row, int(s)))
    t0 = time.perf_counter()
    tokens, counts, recorded = sample_streams(gen_engine, workload.served, workload.syntax, workload.world,
                                              pool, max_len, seed=args.seed + rank, record=record)
    torch.cuda.synchronize()
    sample_s = time.perf_counter() - t0
    del gen_engine
    # -- replay schedule -------------------------------------------------------------------
    # W warm-up steps, then K timed steps.  A step is begin(restarted slots) + sync_apply
    # (sync and apply_mask fused in one kernel); events bracket the whole step, and a
    # second pair brackets the sync_apply kernel alone (the roofline's kernel).
    # then (outside the profile mode) up to 128 more steps without the flush: the warm figure
    warm_steps = 0 if args.profile else min(args.steps, 128)
    total_steps = args.warmup + args.steps + warm_steps
    assigned, restarts = schedule(lengths, rows, total_steps)
    history = torch.zeros((rows, total_steps + 1), dtype=torch.int32, device=device)
    disallowed = np.zeros(total_steps, dtype=np.int64)  # sum over rows of disallowed columns
    counts_h = counts.cpu().numpy()
    vocab = workload.served.vocab_size
    for slot, parts in enumerate(assigned):
        for sid, at in parts:
            n = min(lengths[sid], total_steps - at)
            history[slot, at: at + n] = tokens[sid, :n]
            disallowed[at: at + n] += vocab - counts_h[sid, 1: n + 1]
    restart_t = [torch.tensor(r, dtype=torch.int32, device=device) if r else None for r in restarts]
    prompt = [torch.full((rows,), k, dtype=torch.int32, device=device) for k in range(total_steps)]
    total = [torch.full((rows,), k + 1, dtype=torch.int32, device=device) for k in range(total_steps)]
    slots = torch.arange(rows, dtype=torch.int32, device=device)
    gen = torch.Generator(device=device).manual_seed(7)
    dtype = getattr(torch, cfg.dtype)
    elt = torch.empty(0, dtype=dtype).element_size()
    logits = (torch.randn((rows, vocab), generator=gen, device=device) * 2.0).to(dtype)
    flush = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.int32, device=device)
    engine = Engine(workload.index, workload.served, workload.syntax, rows, device_blob=(blob, meta), **options)
    engine.reset()
    stream = torch.cuda.current_stream(device).cuda_stream
    launches = 0
    step_ms, apply_ms, warm_ms = [], [], []
    clocks = None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for k in range(total_steps):
        timed = args.warmup <= k < args.warmup + args.steps
        warm = k >= args.warmup + args.steps
        if timed and clocks is None:
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            clocks = Clocks(local)
            time.sleep(0.3)
            torch.cuda.nvtx.range_push("timed")
        if k == args.warmup or k == args.warmup + args.steps:
            # hold the stream (a bounded spin, outside every event pair) while the host
            # queues the leg's steps, so host launch latency never falls inside a step
            torch.cuda._sleep(HOLD_CYCLES_PER_STEP * (args.steps if timed else warm_steps))
        if not warm:
            flush.fill_(k)  # evict the logits and tables from L2 between steps
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        if restart_t[k] is not None:
            engine.begin(restart_t[k], stream=stream)
            launches += timed
        e1.record()
        engine.sync_apply(slots, history, prompt[k], total[k], logits, stream=stream)
        e2.record()
        launches += timed
        if timed:
            step_ms.append((e0, e2))
            apply_ms.append((e1, e2))
        elif warm:
            warm_ms.append((e0, e2))
    torch.cuda.synchronize()
    if clocks is not None:
        torch.cuda.nvtx.range_pop()
    clock_info = clocks.stop() if clocks else None
    errors = engine.errors()
    apply_alone = None if args.profile else apply_leg(engine, logits, slots, flush, stream, args.steps, elt)
    steps_ms = [a.elapsed_time(b) for a, b in step_ms]
    applies = [a.elapsed_time(b) for a, b in apply_ms]
    warms = [a.elapsed_time(b) for a, b in warm_ms]
    my_time = sum(steps_ms)
    time_t = torch.tensor([my_time], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(time_t, op=dist.ReduceOp.MAX)
        dist.barrier()
    job_ms = float(time_t.item())
    value = rows * world * args.steps / (job_ms / 1e3)
    # roofline of the apply kernel
    words = engine.words
    timed_steps = range(args.warmup, total_steps)
    # algorithmic bytes of one sync_apply launch: per row the state read+write and token
    # (516 B), the bitmask read once (4 * words) and the -inf stores (elt * disallowed)
    bytes_per_launch = [rows * (516 + 4 * words) + elt * int(disallowed[k]) for k in timed_steps]
    avg_apply_s = statistics.mean(applies) / 1e3
    achieved = statistics.mean(bytes_per_launch) / avg_apply_s / 1e9
    peak, peak_kind = measured_peak()
    result = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": job_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int32", "data": "synthetic",
        "config": {
            "workload": (f"{cfg.name} (config {args.config}): {cfg.entities:,} entities, {cfg.relations} relations, "
                         f"{cfg.triples:,} triples, V={vocab:,}, {rows} rows/GPU, stream lengths U[{lo},{hi}] "
                         f"replenished, paths+committed_paths, escapes on"),
            "rows_per_gpu": rows, "vocab": vocab, "logits_dtype": cfg.dtype, "logits": f"{cfg.dtype} [rows, V] ~ N(0,2)",
            "l2": "flushed between steps (512 MiB write, outside the timed region)",
            "timed_region": "begin(restarted slots) + sync + apply_mask per step, CUDA events, max over ranks",
            "parallelism": f"rows sharded, {world} replica(s), index broadcast once over NCCL",
        },
        "step_ms": {"median": statistics.median(steps_ms), "p90": sorted(steps_ms)[int(0.9 * len(steps_ms))],
                    "min": min(steps_ms), "max": max(steps_ms)},
        "warm": ({"ms_per_step": statistics.median(warms), "value": rows * 1e3 / statistics.median(warms),
                  "unit": UNIT, "steps": len(warms),
                  "note": "the same replay continued without the L2 flush (median step, this rank)"}
                 if warms else None),
        "kernel_ms": {"median": statistics.median(applies), "mean": statistics.mean(applies),
                      "note": "sync_apply kernel alone (events around it), over the K timed steps"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, **recorded_traffic(args.config, cfg.dtype),
                     "kernel": f"sync_apply_kernel<{elt}> ({cfg.dtype}): sync + mask + apply fused",
                     "algorithmic_bytes_per_launch": statistics.mean(bytes_per_launch)},
        "apply_mask_alone": apply_alone,
        "gpu_launches": launches,
        "clocks": clock_info,
        "errors": errors,
        "setup_s": {"workload_build": build_s, "stream_sampling": sample_s},
    }
    if not args.profile:
        e2e = e2e_leg(engine, workload, history, restart_t, prompt, total, slots, rows, vocab, device,
                      min(args.e2e_steps, total_steps), dtype)
        if world > 1:  # whole job: every rank's rows over the slowest rank's time
            e2e_t = torch.tensor([e2e["ms_per_step"]], dtype=torch.float64, device=device)
            dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
            e2e["ms_per_step"] = float(e2e_t.item())
            e2e["value"] = rows * world * 1e3 / e2e["ms_per_step"]
            e2e["timing"] = "max over ranks of each rank's end-to-end time; value over all ranks' rows"
        result["e2e"] = e2e
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    if world == 1 and not args.no_cpu and not args.profile and recorded:
        streams = tokens.cpu().numpy().tolist()
        result["cpu_baseline"] = cpu_baseline(workload, streams, recorded, args.cpu_seconds)
    print(json.dumps(result), flush=True)


def apply_leg(engine, logits, slots, flush, stream, steps, elt):
    """The bandwidth kernel alone: apply_mask (apply_kernel) over the same rows with the
    masks the replay left, `steps` launches with L2 flushed between them, CUDA events
    around each launch.  Algorithmic bytes per launch: the mask words read once per row and
    the -inf stores (counted from one launch on finite logits)."""
    import torch

    probe = torch.zeros_like(logits)
    engine.apply_mask(probe, slots, stream=stream)
    disallowed = int(torch.isneginf(probe).sum())
    del probe
    rows, words = logits.shape[0], engine.words
    bytes_per_launch = rows * 4 * words + elt * disallowed
    times = []
    for k in range(max(3, steps // 4) + 3):
        flush.fill_(k)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        engine.apply_mask(logits, slots, stream=stream)
        e1.record()
        if k >= 3:  # three warm-up launches
            times.append((e0, e1))
    torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in times]
    mean_s = statistics.mean(ms) / 1e3
    achieved = bytes_per_launch / mean_s / 1e9
    peak, peak_kind = measured_peak()
    return {"kernel": f"apply_kernel<{elt}>", "launches": len(ms), "ms_median": statistics.median(ms),
            "ms_mean": statistics.mean(ms), "algorithmic_bytes_per_launch": bytes_per_launch,
            "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind,
            "note": "apply_mask alone on the replay's final masks, L2 flushed between launches"}


def e2e_leg(engine, workload, history, restart_t, prompt, total, slots, rows, vocab, device, steps, dtype):
    """The same steps through the public API with host buffers: each step copies its
    tokens and logits in from pinned host memory and the masked logits back out.  The
    copies run the way a serving loop overlaps them: step k + 1's inputs go up on a copy
    stream while step k's masked logits come down on another (PCIe is full duplex), with
    two device buffers and events ordering each step's upload, step and download."""
    import torch

    host_tokens = history[:, :steps].t().contiguous().cpu().pin_memory()
    host_logits = (torch.randn((rows, vocab)) * 2.0).to(dtype).pin_memory()
    out_logits = torch.empty_like(host_logits).pin_memory()
    dev_hist = torch.zeros_like(history)
    dev_logits = [torch.empty((rows, vocab), dtype=dtype, device=device) for _ in range(2)]
    staging = [torch.empty(rows, dtype=torch.int32, device=device) for _ in range(2)]
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    compute = torch.cuda.current_stream(device)
    stream = compute.cuda_stream
    engine.reset()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(compute)
    up.wait_event(start)
    down.wait_event(start)
    uploaded = [torch.cuda.Event() for _ in range(steps)]
    stepped = [torch.cuda.Event() for _ in range(steps)]
    downloaded = [None, None]
    for k in range(steps):
        b = k & 1
        with torch.cuda.stream(up):
            if downloaded[b] is not None:
                up.wait_event(downloaded[b])  # buffer b's previous result is on the host
            staging[b].copy_(host_tokens[k], non_blocking=True)
            dev_logits[b].copy_(host_logits, non_blocking=True)
            uploaded[k].record(up)
        compute.wait_event(uploaded[k])
        dev_hist[:, k] = staging[b]
        if restart_t[k] is not None:
            engine.begin(restart_t[k], stream=stream)
        engine.sync_apply(slots, dev_hist, prompt[k], total[k], dev_logits[b], stream=stream)
        stepped[k].record(compute)
        with torch.cuda.stream(down):
            down.wait_event(stepped[k])
            out_logits.copy_(dev_logits[b], non_blocking=True)
            downloaded[b] = torch.cuda.Event()
            downloaded[b].record(down)
    compute.wait_stream(down)
    end.record(compute)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    return {"value": rows * steps / (ms / 1e3), "unit": UNIT,
            "h2d_bytes_per_step": rows * 4 + rows * vocab * host_logits.element_size(),
            "d2h_bytes_per_step": rows * vocab * host_logits.element_size(),
            "steps": steps, "ms_per_step": ms / steps,
            "copies": "inputs up and results down on two copy streams, overlapped across steps"}


# ---------------------------------------------------------------------------------------
# reference arm: the oracle port on the host cores

def recorded_traffic(config: int, dtype: str) -> dict:
    """DRAM bytes per launch of the fused kernel from the committed ncu capture of the same
    kernel on the same rows and vocabulary (profiles/sync_apply_paths100k.json), or None
    for another workload.  The capture's logits writes stay in L2 during the kernel."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles", "sync_apply_paths100k.json")
    if config != 3 or dtype != "bfloat16":
        return {"traffic": None}
    try:
        with open(path) as f:
            data = json.load(f)
        return {"traffic": statistics.mean(data["dram_bytes_per_launch"]),
                "traffic_source": f"ncu capture, {data['workload']}: dram__bytes_read.sum + dram__bytes_write.sum"}
    except (OSError, KeyError, ValueError):
        return {"traffic": None}


def reference_arm(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import torch

    from xgraph_b200.engine import Engine
    from xgraph_b200.synthetic import sample_streams

    workload = make_workload(args.config, args.seed)
    cfg = workload.config
    rows = cfg.rows
    rng = np.random.default_rng(args.seed + 100)
    lengths = rng.integers(cfg.lengths[0], cfg.lengths[1] + 1, size=rows).tolist()
    # streams are sampled as in the engine arm (the CPU only replays them)
    engine = Engine(workload.index, workload.served, workload.syntax, rows, **cfg.options)
    record = set()
    for row in range(rows):
        for s in sorted(set(rng.integers(0, lengths[row], size=2).tolist())):
            record.add((row, int(s)))
    tokens, _, recorded = sample_streams(engine, workload.served, workload.syntax, workload.world, rows,
                                         cfg.lengths[1], seed=args.seed, record=record)
    streams = tokens.cpu().numpy().tolist()
    del engine
    torch.cuda.empty_cache()
    budget = max(20.0, min(150.0, 0.3 * (args.steps + args.warmup)))
    base = cpu_baseline(workload, streams, recorded, budget)
    value = base["value"]
    result = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": base["parity_sample"]["row_steps"], "warmup": 0,
        "ms_per_step": 1e3 * rows / value if value else None, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int32", "data": "synthetic",
        "config": {"workload": f"{cfg.name} (config {args.config}), {rows} rows, V={workload.served.vocab_size:,}",
                   "note": "CPU oracle port on the host cores; each step a bounded sample of row-steps"},
        "cpu_baseline": base,
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(result), flush=True)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        reference_arm(args)
    else:
        engine_arm(args)


if __name__ == "__main__":
    main()
