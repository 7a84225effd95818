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
from dataclasses import dataclass

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "mask+advance rows.steps/s at B=256, V=128,256 (bf16 logits)"


def metric_of(config: int, rows: int, vocab: int) -> str:
    """The headline metric's name (config 3); another configuration names its own batch."""
    return METRIC if config == 3 else f"mask+advance rows.steps/s at B={rows}, V={vocab:,} (bf16 logits)"
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
    p.add_argument("--policies", action="store_true",
                   help="time the step with apply_mask's logit policies on (release, escape bias; fresh logits per step)")
    p.add_argument("--synchronized", action="store_true",
                   help="every row enters its first stream at position 0 at step 0 (default: seeded positions)")
    return p.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# ---------------------------------------------------------------------------------------
# workload

def make_workload(config: int, seed: int):
    from xgraph_b200.synthetic import build_workload

    return build_workload(config, seed)


def admissions_tensor(joined: list[tuple[int, int]], device):
    """Device admission records (xgraph_b200.engine.ADMISSION_INTS int32 each) beginning
    each (slot, KG version number) pair's slot on that version (0 = the base KG)."""
    import torch

    from xgraph_b200.engine import ADMISSION_INTS

    records = np.zeros((len(joined), ADMISSION_INTS), dtype=np.int32)
    for k, (slot, version) in enumerate(joined):
        records[k, :3] = (slot, 1, version)
    return torch.from_numpy(records).to(device)


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
# Token streams: the committed fixture both arms replay (tests/golden/make_streams.py made
# it with the engine's sampler on a GPU; tests/test_streams_fixture.py checks every token
# against the oracle).  Configurations without a fixture sample their streams on the GPU.

STREAM_FIXTURES = {3: ROOT / "tests" / "golden" / "streams_paths100k.npz"}


def load_streams(config: int, workload):
    """(tokens [P, L] int32, lengths [P] int32, allowed counts [P, L + 1] int32) of the
    configuration's fixture, or None when it has none."""
    path = STREAM_FIXTURES.get(config)
    if path is None or not path.is_file():
        return None
    data = np.load(path)
    if int(data["config"]) != config or int(data["vocab"]) != workload.served.vocab_size:
        raise RuntimeError(f"{path} was made for another workload")
    if str(data["fingerprint"]) != workload.served.fingerprint:
        raise RuntimeError(f"{path} was made with another tokenizer")
    return data["tokens"].astype(np.int32), data["lengths"].astype(np.int32), data["allowed"].astype(np.int32)


def entry_offsets(lengths, rows: int, seed: int):
    """Where each row enters its first stream: a seeded position uniform in the stream, so
    that the batch is in its replenished steady state (requests at every point of their
    output, as in a serving batch) from the first timed step rather than all starting
    together.  The tokens before it are consumed before the steps (enter_rows)."""
    rng = np.random.default_rng(seed)
    return np.array([int(rng.integers(0, max(int(lengths[r]), 1))) for r in range(rows)], dtype=np.int64)


def row_plan(rows: int, lengths, steps: int, offset: int = 0, start=None):
    """Per row, the (stream, position) it replays at each step: row r replays streams
    offset + r, offset + r + rows, ... back to back (a finished request's slot takes the
    next one, as a serving batch does), entering its first one at position start[r]."""
    n = len(lengths)
    plan = np.zeros((rows, steps, 2), dtype=np.int64)
    for r in range(rows):
        sid, at = (offset + r) % n, 0 if start is None else int(start[r])
        for k in range(steps):
            if at >= lengths[sid]:
                sid, at = (sid + rows) % n, 0
            plan[r, k] = (sid, at)
            at += 1
    return plan


# ---------------------------------------------------------------------------------------
# The oracle on the host cores (spawned workers): the CPU baseline of the engine arm and
# the whole of the reference arm.  Worker w owns rows w, w + workers, ...; at every step
# each of its rows takes its next token, and one of them (in turn) takes it the way a
# CPU decoding loop would (allowed set, masked logits, advance: examples/sampling_loop.py
# of the reference), the others by advance alone.  Throughput = full row-steps / wall time.

_WORKER = {}


def _worker_init(index, served, syntax, options, tokens, vocab, versions=None, row_versions=None):
    from oracle.oracle import Oracle

    _WORKER["oracle"] = Oracle(index, served, syntax, versions=versions, **options)
    _WORKER["row_versions"] = row_versions
    _WORKER["tokens"] = tokens
    _WORKER["vocab"] = vocab
    _WORKER["states"] = {}
    rng = np.random.default_rng(0)
    _WORKER["logits"] = rng.normal(0.0, 2.0, size=vocab).astype(np.float32)


def _worker_step(job):
    """One step of one worker: job = (rows: [(row, stream, position)], full row index,
    mask words expected at the full row-step or None).  Returns (seconds of the full
    row-step, mask mismatch 0/1/None)."""
    oracle, tokens, vocab = _WORKER["oracle"], _WORKER["tokens"], _WORKER["vocab"]
    states = _WORKER["states"]
    rows, full, expected = job
    spent, mismatch = 0.0, None
    for row, sid, pos in rows:
        if pos == 0 or row not in states:
            versions = _WORKER.get("row_versions")
            states[row] = oracle.initial_state(versions[row] if versions else None)
            for earlier in tokens[sid, :pos]:  # a row entering its stream mid-way: the prefix first
                states[row] = oracle.advance(states[row], int(earlier))
        token = int(tokens[sid, pos])
        if row == full:
            t0 = time.perf_counter()
            state = states[row]
            allowed = oracle.allowed(state)
            mask = np.zeros(vocab, dtype=bool)
            mask[list(allowed)] = True
            logits = _WORKER["logits"].copy()
            logits[~mask] = -np.inf
            states[row] = oracle.advance(state, token)
            spent = time.perf_counter() - t0
            if expected is not None:
                bits = np.unpackbits(expected.view(np.uint8), bitorder="little")[:vocab].astype(bool)
                mismatch = int((bits != mask).any())
        else:
            states[row] = oracle.advance(states[row], token)
    return spent, mismatch


def _worker_main(conn, init_args):
    _worker_init(*init_args)
    conn.send("ready")
    while True:
        job = conn.recv()
        if job is None:
            break
        conn.send(_worker_step(job))


def oracle_leg(workload, tokens, lengths, rows: int, steps: int, warmup: int, *, budget: float | None = None,
               expected: dict | None = None, workers: int | None = None, versions: dict | None = None,
               row_versions: list | None = None, start=None) -> dict:
    """The oracle replaying rows x (warmup + steps) of the streams on `workers` spawned
    processes, each owning a fixed set of rows; a step waits for every worker.  With
    `budget` (seconds) the timed steps stop early once it is spent.  expected:
    {(stream, position): mask words} to check the full row-steps against."""
    import multiprocessing as mp

    cores = os.cpu_count() or 1
    workers = workers or max(1, min(cores, 32, rows))
    plan = row_plan(rows, lengths, warmup + steps, start=start)
    owned = [list(range(w, rows, workers)) for w in range(workers)]
    init = (workload.index, workload.served, workload.syntax, dict(workload.config.options), tokens,
            workload.served.vocab_size, versions, row_versions)
    ctx = mp.get_context("spawn")
    t_setup = time.perf_counter()
    pipes, procs = [], []
    for _ in range(workers):
        here, there = ctx.Pipe()
        proc = ctx.Process(target=_worker_main, args=(there, init), daemon=True)
        proc.start()
        pipes.append(here)
        procs.append(proc)
    try:
        for conn in pipes:
            if conn.recv() != "ready":
                raise RuntimeError("an oracle worker failed to start")
        setup = time.perf_counter() - t_setup
        done = mismatches = checked = timed = 0
        busy = wall = 0.0
        for k in range(warmup + steps):
            jobs = []
            for mine in owned:
                full = mine[k % len(mine)]
                want = None
                if expected is not None:
                    want = expected.get((int(plan[full, k, 0]), int(plan[full, k, 1])))
                jobs.append(([(r, int(plan[r, k, 0]), int(plan[r, k, 1])) for r in mine], full, want))
            t0 = time.perf_counter()
            for conn, job in zip(pipes, jobs):
                conn.send(job)
            results = [conn.recv() for conn in pipes]
            elapsed = time.perf_counter() - t0
            if k >= warmup:
                wall += elapsed
                timed += 1
                done += workers
                busy += sum(r[0] for r in results)
            for _, m in results:
                if m is not None:
                    checked += 1
                    mismatches += m
            if budget is not None and k >= warmup and wall > budget:
                break
    finally:
        for conn in pipes:
            try:
                conn.send(None)
            except OSError:
                pass
        for proc in procs:
            proc.join(timeout=30)
            if proc.is_alive():
                proc.terminate()
    return {"row_steps": done, "steps": timed, "wall_s": wall, "busy_s": busy, "workers": workers,
            "setup_s": setup, "checked": checked, "mismatches": mismatches}


def cpu_baseline(workload, tokens, lengths, rows: int, expected: dict, budget: float, start=None) -> dict:
    leg = oracle_leg(workload, tokens, lengths, rows, steps=10_000, warmup=2, budget=budget, expected=expected,
                     start=start)
    value = leg["row_steps"] / leg["wall_s"] if leg["wall_s"] else 0.0
    return {
        "value": value, "unit": UNIT, "cores": leg["workers"], "kind": "port",
        "sample": (f"{leg['row_steps']} row-steps of the same streams (oracle allowed set + masked logits + "
                   f"advance, V={workload.served.vocab_size:,}) over {leg['steps']} steps on {leg['workers']} "
                   f"spawned workers; value = row-steps / wall seconds ({leg['wall_s']:.1f} s)"),
        "per_core_value": leg["row_steps"] / leg["busy_s"] if leg["busy_s"] else 0.0,
        "parity_sample": {"row_steps": leg["checked"], "mask_mismatches": leg["mismatches"]},
    }


# ---------------------------------------------------------------------------------------
# engine arm

@dataclass
class Replay:
    """What the timed loop replays: the engine's slots, each step's rows (slots, in logits
    row order), admissions and token history (history[slot, k] is the token slot `slot`
    consumes at step k), the disallowed columns summed over each step's rows (for the
    roofline's algorithmic bytes), the KG versions to register, and how the streams came."""

    slots: int
    history: object
    step_slots: list
    admissions: list
    live: list
    disallowed: np.ndarray
    versions: list
    streams_source: str
    cpu: dict
    start: np.ndarray | None = None  # per slot, the history column of step 0 (tokens before it: a prefix)


def enter_rows(engine, replay, device) -> None:
    """Before step 0: rows that enter their first stream mid-way begin and consume the
    stream's earlier tokens (one sync over each row's prefix, outside every timed region)."""
    import torch

    if replay.start is None or not replay.start.any():
        return
    rows = replay.slots
    every = torch.arange(rows, dtype=torch.int32, device=device)
    engine.admit(admissions_tensor([(r, 0) for r in range(rows)], device))
    zeros = torch.zeros(rows, dtype=torch.int32, device=device)
    engine.sync(every, replay.history, zeros, torch.from_numpy(replay.start.astype(np.int32)).to(device))


def fixture_replay(args, workload, device, rank: int, total_steps: int, blob_meta, lo_hi) -> Replay:
    """Configs 1-4: rows replay token streams back to back (the committed fixture, rank r its
    own rotation of it, or streams sampled on the GPU when the configuration has none); a
    request joining a slot is an admission (begin, base KG) folded into its step's launch."""
    import torch

    from xgraph_b200.engine import Engine
    from xgraph_b200.synthetic import sample_streams

    cfg = workload.config
    rows, pool, vocab = cfg.rows, 2 * cfg.rows, workload.served.vocab_size
    fixture = load_streams(args.config, workload)
    if fixture is not None:
        all_tokens, all_lengths, all_allowed = fixture
        pick = [(rank * rows + j) % len(all_lengths) for j in range(pool)]
        tokens_np, lengths, counts_h = all_tokens[pick], all_lengths[pick], all_allowed[pick]
        source = f"fixture {STREAM_FIXTURES[args.config].name}"
    else:
        gen_engine = Engine(workload.index, workload.served, workload.syntax, pool, device_blob=blob_meta,
                            **cfg.options)
        rng = np.random.default_rng(args.seed + 100 + rank)
        lengths = rng.integers(cfg.lengths[0], cfg.lengths[1] + 1, size=pool)
        sampled, counts, _ = sample_streams(gen_engine, workload.served, workload.syntax, workload.world,
                                            pool, cfg.lengths[1], seed=args.seed + rank)
        tokens_np, counts_h = sampled.cpu().numpy(), counts.cpu().numpy()
        del gen_engine
        source = "sampled on the GPU with the engine's masks (no fixture for this configuration)"
    lengths = np.maximum(np.minimum(lengths, lo_hi[1]), 1)
    start = None if args.synchronized else entry_offsets(lengths, rows, args.seed + 500 + rank)
    plan = row_plan(rows, lengths, total_steps, start=start)
    sid, pos = plan[:, :, 0], plan[:, :, 1]
    first = np.zeros(rows, dtype=np.int64) if start is None else start
    steps_np = np.ascontiguousarray(tokens_np[sid, pos], dtype=np.int32)
    history_np = np.zeros((rows, int(first.max()) + total_steps), dtype=np.int32)
    for r in range(rows):  # row r: its first stream's prefix, then the tokens of its steps
        history_np[r, : first[r]] = tokens_np[r, : first[r]]
        history_np[r, first[r]: first[r] + total_steps] = steps_np[r]
    history = torch.from_numpy(history_np).to(device)
    disallowed = (vocab - counts_h[sid, pos + 1]).sum(axis=0).astype(np.int64)
    every = torch.arange(rows, dtype=torch.int32, device=device)
    admissions = []
    for k in range(total_steps):
        joined = np.flatnonzero(pos[:, k] == 0).tolist()
        admissions.append(admissions_tensor([(slot, 0) for slot in joined], device) if joined else None)
    return Replay(rows, history, [every] * total_steps, admissions, [rows] * total_steps, disallowed, [], source,
                  {"tokens": tokens_np, "lengths": lengths}, first)


def versions_replay(args, workload, device, rank: int, total_steps: int, blob_meta) -> Replay:
    """The versions configuration: continuous batching on this GPU's share of the arrivals
    (synthetic.arrival_schedule: Poisson, geometric lengths, ragged batches), each request
    carrying 0..max_edits seeded add/remove edits as its own KG version, registered with the
    engine (Engine.add_version, between steps, outside the timed launches) and selected by
    the request's admission; streams sampled on the GPU under each request's version."""
    import torch

    from xgraph_b200.engine import Engine
    from xgraph_b200.synthetic import arrival_schedule, object_sets, request_edits, sample_streams

    cfg = workload.config
    vocab = workload.served.vocab_size
    sched = arrival_schedule(cfg, total_steps, args.seed, rank)
    admitted = [r for r in range(len(sched.arrival)) if sched.slot[r] >= 0]
    pairs = object_sets(workload.world)
    rng = np.random.default_rng(args.seed * 7919 + rank)
    edits = {f"request-{rank}-{r}": request_edits(workload.world, pairs, rng, int(rng.integers(0, cfg.max_edits + 1)))
             for r in admitted}
    names = list(edits)
    steps = max(sched.length[r] for r in admitted)
    gen_engine = Engine(workload.index, workload.served, workload.syntax, len(admitted), device_blob=blob_meta,
                        **cfg.options)
    t0 = time.perf_counter()
    for name in names:
        gen_engine.add_version(name, edits[name])
    torch.cuda.synchronize()
    add_ms = 1e3 * (time.perf_counter() - t0) / max(len(names), 1)
    tokens, counts, _ = sample_streams(gen_engine, workload.served, workload.syntax, workload.world, len(admitted),
                                       steps, seed=args.seed + 31 * rank, versions=names)
    tokens_np, counts_h = tokens.cpu().numpy(), counts.cpu().numpy()
    del gen_engine
    rows = cfg.rows
    history = np.zeros((rows, total_steps), dtype=np.int32)
    disallowed = np.zeros(total_steps, dtype=np.int64)
    joins: list[list[tuple[int, int]]] = [[] for _ in range(total_steps)]
    for j, r in enumerate(admitted):
        slot, k0 = sched.slot[r], sched.start[r]
        n = min(sched.length[r], total_steps - k0)
        history[slot, k0: k0 + n] = tokens_np[j, :n]
        disallowed[k0: k0 + n] += vocab - counts_h[j, 1: n + 1]
        joins[k0].append((slot, j))
    version_of = {j: j + 1 for j in range(len(admitted))}  # numbers in the replay engine: added in this order
    admissions = [admissions_tensor([(slot, version_of[j]) for slot, j in joined], device) if joined else None
                  for joined in joins]
    step_slots = [torch.tensor(live, dtype=torch.int32, device=device) for live in sched.live]
    return Replay(rows, torch.from_numpy(history).to(device), step_slots, admissions,
                  [len(live) for live in sched.live], disallowed, [(name, edits[name]) for name in names],
                  f"sampled on the GPU under each request's version ({len(admitted)} requests)",
                  {"add_version_ms": add_ms, "requests": len(admitted),
                   "edits_mean": float(np.mean([len(e) for e in edits.values()])) if edits else 0.0,
                   "tokens": tokens_np, "names": names, "edits": edits, "lengths": [sched.length[r] for r in admitted]})


def engine_arm(args) -> None:
    import torch
    import torch.distributed as dist

    from xgraph_b200.engine import Engine
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
    if args.policies:
        options.update(release_mass=POLICY_RELEASE_MASS, escape_bias=POLICY_ESCAPE_BIAS)
    vocab = workload.served.vocab_size
    lo, hi = cfg.lengths
    if args.max_len:
        lo, hi = min(lo, args.max_len), min(hi, args.max_len)
    # W warm-up steps, then K timed steps, then (outside the profile mode) up to 128 more
    # steps without the flush: the warm figure.  A step is one sync_apply launch (the step's
    # admissions, sync and apply_mask fused), bracketed by CUDA events.
    warm_steps = 0 if args.profile else min(args.steps, 128)
    total_steps = args.warmup + args.steps + warm_steps
    t0 = time.perf_counter()
    if cfg.arrivals:
        replay = versions_replay(args, workload, device, rank, total_steps, (blob, meta))
    else:
        replay = fixture_replay(args, workload, device, rank, total_steps, (blob, meta), (lo, hi))
    sample_s = time.perf_counter() - t0
    rows, history = replay.slots, replay.history
    first = torch.from_numpy((replay.start if replay.start is not None else np.zeros(rows)).astype(np.int32)).to(device)
    prompt = [first + k for k in range(total_steps)]  # a joining request's first token is its step's column
    total = [first + (k + 1) for k in range(total_steps)]
    gen = torch.Generator(device=device).manual_seed(7)
    dtype = getattr(torch, cfg.dtype)
    elt = torch.empty(0, dtype=dtype).element_size()
    logits = (torch.randn((rows, vocab), generator=gen, device=device) * 2.0).to(dtype)
    fresh = logits.clone() if args.policies else None  # the release mass reads the logits: fresh ones each step
    flush = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.int32, device=device)
    engine = Engine(workload.index, workload.served, workload.syntax, rows, device_blob=(blob, meta), **options)
    for name, edits in replay.versions:
        engine.add_version(name, edits)
    engine.reset()
    enter_rows(engine, replay, device)
    stream = torch.cuda.current_stream(device).cuda_stream
    launches = 0
    step_ms, warm_ms = [], []
    timed_rows = warm_rows = 0
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
        if fresh is not None:
            logits.copy_(fresh)
        if not warm:
            flush.fill_(k)  # evict the logits and tables from L2 between steps
        n = replay.live[k]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        engine.sync_apply(replay.step_slots[k], history, prompt[k], total[k], logits[:n], stream=stream,
                          admissions=replay.admissions[k])
        e1.record()
        if timed:
            launches += 1
            timed_rows += n
            step_ms.append((e0, e1))
        elif warm:
            warm_rows += n
            warm_ms.append((e0, e1))
    torch.cuda.synchronize()
    if clocks is not None:
        torch.cuda.nvtx.range_pop()
    clock_info = clocks.stop() if clocks else None
    errors = engine.errors()
    faults = engine.faults()
    last_slots = replay.step_slots[total_steps - 1]
    apply_alone = (None if args.profile else
                   apply_leg(engine, logits[: len(last_slots)], last_slots, flush, stream, args.steps, elt))
    policies = (None if args.profile or args.policies else
                policies_leg(workload, replay, (blob, meta), options, prompt, total, flush, stream, device,
                             args.warmup, args.steps, dtype, gen))
    steps_ms = [a.elapsed_time(b) for a, b in step_ms]
    warms = [a.elapsed_time(b) for a, b in warm_ms]
    time_t = torch.tensor([sum(steps_ms)], dtype=torch.float64, device=device)
    rows_t = torch.tensor([timed_rows], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(time_t, op=dist.ReduceOp.MAX)
        dist.all_reduce(rows_t, op=dist.ReduceOp.SUM)
        dist.barrier()
    job_ms = float(time_t.item())
    value = float(rows_t.item()) / (job_ms / 1e3)  # every rank's rows over the slowest rank's time
    # algorithmic bytes of one launch: per row of the step the state read+write and token
    # (516 B), the bitmask read once (4 * words) and the -inf stores (elt * disallowed)
    words = engine.words
    timed_steps = range(args.warmup, args.warmup + args.steps)
    bytes_per_launch = [replay.live[k] * (516 + 4 * words) + elt * int(replay.disallowed[k]) for k in timed_steps]
    achieved = statistics.mean(bytes_per_launch) / (statistics.mean(steps_ms) / 1e3) / 1e9
    peak, peak_kind = measured_peak()
    result = {
        "metric": metric_of(args.config, rows, vocab), "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": job_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int32", "data": "synthetic",
        "config": {**workload_config(cfg, args.config, rows, vocab, lo, hi, world, args.synchronized),
                   **({"policies": {"release_mass": POLICY_RELEASE_MASS, "escape_bias": POLICY_ESCAPE_BIAS}}
                      if args.policies else {})},
        "timed_region": "one sync_apply launch per step (admissions of joining requests, sync, apply_mask), "
                        "CUDA events on the launching stream, max over ranks",
        "streams": replay.streams_source,
        "rows_per_step": timed_rows / args.steps,
        "step_ms": {"median": statistics.median(steps_ms), "p90": sorted(steps_ms)[int(0.9 * len(steps_ms))],
                    "min": min(steps_ms), "max": max(steps_ms)},
        "warm": ({"ms_per_step": statistics.median(warms), "value": warm_rows / (sum(warms) / 1e3),
                  "unit": UNIT, "steps": len(warms),
                  "note": "the same replay continued without the L2 flush (median step, this rank)"}
                 if warms else None),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, **recorded_traffic(args.config, cfg.dtype, args.max_len),
                     "level": ("L2: the -inf writes land in the 126 MB L2 during the launch and reach HBM "
                               "when later writes evict them"),
                     "kernel": f"sync_apply_kernel<{elt}> ({cfg.dtype}): admissions + sync + mask + apply fused",
                     "algorithmic_bytes_per_launch": statistics.mean(bytes_per_launch)},
        "apply_mask_alone": apply_alone,
        "policies_on": policies,
        "gpu_launches": launches,
        "clocks": clock_info,
        "errors": errors,
        "device_faults": faults,
        "setup_s": {"workload_build": build_s, "streams": sample_s},
    }
    if "add_version_ms" in replay.cpu:
        result["versions"] = {k: replay.cpu[k] for k in ("requests", "edits_mean", "add_version_ms")}
    if not args.profile:
        e2e = e2e_leg(engine, replay, prompt, total, vocab, device, min(args.e2e_steps, total_steps), dtype)
        if world > 1:  # whole job: every rank's rows over the slowest rank's time
            e2e_t = torch.tensor([e2e["ms_per_step"]], dtype=torch.float64, device=device)
            dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
            e2e["ms_per_step"] = float(e2e_t.item())
            e2e["value"] = e2e["rows_per_step"] * world * 1e3 / e2e["ms_per_step"]
            e2e["timing"] = "max over ranks of each rank's end-to-end time; value over all ranks' rows"
        result["e2e"] = e2e
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    if world == 1 and not args.no_cpu and not args.profile:
        if "add_version_ms" in replay.cpu:
            result["cpu_baseline"] = versions_cpu_baseline(workload, replay, args.cpu_seconds)
        else:
            tokens_np, lengths = replay.cpu["tokens"], replay.cpu["lengths"]
            expected = replay_masks(engine, tokens_np, lengths, rows, CPU_CHECK_STEPS, replay.start)
            result["cpu_baseline"] = cpu_baseline(workload, tokens_np, lengths, rows, expected, args.cpu_seconds,
                                                  replay.start)
    print(json.dumps(result), flush=True)


CPU_CHECK_STEPS = 96  # the CPU leg's first steps, whose full row-steps are checked against the engine's masks


def replay_masks(engine, tokens, lengths, rows: int, steps: int, start=None) -> dict:
    """{(stream, position): mask words} for `steps` positions of streams 0..rows-1 from where
    the oracle leg's rows enter them (start, default 0), from the engine replaying the
    streams with advance + fill_mask (the mask before each position's token)."""
    import torch

    first = np.zeros(rows, dtype=np.int64) if start is None else np.asarray(start)
    engine.reset()
    device = torch.device("cuda", torch.cuda.current_device())
    engine.begin(torch.arange(rows, dtype=torch.int32, device=device))
    view = engine.mask_view()
    out = {}
    horizon = int(min(np.max(first + steps), np.max(lengths[:rows])))
    for at in range(horizon):
        engine.fill_mask(rows)
        keep = [r for r in range(rows) if first[r] <= at < min(first[r] + steps, lengths[r])]
        if keep:
            words = view[:rows, : engine.words].cpu().numpy().view(np.uint32)
            for r in keep:
                out[(r, at)] = words[r].copy()
        engine.advance(np.ascontiguousarray(tokens[:rows, at], dtype=np.int32))
    return out


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


POLICY_RELEASE_MASS = 0.35
POLICY_ESCAPE_BIAS = -0.75


def policies_leg(workload, replay, blob_meta, options, prompt, total, flush, stream, device, warmup, steps,
                 dtype, gen):
    """The same replay through an engine with apply_mask's logit policies on (release below
    POLICY_RELEASE_MASS of allowed mass, POLICY_ESCAPE_BIAS on the committing tokens): each
    span row whose escape marker can go on reads its whole logits row once for its allowed
    mass before its -inf writes.  Fresh N(0, 2) logits every step (copied in outside the
    timed region, then L2 flushed); one sync_apply launch per step between CUDA events."""
    import torch

    from xgraph_b200.engine import Engine

    engine = Engine(workload.index, workload.served, workload.syntax, replay.slots, device_blob=blob_meta,
                    release_mass=POLICY_RELEASE_MASS, escape_bias=POLICY_ESCAPE_BIAS, **options)
    for name, edits in replay.versions:
        engine.add_version(name, edits)
    engine.reset()
    enter_rows(engine, replay, device)
    vocab = workload.served.vocab_size
    fresh = (torch.randn((replay.slots, vocab), generator=gen, device=device) * 2.0).to(dtype)
    logits = torch.empty_like(fresh)
    times, rows = [], 0
    for k in range(warmup + steps):
        logits.copy_(fresh)
        flush.fill_(k)
        n = replay.live[k]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        engine.sync_apply(replay.step_slots[k], replay.history, prompt[k], total[k], logits[:n], stream=stream,
                          admissions=replay.admissions[k])
        e1.record()
        if k >= warmup:
            times.append((e0, e1))
            rows += n
    torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in times]
    faults = engine.faults()
    return {"release_mass": POLICY_RELEASE_MASS, "escape_bias": POLICY_ESCAPE_BIAS, "steps": len(ms),
            "ms_per_step": statistics.mean(ms), "ms_median": statistics.median(ms),
            "value": rows / (sum(ms) / 1e3), "unit": UNIT, "device_faults": faults,
            "note": "the timed replay again with release and escape bias on (one rank), fresh logits per step, "
                    "L2 flushed; span rows read their logits row for the allowed mass"}


def e2e_leg(engine, replay, prompt, total, vocab, device, steps, dtype):
    """The same steps through the public API with host buffers: each step copies its
    tokens and its rows' logits in from pinned host memory and the masked logits back out.
    The copies run the way a serving loop overlaps them: step k + 1's inputs go up on a copy
    stream while step k's masked logits come down on another (PCIe is full duplex), with
    two device buffers and events ordering each step's upload, step and download."""
    import torch

    rows = replay.slots
    history = replay.history
    live = replay.live[:steps]
    first = replay.start if replay.start is not None else np.zeros(rows, dtype=np.int64)
    width = history.shape[1]
    # step k of row r is history column first[r] + k: its flat index, one gather per step
    flat = [torch.from_numpy(np.arange(rows) * width + first + k).to(device) for k in range(steps)]
    host_np = history.cpu().numpy()
    host_tokens = torch.from_numpy(np.stack([host_np[np.arange(rows), first + k] for k in range(steps)])).pin_memory()
    host_logits = (torch.randn((rows, vocab)) * 2.0).to(dtype).pin_memory()
    out_logits = torch.empty_like(host_logits).pin_memory()
    dev_hist = history.clone()  # the prefixes; each step's column is uploaded again in its step
    dev_logits = [torch.empty((rows, vocab), dtype=dtype, device=device) for _ in range(2)]
    staging = [torch.empty(rows, dtype=torch.int32, device=device) for _ in range(2)]
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    compute = torch.cuda.current_stream(device)
    stream = compute.cuda_stream
    engine.reset()
    enter_rows(engine, replay, device)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(compute)
    up.wait_event(start)
    down.wait_event(start)
    uploaded = [torch.cuda.Event() for _ in range(steps)]
    stepped = [torch.cuda.Event() for _ in range(steps)]
    downloaded = [None, None]
    for k in range(steps):
        b, n = k & 1, live[k]
        with torch.cuda.stream(up):
            if downloaded[b] is not None:
                up.wait_event(downloaded[b])  # buffer b's previous result is on the host
            staging[b].copy_(host_tokens[k], non_blocking=True)
            dev_logits[b][:n].copy_(host_logits[:n], non_blocking=True)
            uploaded[k].record(up)
        compute.wait_event(uploaded[k])
        dev_hist.view(-1).index_copy_(0, flat[k], staging[b])
        engine.sync_apply(replay.step_slots[k], dev_hist, prompt[k], total[k], dev_logits[b][:n], stream=stream,
                          admissions=replay.admissions[k])
        stepped[k].record(compute)
        with torch.cuda.stream(down):
            down.wait_event(stepped[k])
            out_logits[:n].copy_(dev_logits[b][:n], non_blocking=True)
            downloaded[b] = torch.cuda.Event()
            downloaded[b].record(down)
    compute.wait_stream(down)
    end.record(compute)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    element = host_logits.element_size()
    mean_rows = sum(live) / steps
    return {"value": sum(live) / (ms / 1e3), "unit": UNIT,
            "h2d_bytes_per_step": int(rows * 4 + mean_rows * vocab * element),
            "d2h_bytes_per_step": int(mean_rows * vocab * element),
            "steps": steps, "ms_per_step": ms / steps, "rows_per_step": mean_rows,
            "copies": "inputs up and results down on two copy streams, overlapped across steps"}


def versions_cpu_baseline(workload, replay, budget: float, workers: int = 4) -> dict:
    """The oracle on the host cores for the versions configuration: `workers` processes, each
    holding the KG versions of the requests it replays (a 10 M-edge oracle per process, so few
    of them), every step one full row-step per worker; value = row-steps / wall seconds."""
    names, edits, tokens = replay.cpu["names"], replay.cpu["edits"], replay.cpu["tokens"]
    lengths = np.asarray(replay.cpu["lengths"], dtype=np.int32)
    rows = min(len(names), 2 * workers)
    chosen = {names[r]: edits[names[r]] for r in range(rows)}
    leg = oracle_leg(workload, tokens[:rows], lengths[:rows], rows, steps=10_000, warmup=1, budget=budget,
                     workers=workers, versions=chosen, row_versions=names[:rows])
    value = leg["row_steps"] / leg["wall_s"] if leg["wall_s"] else 0.0
    return {"value": value, "unit": UNIT, "cores": leg["workers"], "kind": "port",
            "sample": (f"{leg['row_steps']} row-steps of {rows} requests, each under its own KG version (oracle "
                       f"allowed set + masked logits + advance, V={workload.served.vocab_size:,}) over "
                       f"{leg['steps']} steps on {leg['workers']} spawned workers; value = row-steps / wall seconds"),
            "per_core_value": leg["row_steps"] / leg["busy_s"] if leg["busy_s"] else 0.0,
            "oracle_setup_s": leg["setup_s"]}


# ---------------------------------------------------------------------------------------
# reference arm: the oracle port on the host cores

TRAFFIC_RECORD = ROOT / "profiles" / "sync_apply_paths100k.json"


def recorded_traffic(config: int, dtype: str, max_len: int) -> dict:
    """DRAM bytes per launch of the fused step as ncu recorded them for this workload
    (config 3, bf16, full stream lengths) with the command the record names; a record, not a
    measurement of this run (ncu cannot count inside a timed run), and None for any other
    workload."""
    if config != 3 or dtype != "bfloat16" or max_len:
        return {"traffic": None}
    try:
        data = json.loads(TRAFFIC_RECORD.read_text())
        return {"traffic": statistics.mean(data["dram_bytes_per_launch"]),
                "traffic_source": (f"recorded, not measured in this run: ncu dram__bytes_read.sum + "
                                   f"dram__bytes_write.sum of {data['workload']} ({data['command']}, "
                                   f"kernel source {data['kernel_source']})")}
    except (OSError, KeyError, ValueError):
        return {"traffic": None}


REFERENCE_BUDGET_S = 150.0


def reference_arm(args) -> None:
    """The reference's CPU implementation of the path (its Oracle, restated in oracle/) on
    the host cores, replaying the same committed streams as the engine arm: rows of the
    workload split over spawned workers, each step one full row-step per worker (allowed set,
    masked logits, advance) and advance alone for its other rows.  Loads nothing of the
    engine (no CUDA library).  Under torchrun only rank 0 runs."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    workload = make_workload(args.config, args.seed)
    cfg = workload.config
    fixture = load_streams(args.config, workload)
    if fixture is None:
        print(json.dumps({"impl": "reference", "unavailable": f"no committed token streams for config {args.config}"}))
        return
    tokens, lengths, _ = fixture
    rows, pool = cfg.rows, 2 * cfg.rows
    lo, hi = cfg.lengths
    if args.max_len:
        lo, hi = min(lo, args.max_len), min(hi, args.max_len)
        lengths = np.minimum(lengths, args.max_len)
    # every timed step takes about one V-wide allowed set per worker (about a second): the
    # timed steps stop after REFERENCE_BUDGET_S so that a long --steps still ends in minutes
    start = None if args.synchronized else entry_offsets(lengths[:pool], rows, args.seed + 500)
    leg = oracle_leg(workload, tokens[:pool], lengths[:pool], rows, steps=args.steps, warmup=args.warmup,
                     budget=REFERENCE_BUDGET_S, start=start)
    value = leg["row_steps"] / leg["wall_s"] if leg["wall_s"] else 0.0
    result = {
        "impl": "reference", "metric": metric_of(args.config, rows, workload.served.vocab_size), "value": value, "unit": UNIT, "n_gpus": world, "steps": leg["steps"],
        "warmup": args.warmup, "ms_per_step": 1e3 * leg["wall_s"] / max(leg["steps"], 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int32", "data": "synthetic",
        "config": workload_config(cfg, args.config, rows, workload.served.vocab_size, lo, hi, world,
                                  args.synchronized),
        "cpu_baseline": {
            "value": value, "unit": UNIT, "cores": leg["workers"], "kind": "port",
            "sample": (f"each step {leg['workers']} full row-steps (oracle allowed set + masked logits + advance, "
                       f"V={workload.served.vocab_size:,}), one per worker, while every row of the batch advances; "
                       f"value = full row-steps / wall seconds over the {leg['steps']} timed steps"),
            "per_core_value": leg["row_steps"] / leg["busy_s"] if leg["busy_s"] else 0.0,
        },
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "setup_s": {"oracle_workers": leg["setup_s"]},
        "streams": f"fixture {STREAM_FIXTURES[args.config].name}",
        "engine_library_loaded": engine_library_loaded(),
    }
    print(json.dumps(result), flush=True)


def engine_library_loaded() -> bool:
    """Whether this process mapped the engine's CUDA library (the reference arm must not)."""
    try:
        return "libxgraph_b200" in Path("/proc/self/maps").read_text()
    except OSError:
        return False


def workload_config(cfg, number: int, rows: int, vocab: int, lo: int, hi: int, world: int,
                    synchronized: bool = False) -> dict:
    """The `config` object of both arms' lines (the workload, not how an arm runs it)."""
    if cfg.arrivals:
        batching = (f"Poisson arrivals {cfg.arrivals:,.0f} req/s over {cfg.gpus} GPUs on a {cfg.step_ms} ms step "
                    f"clock, output lengths Geometric(mean {cfg.mean_length:.0f}) capped at {hi}, up to {rows} live "
                    f"rows/GPU, 0-{cfg.max_edits} seeded add/remove edits per request as its own KG version")
    else:
        entry = "all at position 0" if synchronized else "each at a seeded position of its first stream"
        batching = f"{rows} rows/GPU, stream lengths U[{lo},{hi}] replenished, rows entering {entry}"
    return {
        "workload": (f"{cfg.name} (config {number}): {cfg.entities:,} entities, {cfg.relations} relations, "
                     f"{cfg.triples:,} triples, V={vocab:,}, {batching}, paths+committed_paths, escapes on"),
        "rows_per_gpu": rows, "vocab": vocab, "logits_dtype": cfg.dtype, "logits": f"{cfg.dtype} [rows, V] ~ N(0,2)",
        "l2": "GPU arm: flushed between steps (512 MiB write, outside the timed region)",
        "parallelism": f"rows sharded, {world} replica(s), index broadcast once over NCCL",
    }


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        reference_arm(args)
    else:
        engine_arm(args)


if __name__ == "__main__":
    main()
