"""Index replicas: a 2-rank gloo group receives rank 0's index object and packed tables
intact (the host-side logic of the multi-GPU path; NCCL carries the same calls on GPUs)."""

from __future__ import annotations

import hashlib
import os
import socket

import numpy as np
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, out) -> None:
    import datetime

    import torch
    import torch.distributed as dist

    from xgraph_b200.replicas import broadcast_index
    from xgraph_b200.synthetic import build_workload
    from xgraph_b200.tables import pack_tables

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        workload = packed = None
        if rank == 0:
            workload = build_workload(1, 1)
            packed = pack_tables(workload.index, workload.served, workload.syntax, escapes=True)
        replica = broadcast_index(workload, packed, torch.device("cpu"))
        blob = replica.blob.numpy().tobytes()
        out.put((rank, hashlib.sha256(blob).hexdigest(), replica.packed.layout.blob_bytes,
                 replica.payload.index.base_fingerprint, replica.payload.served.vocab_size))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_receive_identical_replicas():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    results = sorted(out.get(timeout=10) for _ in range(2))
    assert results[0][1:] == results[1][1:]  # same blob hash, size, index identity, vocabulary
    assert results[0][2] > 0


def test_replay_plan_replenishes_every_slot():
    """Every slot replays whole streams back to back: each step's position lies inside its
    stream, positions advance by one, and a new stream starts at 0 right after one ends."""
    import bench

    lengths = np.random.default_rng(0).integers(3, 9, size=10)
    plan = bench.row_plan(4, lengths, 30, start=bench.entry_offsets(lengths, 4, seed=1))
    for r in range(4):
        for k in range(30):
            sid, pos = plan[r, k]
            assert 0 <= pos < lengths[sid]
            if k:
                psid, ppos = plan[r, k - 1]
                assert (sid, pos) == (psid, ppos + 1) or (pos == 0 and ppos == lengths[psid] - 1)
