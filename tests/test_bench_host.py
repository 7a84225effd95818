"""Host logic of bench.py on the CPU: the replay plan and the oracle legs (the CPU baseline
and the reference arm), on the toy configuration with streams sampled through the host
build of the kernel logic."""

from __future__ import annotations

import numpy as np

import bench


def test_row_plan_replays_streams_back_to_back():
    lengths = np.array([3, 2, 4, 1])
    plan = bench.row_plan(2, lengths, 6)
    # row 0: stream 0 (3 tokens), then stream 2 (4 tokens); row 1: stream 1 (2), then 3 (1), then 1 again
    assert plan[0, :, 0].tolist() == [0, 0, 0, 2, 2, 2]
    assert plan[0, :, 1].tolist() == [0, 1, 2, 0, 1, 2]
    assert plan[1, :, 0].tolist() == [1, 1, 3, 1, 1, 3]
    assert plan[1, :, 1].tolist() == [0, 1, 0, 0, 1, 0]


def test_oracle_leg_replays_and_checks_against_the_kernel_logic():
    import torch

    from tests.seam import SeamEngine
    from tests.test_synthetic import _begin_adapter
    from xgraph_b200.synthetic import build_workload, sample_streams

    w = build_workload(1)
    rows = 4
    engine = SeamEngine(w.index, w.served, w.syntax, 2 * rows, **w.config.options)
    engine.begin = _begin_adapter(engine)  # sample_streams begins a tensor of slots
    steps = 24
    tokens, _, _ = sample_streams(engine, w.served, w.syntax, w.world, 2 * rows, steps, seed=5, device="cpu")
    tokens = tokens.numpy()
    lengths = np.array([steps] * (2 * rows), dtype=np.int32)
    # the kernel logic's masks at every position of streams 0..rows-1
    check = SeamEngine(w.index, w.served, w.syntax, rows, **w.config.options)
    expected = {}
    for slot in range(rows):
        check.begin(slot)
    for at in range(steps):
        masks = check.masks()
        for r in range(rows):
            expected[(r, at)] = masks[r].copy()
        check.advance(tokens[:rows, at])
    leg = bench.oracle_leg(w, tokens, lengths, rows, steps=6, warmup=1, expected=expected, workers=2)
    assert leg["steps"] == 6 and leg["row_steps"] == 12 and leg["workers"] == 2
    assert leg["checked"] == 14 and leg["mismatches"] == 0  # warm-up row-steps are checked too
    assert leg["wall_s"] > 0 and torch is not None


def test_rows_enter_their_first_stream_at_seeded_positions():
    lengths = np.array([5, 9, 3, 7])
    start = bench.entry_offsets(lengths, 2, seed=4)
    assert start.tolist() == bench.entry_offsets(lengths, 2, seed=4).tolist()  # seeded
    assert all(0 <= start[r] < lengths[r] for r in range(2))
    plan = bench.row_plan(2, lengths, 12, start=start)
    for r in range(2):
        assert plan[r, 0].tolist() == [r, start[r]]  # row r enters stream r at its offset
        # then runs to the stream's end and takes the next one from its start
        left = int(lengths[r] - start[r])
        assert plan[r, left].tolist() == [r + 2, 0]
