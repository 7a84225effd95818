"""Admissions in one launch, and the fused step at every grid shape, through the C ABI.

`admit` applies a batch of admissions (begin / end, anchors, KG version, open_span) in one
kernel; `sync_apply(..., admissions=...)` folds them into the decoding step's launch.  Both
must leave every slot exactly as the reference adapter's single calls do
(src/xgraph/vllm.py:569-605: begin, set_reached, set_version, open_span, then sync), and
the fused step must equal sync + apply_mask whether a CTA runs one row or several.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import golden_walks
from tests.test_engine_gpu import engine_for, start

pytestmark = pytest.mark.gpu


def admissions_of(sequences, *, on=True):
    from xgraph_b200.engine import Admission

    return [Admission(k, on, tuple(seq["anchor"] or ()), seq["version"], bool(seq["opened"]))
            for k, seq in enumerate(sequences)]


def assert_same_slots(a, b, n, *, same_numbers=True):
    """Equal states, masks and memory counts (and KG version numbers, unless the engines
    registered their versions in different orders)."""
    sa, sb = a.states_host(n), b.states_host(n)
    for field in sa:
        np.testing.assert_array_equal(sa[field], sb[field], field)
    a.fill_mask(n)
    b.fill_mask(n)
    np.testing.assert_array_equal(a.mask_host(n), b.mask_host(n))
    ma, mb = a.memory_host(n), b.memory_host(n)
    np.testing.assert_array_equal(ma[:, :3], mb[:, :3])  # facts, reached, frontier
    if same_numbers:
        np.testing.assert_array_equal(ma[:, 3], mb[:, 3])  # the KG version number


@pytest.mark.parametrize("name", ["toy_derivation", "bpe_committed", "crowd_committed", "bytes_paths"])
def test_admit_equals_single_calls(name):
    """One admit launch = begin + anchor + set_version + open_span per slot, then the same walk."""
    case = next(c for c in golden_walks() if c["name"] == name)
    sequences = case["sequences"]
    n = len(sequences)
    single, _, _ = engine_for(case)
    batched, _, _ = engine_for(case)
    start(single, sequences)
    batched.reset()
    batched.admit(admissions_of(sequences))
    assert_same_slots(single, batched, n)
    for step in range(min(40, len(sequences[0]["tokens"]))):
        tokens = np.array([seq["tokens"][step] for seq in sequences], dtype=np.int32)
        single.advance(tokens)
        batched.advance(tokens)
    assert_same_slots(single, batched, n)
    assert batched.faults() == 0


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_sync_apply_admissions_equal_separate_admission(dtype):
    """Requests re-admitted mid-replay inside the fused step (one launch) end exactly where
    admit + sync_apply leaves them; an admission for a slot that is not a row of the step,
    and an end (on=False), are applied too."""
    import torch

    from xgraph_b200.engine import Admission

    case = next(c for c in golden_walks() if c["name"] == "bpe_committed")
    sequences = case["sequences"]
    n = len(sequences)
    spare = n  # a slot that is never a row of the steps
    fused, _, served = engine_for(case, slots=n + 1)
    plain, _, _ = engine_for(case, slots=n + 1)
    for engine in (fused, plain):
        engine.reset()
        engine.admit(admissions_of(sequences))
    steps = len(sequences[0]["tokens"])
    width = 2 * steps
    history = torch.zeros((n + 1, width), dtype=torch.int32, device="cuda")
    for k, seq in enumerate(sequences):  # each slot replays its walk twice, re-admitted between
        history[k, :steps] = torch.tensor(seq["tokens"], dtype=torch.int32)
        history[k, steps:] = torch.tensor(seq["tokens"], dtype=torch.int32)
    slots = torch.arange(n, dtype=torch.int32, device="cuda")
    prompt_len = torch.zeros(n + 1, dtype=torch.int32, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(5)
    element = torch.int16 if dtype == "bfloat16" else torch.int32
    for at in range(0, width, 9):
        total = torch.full((n + 1,), min(at + 9, width), dtype=torch.int32, device="cuda")
        admitted = []
        if at <= steps < at + 9:  # the walks restart: a new request per slot, prompt = first walk
            prompt_len[:n] = steps
            admitted = admissions_of(sequences)
            admitted.append(Admission(spare, True, (), sequences[0]["version"], True))
        if at == 45:
            admitted = [Admission(n - 1, False)]  # the last row's request leaves
        logits = torch.randn((n, served.vocab_size + 5), generator=gen, device="cuda").to(getattr(torch, dtype))
        a, b = logits.clone(), logits.clone()
        fused.sync_apply(slots, history, prompt_len, total, a, admissions=admitted or None)
        if admitted:
            plain.admit(admitted)
        plain.sync_apply(slots, history, prompt_len, total, b)
        assert torch.equal(a.view(element), b.view(element)), at
        assert_same_slots(fused, plain, n + 1)
    assert fused.faults() == 0 and plain.faults() == 0


def test_device_admissions_out_of_range_are_skipped_and_counted():
    import torch

    from xgraph_b200.engine import ADMISSION_INTS

    case = next(c for c in golden_walks() if c["name"] == "toy_committed")
    engine, _, _ = engine_for(case, slots=2)
    engine.reset()
    records = np.zeros((2, ADMISSION_INTS), dtype=np.int32)
    records[0, :2] = (0, 1)
    records[1, :3] = (1, 1, 99)  # no KG version 99
    engine.admit(torch.from_numpy(records).cuda())
    assert engine.faults() == 2
    states = engine.states_host(2)
    assert int(states["phase"][0]) == 0
    with pytest.raises(ValueError):
        engine.admit(records)  # host records are checked before anything launches
    assert engine.faults() == 0


@pytest.mark.parametrize("rows", [700, 1300])
def test_fused_step_with_several_rows_per_cta(rows):
    """More rows than one resident wave of CTAs: each CTA runs several rows at once (and, past
    four per CTA, in turn); the result is still sync + apply_mask."""
    import torch

    case = next(c for c in golden_walks() if c["name"] == "bpe_committed")
    sequences = case["sequences"]
    fused, _, served = engine_for(case, slots=rows)
    plain, _, _ = engine_for(case, slots=rows)
    steps = len(sequences[0]["tokens"])
    history = torch.zeros((rows, steps), dtype=torch.int32, device="cuda")
    for r in range(rows):
        history[r] = torch.tensor(sequences[r % len(sequences)]["tokens"], dtype=torch.int32)
    wanted = [sequences[r % len(sequences)] for r in range(rows)]
    for engine in (fused, plain):
        engine.reset()
        engine.admit(admissions_of(wanted))
    slots = torch.arange(rows, dtype=torch.int32, device="cuda").flip(0).contiguous()  # rows in another order
    prompt_len = torch.zeros(rows, dtype=torch.int32, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(9)
    for at in range(0, steps, 13):
        total = torch.full((rows,), min(at + 13, steps), dtype=torch.int32, device="cuda")
        logits = torch.randn((rows, served.vocab_size), generator=gen, device="cuda").to(torch.bfloat16)
        a, b = logits.clone(), logits.clone()
        fused.sync_apply(slots, history, prompt_len, total, a)
        plain.sync(slots, history, prompt_len, total)
        plain.apply_mask(b, slots)
        assert torch.equal(a.view(torch.int16), b.view(torch.int16)), at
    assert_same_slots(fused, plain, rows)
    assert fused.faults() == 0
