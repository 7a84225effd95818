"""The CUDA engine (through its C ABI) against the golden walks and the apply contract.

Mirrors the reference's GPU agreement seam (tests/test_engine.py:1733-2002, 2147-2251):
at every step of every golden walk the device mask must equal the reference Oracle's
allowed set and the device state must agree with the reference state's projection;
apply_mask must write -inf exactly over disallowed columns (and columns past the
vocabulary), leave allowed columns bit-identical, and leave inactive and error rows alone.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.agreement import assert_agrees, engine_state, expected_state
from tests.conftest import case_index, case_options, case_versions, golden_masks, golden_walks, unpack, world

pytestmark = pytest.mark.gpu
CASES = [case["name"] for case in golden_walks()]


def engine_for(case, slots=None):
    from xgraph_b200.engine import Engine
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.syntax import SpanSyntax

    _, served, _ = world(case["world"])
    index = case_index(case)
    edits = case_versions(case)
    versions = build_kg_versions(index, edits) if edits else None
    options = case_options(case)
    engine = Engine(index, served, SpanSyntax(), slots or len(case["sequences"]), versions=versions, **options)
    return engine, index, served


def start(engine, sequences):
    import torch

    engine.reset()
    engine.begin(torch.arange(len(sequences), dtype=torch.int32, device="cuda"))
    for k, seq in enumerate(sequences):
        engine.set_version(k, seq["version"])
        if seq["anchor"]:
            engine.anchor(k, seq["anchor"])
        if seq["opened"]:
            engine.open_span(k)


@pytest.mark.parametrize("name", CASES)
def test_engine_agrees_with_reference_walks(name):
    from xgraph_b200.syntax import SpanSyntax

    case = next(c for c in golden_walks() if c["name"] == name)
    engine, index, served = engine_for(case)
    sequences = case["sequences"]
    start(engine, sequences)
    steps = len(sequences[0]["tokens"])
    paths = case["options"].get("paths", False)
    syntax = SpanSyntax()
    for step in range(steps + 1):
        engine.fill_mask()
        masks = engine.mask_host().view(np.uint32)
        states = engine.states_host()
        for k, seq in enumerate(sequences):
            record = seq["states"][step] if step < steps else seq["final"]
            where = (name, k, step)
            assert_agrees(expected_state(record, index, syntax),
                          engine_state(states, k, engine.view(seq["version"])), paths, where)
            if step < steps:
                expected = unpack(golden_masks()[f"{name}/{k}"][step], served.vocab_size)
                assert unpack(masks[k], served.vocab_size) == expected, where
        if step < steps:
            engine.advance(np.array([seq["tokens"][step] for seq in sequences], dtype=np.int32))
    assert engine.errors() == 0


@pytest.mark.parametrize("name", ["toy_ordinary", "bpe_committed", "crowd_committed"])
def test_sync_over_history_equals_advance(name):
    """sync reads each slot's history in place from prompt_len, then from its cursor."""
    import torch

    case = next(c for c in golden_walks() if c["name"] == name)
    sequences = case["sequences"]
    n = len(sequences)
    a, _, _ = engine_for(case)
    b, _, _ = engine_for(case)
    start(a, sequences)
    start(b, sequences)
    prompt = 5
    width = prompt + len(sequences[0]["tokens"])
    history = torch.zeros((n, width), dtype=torch.int32, device="cuda")
    for k, seq in enumerate(sequences):
        history[k, prompt:] = torch.tensor(seq["tokens"], dtype=torch.int32)
        history[k, :prompt] = 7  # the prompt is never advanced over
    prompt_len = torch.full((n,), prompt, dtype=torch.int32, device="cuda")
    slots = torch.arange(n, dtype=torch.int32, device="cuda")
    done = 0
    for chunk in (1, 3, 17, 1000):
        total = torch.clamp(prompt_len + done + chunk, max=width)
        b.sync(slots, history, prompt_len, total)
        for step in range(done, min(done + chunk, width - prompt)):
            a.advance(np.array([seq["tokens"][step] for seq in sequences], dtype=np.int32))
        done = min(done + chunk, width - prompt)
        a.fill_mask()
        b.fill_mask()
        np.testing.assert_array_equal(a.mask_host(), b.mask_host())
        sa, sb = a.states_host(), b.states_host()
        for field in sa:
            np.testing.assert_array_equal(sa[field], sb[field], field)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("pad", [0, 3, 40])
def test_apply_mask_writes_exactly_the_disallowed_columns(dtype, pad):
    import torch

    case = next(c for c in golden_walks() if c["name"] == "bpe_ordinary")
    sequences = case["sequences"]
    engine, _, served = engine_for(case, slots=len(sequences) + 2)
    start(engine, sequences)
    vocab = served.vocab_size
    rng = np.random.default_rng(5)
    for step in range(40):
        engine.advance(np.array([seq["tokens"][step] for seq in sequences], dtype=np.int32))
    engine.fill_mask()
    masks = engine.mask_host().view(np.uint32)
    # rows: every sequence, one inactive slot, and a repeated row
    row_slots = list(range(len(sequences))) + [len(sequences) + 1, 0]
    cols = vocab + pad
    stride = cols + 5  # rows start off 16-byte boundaries
    torch_dtype = getattr(torch, dtype)
    base = torch.tensor(rng.normal(size=(len(row_slots), stride)), dtype=torch_dtype, device="cuda")
    full = base.clone()
    logits = full[:, :cols]
    engine.apply_mask(logits, torch.tensor(row_slots, dtype=torch.int32, device="cuda"))
    got = logits.float().cpu().numpy()
    before = base[:, :cols].float().cpu().numpy()
    for r, slot in enumerate(row_slots):
        if slot >= len(sequences):
            np.testing.assert_array_equal(got[r], before[r])
            continue
        allowed = np.zeros(cols, dtype=bool)
        allowed[sorted(unpack(masks[slot], vocab))] = True
        assert np.all(np.isneginf(got[r][~allowed])), (r, slot)
        np.testing.assert_array_equal(got[r][allowed], before[r][allowed])
    # the elements between rows (stride padding) are untouched
    np.testing.assert_array_equal(full[:, cols:].float().cpu().numpy(), base[:, cols:].float().cpu().numpy())


def test_error_rows_are_left_untouched_and_counted():
    import torch

    case = next(c for c in golden_walks() if c["name"] == "toy_ordinary")
    engine, _, served = engine_for(case, slots=2)
    engine.reset()
    slots = torch.arange(2, dtype=torch.int32, device="cuda")
    engine.begin(slots)
    opener = served.encode(" ⟦")
    for t in opener:
        engine.advance(np.array([t, t], dtype=np.int32))
    special = sorted(served.special_ids)[0]
    engine.advance(np.array([special], dtype=np.int32))  # a special token inside a span
    assert engine.errors(2) == 1
    logits = torch.zeros((2, served.vocab_size), device="cuda")
    engine.apply_mask(logits, slots)
    assert torch.all(logits[0] == 0)  # error row untouched
    assert torch.isneginf(logits[1]).any()


def test_out_of_range_arguments_raise_value_error():
    import torch

    case = next(c for c in golden_walks() if c["name"] == "toy_committed")
    engine, _, _ = engine_for(case, slots=2)
    with pytest.raises(ValueError):
        engine.set_version(5, None)
    with pytest.raises(ValueError):
        engine.open_span(-1)
    with pytest.raises(ValueError):
        engine.anchor(0, ["no-such-entity"])
    with pytest.raises(ValueError):
        engine.set_version(0, "no-such-version")
    with pytest.raises(ValueError):
        engine.advance(np.zeros(3, dtype=np.int32))
    with pytest.raises(ValueError):
        engine.begin(torch.arange(3, dtype=torch.int32, device="cuda"))


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_sync_apply_equals_sync_then_apply_mask(dtype):
    """The fused step gives the states, masks and logits of sync followed by apply_mask."""
    import torch

    case = next(c for c in golden_walks() if c["name"] == "bpe_committed")
    sequences = case["sequences"]
    n = len(sequences)
    fused, _, served = engine_for(case)
    plain, _, _ = engine_for(case)
    start(fused, sequences)
    start(plain, sequences)
    steps = len(sequences[0]["tokens"])
    history = torch.zeros((n, steps), dtype=torch.int32, device="cuda")
    for k, seq in enumerate(sequences):
        history[k] = torch.tensor(seq["tokens"], dtype=torch.int32)
    slots = torch.arange(n, dtype=torch.int32, device="cuda")
    prompt_len = torch.zeros(n, dtype=torch.int32, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(3)
    for step in range(0, steps, 7):
        total = torch.full((n,), min(step + 7, steps), dtype=torch.int32, device="cuda")
        logits = torch.randn((n, served.vocab_size + 9), generator=gen, device="cuda").to(getattr(torch, dtype))
        a, b = logits.clone(), logits.clone()
        fused.sync_apply(slots, history, prompt_len, total, a)
        plain.sync(slots, history, prompt_len, total)
        plain.apply_mask(b, slots)
        assert torch.equal(a.view(torch.int16 if dtype == "bfloat16" else torch.int32),
                           b.view(torch.int16 if dtype == "bfloat16" else torch.int32)), step
        sa, sb = fused.states_host(), plain.states_host()
        for field in sa:
            np.testing.assert_array_equal(sa[field], sb[field], field)
        fused.fill_mask()
        plain.fill_mask()
        np.testing.assert_array_equal(fused.mask_host(), plain.mask_host())  # the recorded masks too


@pytest.mark.parametrize("name", ["bpe_norepeat", "bpe_committed", "crowd_committed", "toy_derivation"])
def test_draft_rows_mask_as_if_committed(name):
    """apply_mask with local_pos/input_ids (src/xgraph/engine.py:1012-1031): row k of a
    request's block has the mask of its slot's state after the block's first k drafts (the
    golden walk's mask k steps later), the slot's state does not move, a row after a
    disallowed draft and a row whose offset reaches before row 0 are left untouched."""
    import torch

    case = next(c for c in golden_walks() if c["name"] == name)
    sequences = case["sequences"]
    engine, _, served = engine_for(case)
    start(engine, sequences)
    vocab = served.vocab_size
    steps = len(sequences[0]["tokens"])
    drafts = 5
    gen = torch.Generator(device="cuda").manual_seed(11)
    done = 0
    for committed in (0, 17, steps - drafts - 1):
        for step in range(done, committed):
            engine.advance(np.array([seq["tokens"][step] for seq in sequences], dtype=np.int32))
        done = committed
        before = engine.states_host()
        row_slots, local_pos, input_ids, expect = [], [], [], []
        for k, seq in enumerate(sequences):
            for j in range(drafts + 1):
                row_slots.append(k)
                local_pos.append(j)
                fed = seq["tokens"][committed + j - 1] if committed + j > 0 else 0
                input_ids.append(fed)
                expect.append(unpack(golden_masks()[f"{name}/{k}"][committed + j], vocab))
        # one more request on slot 0 whose first draft is disallowed: its rows stay untouched
        allowed0 = unpack(golden_masks()[f"{name}/0"][committed], vocab)
        bad = next(t for t in range(vocab) if t not in allowed0) if len(allowed0) < vocab else None
        if bad is not None:
            for j in range(3):
                row_slots.append(0)
                local_pos.append(j)
                input_ids.append(bad if j == 1 else sequences[0]["tokens"][committed])
                expect.append(expect[0] if j == 0 else None)
        # an offset that reaches before row 0
        row_slots.append(0)
        local_pos.append(len(row_slots))
        input_ids.append(0)
        expect.append(None)
        rows = len(row_slots)
        cols = vocab + 3
        logits = torch.randn((rows, cols), generator=gen, device="cuda")
        original = logits.clone()
        as_t = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")  # noqa: E731
        engine.apply_mask(logits, as_t(row_slots), local_pos=as_t(local_pos), input_ids=as_t(input_ids))
        got, was = logits.cpu().numpy(), original.cpu().numpy()
        for r, want in enumerate(expect):
            if want is None:
                np.testing.assert_array_equal(got[r], was[r], err_msg=f"row {r} should be untouched")
                continue
            allowed = np.zeros(cols, dtype=bool)
            allowed[sorted(want)] = True
            assert np.all(np.isneginf(got[r][~allowed])), (name, committed, r)
            np.testing.assert_array_equal(got[r][allowed], was[r][allowed])
        after = engine.states_host()
        for field in before:
            np.testing.assert_array_equal(before[field], after[field], field)
