"""xg_apply_mask_noalloc (no counterpart in the reference): draft-row masking whose scratch
is a static device array in the library instead of an engine allocation.  Through the C
ABI, two calls in a row must write exactly what xg_apply_mask writes for the same rows,
and a call with more rows than the static array holds must fail without launching.

This file is collected last on purpose: it must pass alone in a fresh process and after
every other test (the static array is shared by every call in the process)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from tests.conftest import case_index, case_options, case_versions, golden_walks, world

pytestmark = pytest.mark.gpu

XG_OK, XG_EINVAL = 0, 1
F32 = 0


def _engine(case):
    from xgraph_b200.engine import Engine
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.syntax import SpanSyntax

    _, served, _ = world(case["world"])
    index = case_index(case)
    edits = case_versions(case)
    versions = build_kg_versions(index, edits) if edits else None
    engine = Engine(index, served, SpanSyntax(), len(case["sequences"]), versions=versions, **case_options(case))
    return engine, served


def _entry_points(engine):
    p, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    lib = engine._lib
    for name in ("xg_apply_mask", "xg_apply_mask_noalloc"):
        fn = getattr(lib, name)
        fn.argtypes = [p, p, i32, i32, i32, i64, p, p, p, p]
        fn.restype = ctypes.c_int
    return lib.xg_apply_mask, lib.xg_apply_mask_noalloc


def _call(fn, engine, logits, row_slots, local_pos, input_ids):
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    return fn(engine._handle, ptr(logits), F32, logits.shape[0], logits.shape[1], logits.stride(0),
              ptr(row_slots), ptr(local_pos), ptr(input_ids), None)


def _blocks(sequences, committed, drafts):
    """One request per slot: rows at offsets 0..drafts fed the walk's next tokens."""
    row_slots, local_pos, input_ids = [], [], []
    for k, seq in enumerate(sequences):
        for j in range(drafts + 1):
            row_slots.append(k)
            local_pos.append(j)
            input_ids.append(seq["tokens"][committed + j - 1] if committed + j > 0 else 0)
    return row_slots, local_pos, input_ids


def test_noalloc_draft_rows_equal_the_allocating_entry_point():
    import torch

    case = next(c for c in golden_walks() if c["name"] == "bpe_committed")
    sequences = case["sequences"]
    engine, served = _engine(case)
    engine.reset()
    engine.begin(torch.arange(len(sequences), dtype=torch.int32, device="cuda"))
    allocating, noalloc = _entry_points(engine)
    as_t = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")  # noqa: E731
    gen = torch.Generator(device="cuda").manual_seed(21)
    done = 0
    for committed in (9, 40):  # two calls in a row, from two different committed states
        for step in range(done, committed):
            engine.advance(np.array([seq["tokens"][step] for seq in sequences], dtype=np.int32))
        done = committed
        row_slots, local_pos, input_ids = (as_t(v) for v in _blocks(sequences, committed, 4))
        logits = torch.randn((len(row_slots), served.vocab_size + 3), generator=gen, device="cuda")
        want, got = logits.clone(), logits.clone()
        assert _call(allocating, engine, want, row_slots, local_pos, input_ids) == XG_OK
        assert _call(noalloc, engine, got, row_slots, local_pos, input_ids) == XG_OK
        torch.cuda.synchronize()
        assert torch.equal(want.view(torch.int32), got.view(torch.int32)), committed
        assert torch.isneginf(got).any() and not torch.equal(got, logits)


def test_noalloc_rejects_more_rows_than_its_scratch_holds():
    import torch

    case = next(c for c in golden_walks() if c["name"] == "bpe_committed")
    engine, served = _engine(case)
    _, noalloc = _entry_points(engine)
    # each row needs more than its mask's 4 * words bytes, so this many rows exceed 8 MiB
    rows = (8 << 20) // (4 * engine.words) + 1
    logits = torch.zeros((rows, served.vocab_size), device="cuda")
    zeros = torch.zeros(rows, dtype=torch.int32, device="cuda")
    assert _call(noalloc, engine, logits, zeros, zeros, zeros) == XG_EINVAL
    message = engine._lib.xg_last_error().decode()
    assert "scratch" in message and "xg_apply_mask" in message, message
    torch.cuda.synchronize()
    assert not logits.any()  # nothing was launched
