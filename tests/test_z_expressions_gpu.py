"""Expressions on the GPU: the CUDA engine through the C ABI reproduces every reference
walk of tests/golden/expression_cases.json.gz (date and value comparisons; see
tests/test_expressions.py for the fixture and the CPU checks), by advance + fill_mask and by
the fused step.  Collected after the other GPU tests of the engine's established
policies."""

from __future__ import annotations

import pytest

from tests.conftest import world
from tests.test_expressions import check_operator_fields, dated_index, edits_of, expression_cases


def replay(engine, served, index, syntax, case, n, walk, fused: bool):
    """Drive one walk through slot 0 of the engine (advance + fill_mask, or one fused step
    per token); check every mask, state projection and expression field."""
    import numpy as np
    import torch

    from tests.agreement import assert_agrees, engine_state, expected_state
    from tests.conftest import unpack

    vocab = served.vocab_size
    engine.begin(torch.zeros(1, dtype=torch.int32, device="cuda"))
    if walk["version"] is not None:
        engine.set_version(0, walk["version"])
    tokens = torch.tensor([walk["tokens"]], dtype=torch.int32, device="cuda")
    slots = torch.zeros(1, dtype=torch.int32, device="cuda")
    prompt = torch.zeros(1, dtype=torch.int32, device="cuda")
    view = engine.view(walk["version"])
    for k in range(len(walk["tokens"]) + 1):
        record = walk["states"][k] if k < len(walk["tokens"]) else walk["final"]
        allowed = walk["allowed"][k] if k < len(walk["tokens"]) else walk["final_allowed"]
        where = (case["world"], n, k, "fused" if fused else "advance")
        if fused:
            logits = torch.zeros((1, vocab), dtype=torch.float32, device="cuda")
            engine.sync_apply(slots, tokens, prompt, torch.full((1,), k, dtype=torch.int32, device="cuda"), logits)
            kept = set(np.flatnonzero(~torch.isneginf(logits[0]).cpu().numpy()).tolist())
            assert sorted(kept) == allowed, where
        else:
            engine.fill_mask(1)
            assert sorted(unpack(engine.mask_host(1)[0], vocab)) == allowed, where
        states = engine.states_host(1)
        assert_agrees(expected_state(record, index, syntax), engine_state(states, 0, view), True, where)
        check_operator_fields(record, states, 0, view, where)
        if not fused and k < len(walk["tokens"]):
            engine.advance(np.array([walk["tokens"][k]], dtype=np.int32))


@pytest.mark.gpu
def test_engine_reproduces_the_expression_walks():
    """The CUDA engine through the C ABI: every walk by advance + fill_mask and by the fused
    step, masks, state projections and expression fields at every step."""
    from xgraph_b200.engine import Engine
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.syntax import SpanSyntax

    syntax = SpanSyntax()
    for case in expression_cases():
        _, served, _ = world(case["world"])
        index = dated_index(case["world"])
        edits = edits_of(case)
        versions = build_kg_versions(index, edits) if edits else None
        engine = Engine(index, served, syntax, 1, paths=True, committed_paths=True, versions=versions,
                        expressions=True)
        for n, w in enumerate(case["walks"]):
            replay(engine, served, index, syntax, case, n, w, fused=False)
            replay(engine, served, index, syntax, case, n, w, fused=True)
        assert engine.faults() == 0
