"""The engine's per-row logic, compiled for the host (test seam), against the golden walks.

Every golden walk is replayed through the seam: at every step its mask must equal the
reference Oracle's allowed set and its state must agree with the reference state's
public projection (the reference's agreement contract, tests/test_engine.py:1733-2002).
"""

from __future__ import annotations

import pytest

from tests.agreement import assert_agrees, engine_state, expected_state
from tests.conftest import case_index, case_options, case_versions, golden_masks, golden_walks, unpack, world

CASES = [case["name"] for case in golden_walks()]


def seam_for(case):
    from tests.seam import SeamEngine
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.syntax import SpanSyntax

    _, served, _ = world(case["world"])
    index = case_index(case)
    edits = case_versions(case)
    versions = build_kg_versions(index, edits) if edits else None
    options = case_options(case)
    return SeamEngine(index, served, SpanSyntax(), len(case["sequences"]), versions=versions, **options), index


@pytest.mark.parametrize("name", CASES)
def test_seam_agrees_with_reference_walks(name):
    from xgraph_b200.syntax import SpanSyntax

    case = next(c for c in golden_walks() if c["name"] == name)
    engine, index = seam_for(case)
    syntax = SpanSyntax()
    vocab = world(case["world"])[1].vocab_size
    sequences = case["sequences"]
    for k, seq in enumerate(sequences):
        engine.begin(k)
        engine.set_version(k, seq["version"])
        if seq["anchor"]:
            engine.anchor(k, seq["anchor"])
        if seq["opened"]:
            engine.open_span(k)
    steps = len(sequences[0]["tokens"])
    paths = case["options"].get("paths", False)
    for step in range(steps + 1):
        masks = engine.masks()
        states = engine.states()
        for k, seq in enumerate(sequences):
            record = seq["states"][step] if step < steps else seq["final"]
            where = (name, k, step)
            expected = expected_state(record, index, syntax)
            got = engine_state(states, k, engine.view(seq["version"]))
            assert_agrees(expected, got, paths, where)
            if step < steps:
                assert unpack(masks[k], vocab) == unpack(golden_masks()[f"{name}/{k}"][step], vocab), where
        if step < steps:
            engine.advance([seq["tokens"][step] for seq in sequences])
