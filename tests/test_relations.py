"""The weaker relation supports, relations="vocabulary" / "successor" (the reference's
src/xgraph/oracle.py:67-79, 865-878, 1060-1078, 1138-1147, 1599-1605, 1809-1822;
src/xgraph/relations.py; csrc/engine.cu:618-670, 1549-1552, 1779-1781, 1873-1900).

The fixture (tests/golden/make_relation_cases.py) holds walks of the reference Oracle in
path mode with committed paths under either support, with every state and allowed set, on
four golden worlds (two with KG versions).  CPU: the successor tables equal the oracle's
sets; the oracle reproduces every walk; the engine's per-row logic (core.cuh, host seam)
reproduces every walk.  GPU: the engine through the C ABI reproduces every walk, by advance
+ fill_mask and by the fused step."""

from __future__ import annotations

import gzip
import json
from functools import cache

import numpy as np
import pytest

from tests.conftest import GOLDEN, state_record, unpack, world, world_index


@cache
def relation_cases():
    with gzip.open(GOLDEN / "relation_cases.json.gz", "rt", encoding="utf-8") as f:
        return json.load(f)["cases"]


def edits_of(case) -> dict | None:
    return {k: [tuple(e) for e in v] for k, v in case["versions"].items()} or None


def make_oracle(case):
    from oracle.oracle import Oracle
    from xgraph_b200.syntax import SpanSyntax

    _, served, _ = world(case["world"])
    return Oracle(world_index(case["world"], False), served, SpanSyntax(), paths=True, committed_paths=True,
                  relations=case["mode"], versions=edits_of(case))


def test_oracle_reproduces_the_relation_walks():
    """Every state and allowed set of every walk; the walks close plans and take
    separators between relations."""
    plans = separated = 0
    for case in relation_cases():
        oracle = make_oracle(case)
        for n, w in enumerate(case["walks"]):
            state = oracle.initial_state(w["version"])
            for k, token in enumerate(w["tokens"]):
                where = (case["world"], case["mode"], n, k)
                assert state_record(state) == w["states"][k], where
                assert sorted(oracle.allowed(state)) == w["allowed"][k], where
                plans += bool(state.last_span is not None and not state.last_span.resolved and state.last_span.labels)
                separated += state.segment.value == "relation" and len(state.written) > 1
                state = oracle.advance(state, token)
            assert state_record(state) == w["final"]
            assert sorted(oracle.allowed(state)) == w["final_allowed"]
    assert plans > 100 and separated > 20, (plans, separated)


def test_successor_tables_equal_the_oracle_sets():
    """xgraph_b200.relations.relation_successors, per version, against the oracle's
    successor sets (src/xgraph/relations.py:31-60 semantics)."""
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.relations import relation_successors

    for case in relation_cases():
        if case["mode"] != "successor":
            continue
        index = world_index(case["world"], False)
        edits = edits_of(case)
        versions = build_kg_versions(index, edits) if edits else None
        tables = relation_successors(index, versions)
        oracle = make_oracle(case)
        owners = index.relations.owner_ids
        for v, name in enumerate([None, *(versions.names if versions else [])]):
            want = oracle._successors[name]
            for r1, relation in enumerate(owners):
                bits = np.unpackbits(tables[v, r1].view(np.uint8), bitorder="little")[: len(owners)]
                got = {owners[r2] for r2 in np.flatnonzero(bits)}
                assert got == want.get(relation, set()), (case["world"], name, relation)


def test_weaker_relations_need_path_mode_without_stop():
    from oracle.oracle import Oracle
    from xgraph_b200.syntax import SpanSyntax

    _, served, _ = world("toy")
    index = world_index("toy", False)
    with pytest.raises(ValueError, match="path mode"):
        Oracle(index, served, SpanSyntax(), relations="vocabulary")
    with pytest.raises(ValueError, match="unknown relations"):
        Oracle(index, served, SpanSyntax(), paths=True, relations="other")


def replay(engine, served, index, syntax, case, walk, fused: bool):
    """Drive one walk through slot 0 of the engine (advance + fill_mask, or one fused step
    per token); check every mask and state projection."""
    import torch

    from tests.agreement import assert_agrees, engine_state, expected_state

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
        where = (case["world"], case["mode"], walk["version"], k, "fused" if fused else "advance")
        if fused:
            logits = torch.zeros((1, vocab), dtype=torch.float32, device="cuda")
            engine.sync_apply(slots, tokens, prompt, torch.full((1,), k, dtype=torch.int32, device="cuda"), logits)
            kept = set(np.flatnonzero(~torch.isneginf(logits[0]).cpu().numpy()).tolist())
            assert sorted(kept) == allowed, where
        else:
            engine.fill_mask(1)
            assert sorted(unpack(engine.mask_host(1)[0], vocab)) == allowed, where
        assert_agrees(expected_state(record, index, syntax), engine_state(engine.states_host(1), 0, view), True, where)
        if not fused and k < len(walk["tokens"]):
            engine.advance(np.array([walk["tokens"][k]], dtype=np.int32))


def test_seam_reproduces_the_relation_walks():
    """The kernels' per-row logic (core.cuh on the host): every mask and state projection
    of every walk."""
    from tests.agreement import assert_agrees, engine_state, expected_state
    from tests.seam import SeamEngine
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.syntax import SpanSyntax

    syntax = SpanSyntax()
    for case in relation_cases():
        _, served, _ = world(case["world"])
        index = world_index(case["world"], False)
        edits = edits_of(case)
        versions = build_kg_versions(index, edits) if edits else None
        seam = SeamEngine(index, served, syntax, 1, paths=True, committed_paths=True, versions=versions,
                          relations=case["mode"])
        for n, w in enumerate(case["walks"]):
            seam.begin(0)
            seam.set_version(0, w["version"])
            view = seam.view(w["version"])
            for k in range(len(w["tokens"]) + 1):
                record = w["states"][k] if k < len(w["tokens"]) else w["final"]
                allowed = w["allowed"][k] if k < len(w["tokens"]) else w["final_allowed"]
                where = (case["world"], case["mode"], n, k)
                assert sorted(unpack(seam.masks()[0], served.vocab_size)) == allowed, where
                assert_agrees(expected_state(record, index, syntax), engine_state(seam.states(), 0, view), True, where)
                if k < len(w["tokens"]):
                    seam.advance([w["tokens"][k]])


@pytest.mark.gpu
def test_engine_reproduces_the_relation_walks():
    """The CUDA engine through the C ABI: every walk by advance + fill_mask and by the fused
    step, masks and state projections at every step."""
    from xgraph_b200.engine import Engine
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.syntax import SpanSyntax

    syntax = SpanSyntax()
    for case in relation_cases():
        _, served, _ = world(case["world"])
        index = world_index(case["world"], False)
        edits = edits_of(case)
        versions = build_kg_versions(index, edits) if edits else None
        engine = Engine(index, served, syntax, 1, paths=True, committed_paths=True, versions=versions,
                        relations=case["mode"])
        for w in case["walks"]:
            replay(engine, served, index, syntax, case, w, fused=False)
            replay(engine, served, index, syntax, case, w, fused=True)
        assert engine.faults() == 0


@pytest.mark.gpu
def test_engine_refuses_weaker_relations_without_path_mode():
    from xgraph_b200.engine import Engine
    from xgraph_b200.syntax import SpanSyntax

    _, served, _ = world("toy")
    index = world_index("toy", False)
    with pytest.raises(ValueError, match="path mode"):
        Engine(index, served, SpanSyntax(), 1, relations="successor")
    with pytest.raises(ValueError, match="STOP"):
        Engine(index, served, SpanSyntax(), 1, paths=True, committed_paths=True, relations="vocabulary",
               stop="residual-goal")
    engine = Engine(index, served, SpanSyntax(), 1, paths=True, committed_paths=True, relations="successor")
    with pytest.raises(ValueError, match="successor"):
        engine.add_version("late", [])
