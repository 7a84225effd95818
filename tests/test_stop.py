"""Residual-goal STOP (the reference's src/xgraph/oracle.py:1081-1111, 1608-1635,
src/xgraph/stopping.py:74-133; csrc/engine.cu:1001-1072, 1580-1583).

The fixture (tests/golden/make_stop_cases.py) holds walks of the reference Oracle under a
question each, with every state and allowed set, on three golden worlds and on the worlds
of the reference's own STOP tests, and the reference's STOP table of every question.  CPU:
the host table (xgraph_b200.stopping) equals the reference's, the oracle reproduces every
walk, and the engine's per-row logic (core.cuh, host seam) reproduces every walk.  GPU:
the engine through the C ABI reproduces every walk."""

from __future__ import annotations

import gzip
import json
from functools import cache

import numpy as np
import pytest

from tests.conftest import GOLDEN, state_record, unpack, world


@cache
def stop_cases():
    with gzip.open(GOLDEN / "stop_cases.json.gz", "rt", encoding="utf-8") as f:
        return json.load(f)["cases"]


@cache
def stop_world(name: str):
    """(index, served tokenizer, syntax) of a fixture world."""
    from tokenizers import Tokenizer

    from xgraph_b200 import Entity, KnowledgeGraph, ServedTokenizer, SpanSyntax, build_kg_index
    from xgraph_b200.kg import Relation

    case = next(c for c in stop_cases() if c["world"] == name)
    if "kg" not in case:  # a golden world
        kg, served, _ = world(name)
        return build_kg_index(kg, served, SpanSyntax()), served, SpanSyntax()
    served = ServedTokenizer(Tokenizer.from_str(case["tokenizer"]))
    syntax = SpanSyntax(**case["syntax"])
    kg = KnowledgeGraph(tuple(Entity(i, tuple(ls)) for i, ls in case["kg"]["entities"]),
                        tuple(Relation(i, tuple(ls)) for i, ls in case["kg"]["relations"]),
                        tuple(tuple(t) for t in case["kg"]["triples"]))
    return build_kg_index(kg, served, syntax), served, syntax


def stop_oracle(name: str):
    from oracle.oracle import Oracle

    index, served, syntax = stop_world(name)
    return Oracle(index, served, syntax, paths=True, committed_paths=True, stop="residual-goal")


def test_stop_tables_equal_the_reference():
    from xgraph_b200.stopping import RelationTerms

    for case in stop_cases():
        index, served, _ = stop_world(case["world"])
        terms = RelationTerms.from_index(index, served)
        for question, want in case["tables"].items():
            goal = terms.for_question(question)
            got = {"head": sorted(goal.head), "words": list(goal.words),
                   "coverage": sorted([r, m] for r, m in goal.coverage.items())}
            assert got == want, (case["world"], question)


def test_oracle_reproduces_the_stop_walks():
    """Every state and allowed set of every walk; the walks reach forced closers."""
    forced = 0
    for case in stop_cases():
        oracle = stop_oracle(case["world"])
        for w in case["walks"]:
            state = oracle.initial_state(question=w["question"])
            for k, token in enumerate(w["tokens"]):
                assert state_record(state) == w["states"][k], (case["world"], w["question"], k)
                assert sorted(oracle.allowed(state)) == w["allowed"][k], (case["world"], w["question"], k)
                if state.phase.value == "span" and state.typed is not None and oracle._context(state).forced:
                    forced += 1
                state = oracle.advance(state, token)
            assert state_record(state) == w["final"]
            assert sorted(oracle.allowed(state)) == w["final_allowed"]
    assert forced > 10, forced


def test_stop_needs_committed_paths_and_a_question():
    from oracle.oracle import Oracle

    index, served, syntax = stop_world("toy")
    with pytest.raises(ValueError, match="committed"):
        Oracle(index, served, syntax, paths=True, stop="residual-goal")
    with pytest.raises(ValueError, match="STOP"):
        Oracle(index, served, syntax, paths=True, committed_paths=True, stop="other")
    with pytest.raises(ValueError, match="question"):
        stop_oracle("toy").initial_state()


def test_seam_reproduces_the_stop_walks():
    """The kernels' per-row logic (core.cuh on the host): every mask and state projection of
    every walk, each walk in a slot begun again with its question's STOP table."""
    from tests.agreement import assert_agrees, engine_state, expected_state
    from tests.seam import SeamEngine

    for case in stop_cases():
        index, served, syntax = stop_world(case["world"])
        seam = SeamEngine(index, served, syntax, 1, paths=True, committed_paths=True)
        seam.enable_stop(served)
        for w in case["walks"]:
            seam.begin(0)
            seam.set_stop(0, w["question"])
            for k in range(len(w["tokens"]) + 1):
                record = w["states"][k] if k < len(w["tokens"]) else w["final"]
                allowed = w["allowed"][k] if k < len(w["tokens"]) else w["final_allowed"]
                where = (case["world"], w["question"], k)
                assert sorted(unpack(seam.masks()[0], served.vocab_size)) == allowed, where
                assert_agrees(expected_state(record, index, syntax), engine_state(seam.states(), 0, index), True,
                              where)
                if k < len(w["tokens"]):
                    seam.advance([w["tokens"][k]])


def test_engine_refuses_stop_without_committed_paths():
    from xgraph_b200.engine import Engine, EngineUnavailable

    index, served, syntax = stop_world("toy")
    try:
        with pytest.raises(ValueError, match="committed"):
            Engine(index, served, syntax, 1, paths=True, stop="residual-goal")
        with pytest.raises(ValueError, match="STOP"):
            Engine(index, served, syntax, 1, paths=True, committed_paths=True, stop="other")
    except EngineUnavailable:
        pytest.skip("the engine library is not built")


# ------------------------------------------------------------------------------------ GPU

@pytest.mark.gpu
@pytest.mark.parametrize("path", ["advance", "sync_apply"])
def test_engine_reproduces_the_stop_walks(path):
    """Through the C ABI: every mask and state projection of every walk (advance +
    fill_mask, or one fused sync_apply step per token with the kept columns of fp32
    logits), each walk in a slot begun again with its question's STOP table."""
    import torch

    from tests.agreement import assert_agrees, engine_state, expected_state
    from xgraph_b200.engine import Engine

    slot = torch.zeros(1, dtype=torch.int32, device="cuda")
    for case in stop_cases():
        index, served, syntax = stop_world(case["world"])
        engine = Engine(index, served, syntax, 1, paths=True, committed_paths=True, stop="residual-goal")
        vocab = served.vocab_size
        for w in case["walks"]:
            engine.begin(slot)
            engine.set_stop(0, w["question"])
            history = torch.tensor([w["tokens"]], dtype=torch.int32, device="cuda")
            zero = torch.zeros(1, dtype=torch.int32, device="cuda")
            for k in range(len(w["tokens"]) + 1):
                record = w["states"][k] if k < len(w["tokens"]) else w["final"]
                allowed = w["allowed"][k] if k < len(w["tokens"]) else w["final_allowed"]
                where = (case["world"], w["question"], k)
                if path == "sync_apply":
                    logits = torch.zeros((1, vocab), device="cuda")
                    engine.sync_apply(slot, history, zero, torch.full_like(zero, k), logits)
                    kept = torch.nonzero(~torch.isneginf(logits[0])).flatten().tolist()
                else:
                    engine.fill_mask()
                    kept = sorted(unpack(engine.mask_host().view(np.uint32)[0], vocab))
                assert kept == allowed, where
                assert_agrees(expected_state(record, index, syntax), engine_state(engine.states_host(1), 0, index),
                              True, where)
                if path == "advance" and k < len(w["tokens"]):
                    engine.advance(np.array([w["tokens"][k]], dtype=np.int32))
        assert engine.errors() == 0 and engine.faults() == 0


@pytest.mark.gpu
def test_stop_draft_rows_and_a_new_request():
    """Draft rows read the slot's STOP table in place (every prefix of a walk as one draft
    batch); the slot's next begin clears the table (its walk then masks as without STOP:
    the host seam with no table)."""
    import torch

    from tests.seam import SeamEngine
    from xgraph_b200.engine import Engine

    case = next(c for c in stop_cases() if c["world"] == "toy")
    index, served, syntax = stop_world("toy")
    engine = Engine(index, served, syntax, 1, paths=True, committed_paths=True, stop="residual-goal")
    vocab = served.vocab_size
    slot = torch.zeros(1, dtype=torch.int32, device="cuda")
    for w in case["walks"][:8]:
        engine.begin(slot)
        engine.set_stop(0, w["question"])
        tokens = w["tokens"]
        first = tokens[0]
        engine.advance(np.array([first], dtype=np.int32))  # one committed token, the rest as drafts
        rows = len(tokens)
        logits = torch.zeros((rows, vocab), device="cuda")
        local = torch.arange(rows, dtype=torch.int32, device="cuda")
        inputs = torch.tensor(tokens, dtype=torch.int32, device="cuda")
        engine.apply_mask(logits, torch.zeros(rows, dtype=torch.int32, device="cuda"), local_pos=local,
                          input_ids=inputs)
        for k in range(rows):  # row k: the state after tokens[0 .. k]
            allowed = w["allowed"][k + 1] if k + 1 < len(tokens) else w["final_allowed"]
            assert torch.nonzero(~torch.isneginf(logits[k])).flatten().tolist() == allowed, (w["question"], k)
    seam = SeamEngine(index, served, syntax, 1, paths=True, committed_paths=True)
    seam.enable_stop(served)
    w = max(case["walks"], key=lambda w: len(w["tokens"]))
    engine.begin(slot)
    engine.set_stop(0, w["question"])
    engine.begin(slot)  # a new request: no STOP table
    seam.begin(0)
    for token in w["tokens"]:
        engine.fill_mask()
        assert (engine.mask_host().view(np.uint32)[0] == seam.masks()[0]).all()
        engine.advance(np.array([token], dtype=np.int32))
        seam.advance([token])
    with pytest.raises(ValueError, match="stop"):
        Engine(index, served, syntax, 1, paths=True, committed_paths=True).set_stop(0, "Which spouse has Ada?")
    assert engine.errors() == 0 and engine.faults() == 0
