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
