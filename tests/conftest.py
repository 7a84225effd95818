"""Shared fixtures: the golden worlds and walks made from the reference implementation."""

from __future__ import annotations

import gzip
import json
import sys
from functools import cache
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built engine library")


@cache
def golden_worlds() -> dict:
    with gzip.open(GOLDEN / "worlds.json.gz", "rt", encoding="utf-8") as f:
        return json.load(f)


@cache
def golden_walks() -> list[dict]:
    with gzip.open(GOLDEN / "walks.json.gz", "rt", encoding="utf-8") as f:
        return json.load(f)


@cache
def golden_masks():
    return np.load(GOLDEN / "masks.npz")


@cache
def golden_index():
    return np.load(GOLDEN / "index.npz")


@cache
def world(name: str):
    """(KnowledgeGraph, ServedTokenizer, sitelinks) of a golden world."""
    from tokenizers import Tokenizer

    from xgraph_b200.kg import Entity, KnowledgeGraph, Relation
    from xgraph_b200.tokenizer import ServedTokenizer

    w = golden_worlds()[name]
    kg = KnowledgeGraph(
        tuple(Entity(i, tuple(ls)) for i, ls in w["entities"]),
        tuple(Relation(i, tuple(ls)) for i, ls in w["relations"]),
        tuple(tuple(t) for t in w["triples"]),
    )
    return kg, ServedTokenizer(Tokenizer.from_str(w["tokenizer"])), w["sitelinks"]


@cache
def world_index(name: str, with_sitelinks: bool):
    from xgraph_b200.index import build_kg_index
    from xgraph_b200.syntax import SpanSyntax

    kg, served, sitelinks = world(name)
    return build_kg_index(kg, served, SpanSyntax(), sitelinks=sitelinks if with_sitelinks else None)


def case_options(case: dict) -> dict:
    return dict(case["options"])


def case_index(case: dict):
    return world_index(case["world"], case["options"].get("start_rank") == "sitelinks")


def case_versions(case: dict):
    if not case["versions"]:
        return None
    return {k: [tuple(e) for e in v] for k, v in case["versions"].items()}


def unpack(words: np.ndarray, vocab: int) -> set[int]:
    bits = np.unpackbits(np.ascontiguousarray(words, dtype=np.uint32).view(np.uint8), bitorder="little")
    return {int(t) for t in np.flatnonzero(bits[:vocab])}


@pytest.fixture(scope="session")
def walks():
    return golden_walks()


def state_record(state) -> dict:
    """An oracle state as the golden walks record it (every in-scope field, JSON-shaped)."""

    def hexed(b):
        return None if b is None else b.hex()

    def closed(span):
        if span is None:
            return None
        return {
            "labels": [list(x) for x in span.labels], "entity_ids": list(span.entity_ids),
            "triples": [list(t) for t in span.triples], "resolved": span.resolved,
        }

    return {
        "phase": state.phase.value, "tail": state.tail.hex(), "segment": state.segment.value,
        "subjects": sorted(state.subjects), "relations": sorted(state.relations),
        "written": [list(x) for x in state.written],
        "typed": None if state.typed is None else list(state.typed),
        "closing": hexed(state.closing), "closing_label": list(state.closing_label),
        "separating": hexed(state.separating), "separating_label": list(state.separating_label),
        "escaping": hexed(state.escaping), "last_span": closed(state.last_span),
        "facts": [[list(x) for x in f] for f in state.facts],
        "reached": None if state.reached is None else sorted(state.reached),
        "ranks": sorted([list(x) for x in state.ranks]), "version": state.version,
        "answer_complete": state.answer_complete,
    }


def make_oracle(case: dict):
    from oracle.oracle import Oracle
    from xgraph_b200.syntax import SpanSyntax

    _, served, _ = world(case["world"])
    return Oracle(case_index(case), served, SpanSyntax(), versions=case_versions(case), **case_options(case))


def start_state(oracle, sequence: dict):
    state = (
        oracle.anchored_state(sequence["anchor"], sequence["version"])
        if sequence["anchor"]
        else oracle.initial_state(sequence["version"])
    )
    return oracle.opened_state(state) if sequence["opened"] else state
