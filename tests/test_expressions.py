"""Expressions: date and value comparisons (the reference's src/xgraph/oracle.py:104-133,
1048-1130, 1669-1737, 1830-1905; csrc/engine.cu:547-611, 988-1125, 1777-1935, 2245-2250).

The fixture (tests/golden/make_expression_cases.py) holds walks of the reference Oracle in
path mode with committed paths and expressions on, with every state and allowed set, on
four golden worlds with seeded date tables (three of them with the verdict entities, two
with KG versions).  CPU: the index's date table and verdicts; the oracle reproduces every
walk; the engine's per-row logic (core.cuh, host seam) reproduces every walk.  The same
walks through the CUDA engine: tests/test_z_expressions_gpu.py."""

from __future__ import annotations

import gzip
import json
from functools import cache

import pytest

from tests.conftest import GOLDEN, state_record, world


@cache
def expression_cases():
    with gzip.open(GOLDEN / "expression_cases.json.gz", "rt", encoding="utf-8") as f:
        return json.load(f)["cases"]


def expression_record(state) -> dict:
    """state_record plus the expression fields (as the fixture records them)."""
    record = state_record(state)
    record["operating"] = None if state.operating is None else state.operating.hex()
    record["operator"] = state.operator
    record["starts"] = [list(s) for s in state.starts]
    record["ranks_b"] = sorted([list(x) for x in state.ranks_b])
    if state.last_span is not None:
        record["last_span"]["operator"] = state.last_span.operator
        record["last_span"]["operands"] = list(state.last_span.operands)
    return record


@cache
def dated_index(world_name: str):
    from xgraph_b200.dates import Date
    from xgraph_b200.index import build_kg_index
    from xgraph_b200.syntax import SpanSyntax

    case = next(c for c in expression_cases() if c["world"] == world_name)
    kg, served, _ = world(world_name)
    dates = {e: Date(*d) for e, d in case["dates"].items()}
    return build_kg_index(kg, served, SpanSyntax(), dates=dates, verdicts=case["verdicts"])


def edits_of(case) -> dict | None:
    return {k: [tuple(e) for e in v] for k, v in case["versions"].items()} or None


def make_oracle(case):
    from oracle.oracle import Oracle
    from xgraph_b200.syntax import SpanSyntax

    _, served, _ = world(case["world"])
    return Oracle(dated_index(case["world"]), served, SpanSyntax(), paths=True, committed_paths=True,
                  expressions=True, versions=edits_of(case))


def test_date_keys_and_bounds():
    """Keys sort by year, month, day, precision; bounds compare as Date.lo / Date.hi do."""
    from xgraph_b200.dates import Date, date_hi, date_lo, pack_date, unpack_date

    dates = [Date(1890), Date(1890, 1, 1, "year"), Date(1890, 3), Date(1890, 3, 4), Date(-44, 3, 15),
             Date(1890, 12, 31)]
    for d in dates:
        assert unpack_date(pack_date(d)) == d
    for a in dates:
        for b in dates:
            lo_b, hi_a = date_lo([pack_date(b)])[0], date_hi([pack_date(a)])[0]
            assert (hi_a < lo_b) == a.before(b), (a, b)
    assert sorted(dates, key=pack_date) == sorted(dates, key=lambda d: (d.year, d.month or 0, d.day or 0))


def test_index_holds_the_date_table_and_the_verdicts():
    from xgraph_b200.dates import VERDICTS, pack_date, Date
    from xgraph_b200.index import load_kg_index, save_kg_index

    for case in expression_cases():
        index = dated_index(case["world"])
        ids = index.labels.owner_ids
        assert [ids[e] for e in index.date_entities] == sorted(case["dates"], key=ids.index)
        assert [int(k) for k in index.date_keys] == [pack_date(Date(*case["dates"][ids[e]]))
                                                     for e in index.date_entities]
        if case["verdicts"]:
            assert index.verdicts == VERDICTS and tuple(ids[-2:]) == tuple(VERDICTS.values())
        else:
            assert index.verdicts is None
    import tempfile

    index = dated_index("toy")
    with tempfile.TemporaryDirectory() as tmp:
        save_kg_index(index, tmp)
        again = load_kg_index(tmp)
    assert again.verdicts == index.verdicts and again.base_fingerprint == index.base_fingerprint
    assert (again.date_entities == index.date_entities).all() and (again.date_keys == index.date_keys).all()


def test_fixture_covers_comparisons():
    """Walks close date comparisons with one and with two (undetermined) results, value
    comparisons with either verdict, and answer spans bound to a comparison's result."""
    closed = set()
    answered = 0
    for case in expression_cases():
        for w in case["walks"]:
            for s in [*w["states"], w["final"]]:
                span = s["last_span"]
                if span and span.get("operator"):
                    closed.add((span["operator"], tuple(span["entity_ids"]) if span["operator"] == "same"
                                else len(span["entity_ids"])))
                    answered += s["phase"] == "span"
    assert {("earlier", 1), ("earlier", 2), ("later", 1)} <= closed, closed
    assert any(op == "same" for op, _ in closed), closed
    assert answered > 5


def test_oracle_reproduces_the_expression_walks():
    for case in expression_cases():
        oracle = make_oracle(case)
        for n, w in enumerate(case["walks"]):
            state = oracle.initial_state(w["version"])
            for k, token in enumerate(w["tokens"]):
                where = (case["world"], n, k)
                assert expression_record(state) == w["states"][k], where
                assert sorted(oracle.allowed(state)) == w["allowed"][k], where
                state = oracle.advance(state, token)
            assert expression_record(state) == w["final"]
            assert sorted(oracle.allowed(state)) == w["final_allowed"]


def test_expressions_need_committed_paths_and_escapes():
    from oracle.oracle import Oracle
    from xgraph_b200.syntax import SpanSyntax

    _, served, _ = world("toy")
    index = dated_index("toy")
    with pytest.raises(ValueError, match="committed paths"):
        Oracle(index, served, SpanSyntax(), paths=True, expressions=True)
    with pytest.raises(ValueError, match="escapes"):
        Oracle(index, served, SpanSyntax(), paths=True, committed_paths=True, escapes=False, expressions=True)
    from tests.conftest import world_index

    with pytest.raises(ValueError, match="date table"):
        Oracle(world_index("toy", False), served, SpanSyntax(), paths=True, committed_paths=True, expressions=True)


def check_operator_fields(record: dict, states: dict, slot: int, view, where) -> None:
    """The expression fields the agreement projection leaves out: the operator branch's
    byte position, the span's operator, and a closed comparison's operands."""
    from xgraph_b200.engine import closed_span

    if record["phase"] == "span":
        operating = bytes.fromhex(record["operating"]) if record["operating"] else b""
        assert int(states["op_pos"][slot]) == len(operating), (where, "op_pos")
        assert int(states["op"][slot]) == record["operator"], (where, "op")
    span = record["last_span"]
    if span and span.get("operator"):
        closed = closed_span(view, states, slot)
        assert (closed.operator, closed.operands) == (span["operator"], tuple(span["operands"])), where


def test_seam_reproduces_the_expression_walks():
    """The kernels' per-row logic (core.cuh on the host): every mask, state projection and
    expression field of every walk."""
    from tests.agreement import assert_agrees, engine_state, expected_state
    from tests.conftest import unpack
    from tests.seam import SeamEngine
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.syntax import SpanSyntax

    syntax = SpanSyntax()
    for case in expression_cases():
        _, served, _ = world(case["world"])
        index = dated_index(case["world"])
        edits = edits_of(case)
        versions = build_kg_versions(index, edits) if edits else None
        seam = SeamEngine(index, served, syntax, 1, paths=True, committed_paths=True, versions=versions,
                          expressions=True)
        for n, w in enumerate(case["walks"]):
            seam.begin(0)
            seam.set_version(0, w["version"])
            view = seam.view(w["version"])
            for k in range(len(w["tokens"]) + 1):
                record = w["states"][k] if k < len(w["tokens"]) else w["final"]
                allowed = w["allowed"][k] if k < len(w["tokens"]) else w["final_allowed"]
                where = (case["world"], n, k)
                assert sorted(unpack(seam.masks()[0], served.vocab_size)) == allowed, where
                states = seam.states()
                assert_agrees(expected_state(record, index, syntax), engine_state(states, 0, view), True, where)
                check_operator_fields(record, states, 0, view, where)
                if k < len(w["tokens"]):
                    seam.advance([w["tokens"][k]])


def test_engine_refuses_expressions_without_their_needs():
    """The Engine's checks run before any device call (CPU): committed paths, escapes, the
    date table, frontier support."""
    from tests.conftest import world_index
    from xgraph_b200.engine import Engine
    from xgraph_b200.syntax import SpanSyntax

    _, served, _ = world("toy")
    index = dated_index("toy")
    with pytest.raises(ValueError, match="committed paths"):
        Engine(index, served, SpanSyntax(), 1, paths=True, expressions=True)
    with pytest.raises(ValueError, match="escapes"):
        Engine(index, served, SpanSyntax(), 1, paths=True, committed_paths=True, escapes=False, expressions=True)
    with pytest.raises(ValueError, match="date table"):
        Engine(world_index("toy", False), served, SpanSyntax(), 1, paths=True, committed_paths=True,
               expressions=True)
    with pytest.raises(ValueError, match="expressions"):
        Engine(index, served, SpanSyntax(), 1, paths=True, committed_paths=True, expressions=True,
               relations="vocabulary")


def test_seam_refuses_malformed_expression_tables():
    """xg_set_expressions' table checks (parse_packed_delims, shared with the host seam):
    the packed lists must parse exactly, tokens lie in the vocabulary and ascend per byte
    position, next positions stay inside the delimiter; the third operator needs the
    verdict entities."""
    import ctypes

    import numpy as np

    from tests.seam import SeamEngine
    from xgraph_b200.syntax import SpanSyntax

    _, served, _ = world("toy")
    seam = SeamEngine(dated_index("toy"), served, SpanSyntax(), 1, paths=True, committed_paths=True,
                      expressions=True)
    delims, operators, lcp, entities, keys, verdicts = seam._expr

    def call(d, ops=operators, v=verdicts):
        d = np.ascontiguousarray(d, dtype=np.int32)
        ptr = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
        return seam.lib.xgs_set_expressions(seam.handle, ptr(d), len(d), ops, ptr(lcp), ptr(entities), ptr(keys),
                                            len(entities), ptr(v))

    assert call(delims) == 0
    assert call(delims[:-1]) == 1                      # cut short
    assert call(np.concatenate([delims, [0]])) == 1    # not used up
    bad = delims.copy()
    bad[0] = 0                                         # a delimiter of no bytes
    assert call(bad) == 1
    n = int(delims[1 + delims[0]])                     # the operand separator's token count
    bad = delims.copy()
    bad[2 + delims[0]] = served.vocab_size             # a token outside the vocabulary
    assert call(bad) == 1
    bad = delims.copy()
    bad[2 + delims[0] + n] = int(delims[0]) + 1        # a next position past the delimiter
    assert call(bad) == 1
    assert call(delims, v=None) == 1                   # the value comparison without verdicts
