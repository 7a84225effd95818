"""Engine/oracle agreement: the public state projection both sides must share.

Restates the reference's agreement harness (tests/test_engine.py:1588-1730:
allowed_from_mask, expected_state, engine_state, assert_agrees) over this repository's
oracle state records (tests/conftest.py state_record) and engine state arrays.
"""

from __future__ import annotations

from xgraph_b200.engine import SEGMENTS, closed_span

CODES = {"free text": 0, "span": 1, "escaped": 2}


def partial_match(tail: bytes, delimiter: bytes) -> int:
    return max(k for k in range(len(delimiter)) if tail.endswith(delimiter[:k]))


def last_span(record) -> tuple | None:
    closed = record["last_span"]
    if closed is None:
        return None
    if closed.get("operator"):  # a comparison: its result (the operands are checked apart)
        return ("comparison", tuple(closed["entity_ids"]), ())
    if not closed["resolved"]:  # an escape (no labels) or a plan under a weaker relation support
        return ("relation plan" if closed["labels"] else "unresolved", (), ())
    if not closed["triples"] and len(closed["labels"]) > 1:
        return ("path span", (), ())  # the engine records no path endpoints
    kind = "fact span" if closed["triples"] else "entity span"
    return (kind, tuple(closed["entity_ids"]), tuple(tuple(t) for t in closed["triples"]))


def expected_state(record: dict, index, syntax) -> dict:
    fields = {
        "phase": CODES[record["phase"]],
        "last": last_span(record),
        "resolved": record["last_span"] is not None and record["last_span"]["resolved"],
        "answer_complete": record["answer_complete"],
    }
    tail = bytes.fromhex(record["tail"])
    if record["phase"] == "span":
        fields["segment"] = SEGMENTS.index(record["segment"])
        rows = index.relations if record["segment"] == "relation" else index.labels
        typed = record["typed"]
        fields["range"] = None if typed is None else rows.prefix_range(typed)
        fields["depth"] = None if typed is None else len(typed)
        for name, key in (("close_pos", "closing"), ("sep_pos", "separating"), ("esc_pos", "escaping")):
            fields[name] = len(bytes.fromhex(record[key])) if record[key] else 0
        fields["subjects"] = set(record["subjects"])
        fields["relations"] = set(record["relations"])
    elif record["phase"] == "free text":
        fields["pos"] = partial_match(tail, syntax.opener.encode("utf-8"))
    else:
        fields["pos"] = partial_match(tail, syntax.closer.encode("utf-8"))
    return fields


def engine_state(states: dict, seq: int, view) -> dict:
    field = {name: int(values[seq]) for name, values in states.items()}
    subjects = {
        view.labels.owner_id(r)
        for r in range(field["subj_lo"], field["subj_hi"])
        if view.relations_of(view.labels.owner_id(r))
    }
    relations = {
        view.relations.owner_id(r)
        for r in range(field["rel_lo"], field["rel_hi"])
        if any(view.relations.owner_id(r) in view.relations_of(s) for s in subjects)
    }
    closed = closed_span(view, states, seq)
    return {
        **field,
        "subjects": subjects,
        "relations": relations,
        "last": None if closed.kind == "none" else (closed.kind, closed.entity_ids, closed.triples),
        "resolved": closed.resolved,
    }


def assert_agrees(expected: dict, got: dict, frontier: bool, where=()) -> None:
    assert got["phase"] == expected["phase"], (where, "phase", got["phase"], expected["phase"])
    assert got["resolved"] == expected["resolved"], (where, "resolved")
    assert bool(got["answer_complete"]) == expected["answer_complete"], (where, "answer_complete")
    if expected["phase"] == 1:
        assert got["segment"] == expected["segment"], (where, "segment")
        if expected["range"] is None:
            assert got["lo"] < 0, (where, "dead label", got["lo"])
        else:
            assert (got["lo"], got["hi"]) == expected["range"], (where, "range", (got["lo"], got["hi"]), expected["range"])
            assert got["depth"] == expected["depth"], (where, "depth")
        for name in ("close_pos", "sep_pos", "esc_pos"):
            assert got[name] == expected[name], (where, name, got[name], expected[name])
        if expected["segment"] != 0 and not frontier:
            assert got["subjects"] == expected["subjects"], (where, "subjects", got["subjects"], expected["subjects"])
        if expected["segment"] == 2:
            assert got["relations"] == expected["relations"], (where, "relations")
    else:
        assert got["pos"] == expected["pos"], (where, "pos", got["pos"], expected["pos"])
    assert got["last"] == expected["last"], (where, "last", got["last"], expected["last"])
