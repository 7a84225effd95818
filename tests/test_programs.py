"""Offline path execution (xgraph_b200/programs.py) against the reference's MatchedExecutor.

tests/golden/matched_cases.json.gz (tests/golden/make_matched_cases.py) holds 704 written
paths over four golden worlds and four executor settings, with what the reference's
MatchedExecutor (src/xgraph/programs.py:368-1130) made of each: entities reached in
best-connected order, answer, plan.  The GPU executor runs each world's paths as batches
of engine slots and must return the same three fields for every path.
"""

from __future__ import annotations

import gzip
import json
from collections import defaultdict
from functools import cache

import pytest

from tests.conftest import GOLDEN, world, world_index

MAX_PATH_RELATIONS = 8


@cache
def fixture() -> dict:
    with gzip.open(GOLDEN / "matched_cases.json.gz", "rt", encoding="utf-8") as f:
        return json.load(f)


def test_matched_fixture_covers_the_cases():
    """The recorded paths hold every kind the generator writes: reaching several entities,
    reaching nothing, entity spans, and walks cut at the 8-relation cap; and the reference's
    plan is the start and the (capped) relations exactly where a path reaches something."""
    cases = fixture()["cases"]
    assert len(cases) == 704
    assert sum(1 for c in cases if len(c["reached"]) > 1) > 100
    assert sum(1 for c in cases if not c["reached"]) > 100
    assert any(not c["relations"] and c["reached"] for c in cases)
    assert any(len(c["relations"]) > MAX_PATH_RELATIONS and c["reached"] for c in cases)
    for c in cases:
        if c["reached"] and c["relations"]:
            assert c["plan"] == [c["start"], *c["relations"][:MAX_PATH_RELATIONS]]
            assert c["answer"] in c["reached"]
        else:
            assert c["plan"] is None


def _executor(world_name: str, setting: str, max_paths: int = 256):
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.programs import MatchedExecutor

    data = fixture()
    _, served, _ = world(world_name)
    index = world_index(world_name, True)
    edits = {name: [tuple(e) for e in v] for name, v in data["edits"][world_name].items()}
    versions = build_kg_versions(index, edits)
    return MatchedExecutor(index, served, versions=versions, max_paths=max_paths, **data["settings"][setting])


@pytest.mark.gpu
def test_matched_execution_equals_the_reference():
    """Every recorded path, executed on the GPU a world and setting at a time, reaches the
    reference's entities in its order, delivers its answer and reports its plan."""
    groups = defaultdict(list)
    for case in fixture()["cases"]:
        groups[(case["world"], case["setting"])].append(case)
    for (world_name, setting), cases in groups.items():
        executor = _executor(world_name, setting)
        got = executor.execute_many([(c["start"], c["relations"], c["version"]) for c in cases])
        for case, path in zip(cases, got, strict=True):
            where = (world_name, setting, case["start"], case["relations"], case["version"])
            assert list(path.reached) == case["reached"], where
            assert path.answer == case["answer"], where
            assert (None if path.plan is None else list(path.plan)) == case["plan"], where


@pytest.mark.gpu
def test_matched_execution_in_small_batches_and_single_calls():
    """A batch larger than the executor's slots runs in pieces with the same results, and
    `execute` (one path) agrees with the batch."""
    cases = [c for c in fixture()["cases"] if c["world"] == "rand_bpe" and c["setting"] == "committed"]
    executor = _executor("rand_bpe", "committed", max_paths=7)
    got = executor.execute_many([(c["start"], c["relations"], c["version"]) for c in cases])
    assert [list(p.reached) for p in got] == [c["reached"] for c in cases]
    for case in cases[:5]:
        one = executor.execute(case["start"], case["relations"], version=case["version"])
        assert list(one.reached) == case["reached"] and one.answer == case["answer"]


@pytest.mark.gpu
def test_matched_executor_refuses_what_it_does_not_serve():
    executor = _executor("toy", "committed", max_paths=2)
    with pytest.raises(ValueError, match="anchored"):
        executor.execute("Paris Hilton", ["place of birth"], anchor=["Q5"])
    with pytest.raises(ValueError, match="repair"):
        executor.execute("Paris Hilton", ["place of birth"], repair=True)
    with pytest.raises(ValueError, match="no KG version"):
        executor.execute("Paris Hilton", ["place of birth"], version="v9")
    from xgraph_b200.programs import MatchedExecutor

    _, served, _ = world("toy")
    with pytest.raises(ValueError, match="strip_quotes"):
        MatchedExecutor(world_index("toy", True), served, strip_quotes=True)
