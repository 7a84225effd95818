"""Offline path execution (xgraph_b200/programs.py) against the reference's MatchedExecutor.

tests/golden/matched_cases.json.gz (tests/golden/make_matched_cases.py) holds 1157 written
paths over four golden worlds and five executor settings, 325 of them anchored, with what
the reference's MatchedExecutor (src/xgraph/programs.py:368-1130) made of each: entities
reached in best-connected order, answer, plan (or its error).  The executor runs each
world's paths as batches of engine slots and must return the same three fields for every
path it serves (and the live frontier, derivations, execute_set, repairs and stripped
starts) -- on the GPU, and on the CPU with the host seam of the kernels' row logic in place
of the CUDA engine -- and refuse what it does not serve.
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
    assert len(cases) == 1157
    assert sum(1 for c in cases if c.get("stripped")) > 40
    anchored = [c for c in cases if "anchor" in c]
    assert len(anchored) == 325 and sum(1 for c in anchored if c.get("fallback")) == 78
    assert sum(1 for c in anchored if "error" in c) == 13
    assert sum(1 for c in served(anchored) if len(c["reached"]) > 1) > 50
    assert any(not c["relations"] and c["reached"] for c in served(anchored))
    cases = served(cases)
    assert sum(1 for c in cases if len(c["frontier"]) > 1) > 200 and sum(1 for c in cases if c["frontier_relations"]) > 400
    assert sum(1 for c in cases if len(c["starts"]) > 1) > 100
    assert sum(1 for c in cases if any(n > 1 for _, n in c["derivations"])) > 20
    stages = {e["stage"] for c in cases for e in c["execute_set"]["cap_events"]}
    assert stages >= {"path_relations", "starts", "frontier", "answer_label_rows"}, stages
    assert any(c["execute_set"]["uncapped_reached"] != c["execute_set"]["reached"] for c in cases)
    assert sum(1 for c in cases if len(c["witnesses"].get("witnesses", {})) > 1) > 50
    assert sum(1 for c in cases if c["repaired"]["reached"] != c["reached"]) > 50
    assert sum(1 for c in cases if len(c["reached"]) > 1) > 100
    assert sum(1 for c in cases if not c["reached"]) > 100
    assert any(not c["relations"] and c["reached"] for c in cases)
    assert any(len(c["relations"]) > MAX_PATH_RELATIONS and c["reached"] for c in cases)
    assert sum(1 for c in cases if c.get("fallback") and c["reached"]) > 20
    for c in cases:
        if c["reached"] and c["relations"] and not c.get("fallback"):
            start = c["plan"][0] if c.get("stripped") else c["start"]  # (a stripped start plans as read)
            assert c["plan"] == [start, *c["relations"][:MAX_PATH_RELATIONS]]
            assert c["answer"] in c["reached"]
        else:  # (a fallback start plans nothing)
            assert c["plan"] is None


class SeamRunner:
    """The executor's runner over the host seam (core.cuh built with g++): the same
    admissions and the same two syncs, one token at a time per slot, so the executor's host
    logic and the kernels' row logic run on the CPU."""

    def __init__(self, index, tokenizer, versions, settings, slots):
        from tests.seam import SeamEngine

        self.seam = SeamEngine(index, tokenizer, index.span_syntax, slots, versions=versions, paths=True,
                               committed_paths=settings.get("committed_paths", True),
                               start_rank=settings.get("start_rank", "degree"),
                               unquoted_starts=settings.get("unquoted_starts", False))
        self.versions, self.max_sequences = versions, slots

    def view(self, version):
        if version is not None and (self.versions is None or version not in self.versions.names):
            raise ValueError(f"no KG version {version!r}")
        return self.seam.view(version)

    def run(self, history, before, total, admissions):
        seam, n = self.seam, len(admissions)
        for k, version, anchor in admissions:
            seam.begin(k)
            if anchor:
                seam.anchor(k, anchor)
            seam.set_version(k, version)
        out = []
        for upto in (before, total):
            for k in range(n):
                done = 0 if upto is before else int(before[k])
                for token in history[k, done: int(upto[k])].tolist():
                    seam.advance_slot(k, token)
            states = seam.states()
            out += [{name: v[:n] for name, v in states.items()}, seam.memory()[:n]]
        return tuple(out)


def _executor(world_name: str, setting: str, max_paths: int = 256, seam: bool = False):
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.programs import MatchedExecutor

    data = fixture()
    _, served, _ = world(world_name)
    index = world_index(world_name, True)
    edits = {name: [tuple(e) for e in v] for name, v in data["edits"][world_name].items()}
    versions = build_kg_versions(index, edits)
    settings = data["settings"][setting]
    runner = SeamRunner(index, served, versions, settings, max_paths) if seam else None
    return MatchedExecutor(index, served, versions=versions, max_paths=max_paths, _runner=runner, **settings)


def served(cases):
    """The cases the executor serves: all but the anchors without label rows (errors);
    the anchored fallbacks included (every fixture fallback anchors one entity)."""
    return [c for c in cases if "error" not in c]


def _groups():
    groups = defaultdict(list)
    for case in fixture()["cases"]:
        groups[(case["world"], case["setting"])].append(case)
    return groups


def _refusals(executor, cases):
    """Anchors without label rows, one call each: ValueError."""
    for case in cases:
        if "error" in case:
            with pytest.raises(ValueError, match="anchor has no writable label rows"):
                executor.execute(case["start"], case["relations"], anchor=case["anchor"], version=case["version"])


def _job(case) -> tuple:
    return (case["start"], case["relations"], case["version"], case.get("anchor"))


def _check(cases, got, where):
    for case, path in zip(cases, got, strict=True):
        at = (*where, case["start"], case["relations"], case["version"], case.get("anchor"))
        assert list(path.reached) == case["reached"], at
        assert path.answer == case["answer"], at
        assert (None if path.plan is None else list(path.plan)) == case["plan"], at
        assert path.stripped == case.get("stripped", False), at


def _check_live(executor, cases, where):
    """The live frontier of every served case (starts and frontiers of a world's paths in
    one batch): starts, frontier, frontier_relations, derivations, execute_set (with and
    without witnesses) and execution with repair equal the reference executor's."""
    ids = executor._index.labels.owner_ids
    jobs = [(c["start"], [], c["version"], c.get("anchor")) for c in cases]
    # (frontier reads the start as written, stripped of quotation marks where that names
    # something; starts takes it as written)
    jobs += [(executor._read(c["start"], c.get("anchor"), c["version"]), c["relations"], c["version"], c.get("anchor"))
             for c in cases]
    got = executor.frontiers(jobs)
    for case, starts, frontier in zip(cases, got[: len(cases)], got[len(cases):], strict=True):
        at = (*where, case["start"], case["relations"], case["version"], case.get("anchor"))
        assert [ids[e] for e, _ in starts] == case["starts"], at
        assert [ids[e] for e, _ in frontier] == case["frontier"], at
    for case in cases:
        at = (*where, case["start"], case["relations"], case["version"], case.get("anchor"))
        relations = executor.frontier_relations(case["start"], case["relations"], case.get("anchor"), case["version"])
        assert [list(x) for x in relations] == case["frontier_relations"], at
        derivations = executor.derivations(case["start"], case["relations"], case.get("anchor"), case["version"])
        assert [list(x) for x in derivations] == case["derivations"], at
        complete = executor.execute_set(case["start"], case["relations"], case.get("anchor"), case["version"])
        assert complete == case["execute_set"], at
        if "error" in case["witnesses"]:  # an id whose tail is no number ranks no chain
            with pytest.raises(ValueError, match="invalid literal"):
                executor.execute_set(case["start"], case["relations"], case.get("anchor"), case["version"],
                                     witnesses=True)
        else:
            assert executor.execute_set(case["start"], case["relations"], case.get("anchor"), case["version"],
                                        witnesses=True) == case["witnesses"], at
        want = case["repaired"]
        try:
            path = executor.execute(case["start"], case["relations"], anchor=case.get("anchor"),
                                    version=case["version"], repair=True)
        except ValueError as error:  # a repaired relation without a label of its own: no span writes it
            assert "no label of its own" in str(error) and want["plan"] is None, at
            continue
        assert (list(path.reached), path.answer, None if path.plan is None else list(path.plan)) == (
            want["reached"], want["answer"], want["plan"]), at


def test_matched_execution_on_the_host_seam_equals_the_reference():
    """Every recorded path through the executor with the kernels' row logic on the CPU (the
    host seam in place of the CUDA engine): the reference's entities in its order, its
    answer and its plan."""
    for (world_name, setting), cases in _groups().items():
        executor = _executor(world_name, setting, max_paths=64, seam=True)
        _check(served(cases), executor.execute_many([_job(c) for c in served(cases)]), (world_name, setting))
        _refusals(executor, cases)
        _check_live(executor, served(cases), (world_name, setting))


@pytest.mark.gpu
def test_matched_execution_equals_the_reference():
    """Every recorded path, executed on the GPU a world and setting at a time, reaches the
    reference's entities in its order, delivers its answer and reports its plan; its
    starts, live frontier and frontier relations are the reference executor's."""
    for (world_name, setting), cases in _groups().items():
        executor = _executor(world_name, setting)
        _check(served(cases), executor.execute_many([_job(c) for c in served(cases)]), (world_name, setting))
        _refusals(executor, cases)
        _check_live(executor, served(cases), (world_name, setting))


@pytest.mark.gpu
def test_matched_execution_in_small_batches_and_single_calls():
    """A batch larger than the executor's slots runs in pieces with the same results, and
    `execute` (one path) agrees with the batch."""
    cases = [c for c in served(fixture()["cases"]) if c["world"] == "rand_bpe" and c["setting"] == "committed"
             and "anchor" not in c]
    executor = _executor("rand_bpe", "committed", max_paths=7)
    got = executor.execute_many([(c["start"], c["relations"], c["version"]) for c in cases])
    assert [list(p.reached) for p in got] == [c["reached"] for c in cases]
    for case in cases[:5]:
        one = executor.execute(case["start"], case["relations"], version=case["version"])
        assert list(one.reached) == case["reached"] and one.answer == case["answer"]


def test_frontier_labels_name_the_frontier_relations():
    """frontier_labels: the written labels (and aliases) of exactly the relations
    frontier_relations lists, each naming one of them; named: the entities a label names."""
    case = next(c for c in served(fixture()["cases"]) if c["world"] == "toy" and c["frontier_relations"])
    executor = _executor("toy", case["setting"], max_paths=4, seam=True)
    _, served_tokenizer, _ = world("toy")
    args = (case["start"], case["relations"], case.get("anchor"), case["version"])
    labels = executor.frontier_labels(*args)
    want = {r for r, _ in case["frontier_relations"]}
    relations = executor._index.relations
    assert labels and labels == sorted(set(labels)) and set(labels) <= set(executor.relation_labels())
    for label in labels:
        lo, hi = relations.prefix_range(list(served_tokenizer.encode(" " + label)))
        assert {relations.owner_id(r) for r in range(lo, hi)} & want, label
    assert set(case["starts"]) <= executor.named(case["start"])


def test_matched_executor_refuses_what_it_does_not_serve():
    executor = _executor("toy", "committed", max_paths=2, seam=True)
    kg, _, _ = world("toy")
    a, b = [e for e in kg.entities if e.labels][:2]
    assert not set(a.labels) & set(b.labels)
    with pytest.raises(ValueError, match="no one label names them all"):  # a fallback no span can write
        executor.execute("Nobody Here", ["place of birth"], anchor=[a.id, b.id])
    with pytest.raises(ValueError, match="no KG version"):
        executor.execute("Paris Hilton", ["place of birth"], version="v9")
    from xgraph_b200.programs import MatchedExecutor

    _, served, _ = world("toy")
    with pytest.raises(ValueError, match="observe_required"):
        MatchedExecutor(world_index("toy", True), served, observe_required=True)
