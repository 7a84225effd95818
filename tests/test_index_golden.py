"""The index builder and version tables against the reference's compiled arrays."""

from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import case_index, case_versions, golden_index, golden_walks, golden_worlds, world


@pytest.mark.parametrize("name", sorted(golden_worlds()))
def test_index_arrays_equal_reference(name):
    from xgraph_b200.index import build_kg_index
    from xgraph_b200.syntax import SpanSyntax

    kg, served, sitelinks = world(name)
    index = build_kg_index(kg, served, SpanSyntax(), sitelinks=sitelinks)
    ref = golden_index()
    for part in ("labels", "relations"):
        rows = getattr(index, part)
        for field in ("tokens", "offsets", "owners"):
            np.testing.assert_array_equal(getattr(rows, field), ref[f"{name}/{part}.{field}"], f"{part}.{field}")
    for field in ("adjacency_offsets", "edge_relations", "edge_objects", "sitelinks"):
        np.testing.assert_array_equal(getattr(index, field), ref[f"{name}/{field}"], field)
    assert index.unwritable_triples == int(ref[f"{name}/unwritable"][0])
    excluded = [f"{e.owner_id}\t{e.label}\t{e.reason}" for e in index.labels.excluded]
    assert excluded == list(ref[f"{name}/excluded"])


@pytest.mark.parametrize("name", [c["name"] for c in golden_walks() if c["versions"]])
def test_version_tables_equal_reference(name):
    from xgraph_b200.kgversions import build_kg_versions

    case = next(c for c in golden_walks() if c["name"] == name)
    versions = build_kg_versions(case_index(case), case_versions(case))
    ref = golden_index()
    for mine, theirs in (
        ("offsets", "version_offsets"), ("subjects", "version_subjects"),
        ("adjacency", "version_adjacency"), ("edge_relations", "version_edge_relations"),
        ("edge_objects", "version_edge_objects"),
    ):
        np.testing.assert_array_equal(getattr(versions, mine), ref[f"{name}/{theirs}"], mine)


def test_prefix_range_matches_linear_scan():
    index = case_index({"world": "toy", "options": {}})
    labels = index.labels
    rows = [labels.row_tokens(r) for r in range(labels.num_rows)]
    prefixes = {row[:k] for row in rows for k in range(len(row) + 1)}
    for prefix in prefixes:
        hits = [r for r, row in enumerate(rows) if row[: len(prefix)] == prefix]
        assert labels.prefix_range(prefix) == (hits[0], hits[-1] + 1)


def test_reads_the_reference_on_disk_index():
    """An index saved by the reference's own save_kg_index (tests/golden/reference_index_toy,
    made by tests/golden/make_reference_index.py) loads with the arrays this library builds
    for the same world, and packs into the same device tables."""
    from pathlib import Path

    from tests.conftest import world, world_index
    from xgraph_b200.index import load_kg_index
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.tables import pack_tables

    loaded = load_kg_index(Path(__file__).parent / "golden" / "reference_index_toy")
    built = world_index("toy", True)
    for part in ("labels", "relations"):
        a, b = getattr(loaded, part), getattr(built, part)
        assert a.owner_ids == b.owner_ids
        for name in ("tokens", "offsets", "owners"):
            np.testing.assert_array_equal(getattr(a, name), getattr(b, name))
    for name in ("adjacency_offsets", "edge_relations", "edge_objects", "sitelinks"):
        np.testing.assert_array_equal(getattr(loaded, name), getattr(built, name))
    assert loaded.span_syntax == SpanSyntax() and loaded.unwritable_triples == built.unwritable_triples
    _, served, _ = world("toy")
    a = pack_tables(loaded, served, loaded.span_syntax, escapes=True)
    b = pack_tables(built, served, built.span_syntax, escapes=True)
    np.testing.assert_array_equal(a.blob, b.blob)


def _rand_bpe_served():
    from tests.conftest import world

    _, served, _ = world("rand_bpe")
    return served


@pytest.mark.parametrize("unique", [False, True])
def test_builds_the_reference_kg_directory_index(unique):
    """A KG directory in the reference's layout (tests/golden/kg_directory_toy: spread-out
    item numbers, an alias-only property, triples naming unknown items and properties,
    sitelink counts, aliases that are another property's label or shared by two) builds the
    index the reference's own directory builder saved from it, with and without
    unique_aliases (tests/golden/kg_directory_toy_index[_unique], all made by
    tests/golden/make_kg_directory.py): the same arrays, unwritable count and packed
    device tables."""
    from pathlib import Path

    from xgraph_b200.index import build_kg_directory_index, load_kg_index
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.tables import pack_tables

    golden = Path(__file__).parent / "golden"
    served = _rand_bpe_served()
    built = build_kg_directory_index(golden / "kg_directory_toy", served, SpanSyntax(), unique_aliases=unique)
    saved = load_kg_index(golden / ("kg_directory_toy_index_unique" if unique else "kg_directory_toy_index"))
    for part in ("labels", "relations"):
        a, b = getattr(built, part), getattr(saved, part)
        assert a.owner_ids == b.owner_ids
        for name in ("tokens", "offsets", "owners"):
            np.testing.assert_array_equal(getattr(a, name), getattr(b, name))
    for name in ("adjacency_offsets", "edge_relations", "edge_objects", "sitelinks"):
        np.testing.assert_array_equal(getattr(built, name), getattr(saved, name))
    assert built.unwritable_triples == saved.unwritable_triples == 2
    a = pack_tables(built, served, built.span_syntax, escapes=True)
    b = pack_tables(saved, served, saved.span_syntax, escapes=True)
    np.testing.assert_array_equal(a.blob, b.blob)


def test_kg_directory_errors_and_relation_names(tmp_path):
    import json

    from xgraph_b200.index import build_kg_directory_index, relation_names
    from xgraph_b200.kg import KGFormatError
    from xgraph_b200.syntax import SpanSyntax

    rows = [("P1", "head of state", "label"), ("P2", "office held", "label"), ("P2", "Head of State", "alias"),
            ("P2", "chief", "alias"), ("P3", "leader", "label"), ("P3", "chief", "alias")]
    assert relation_names(rows) == {"P1": ["head of state"], "P2": ["office held", "chief"],
                                    "P3": ["leader", "chief"]}
    assert relation_names(rows, unique_aliases=True) == {"P1": ["head of state"], "P2": ["office held"],
                                                         "P3": ["leader"]}
    served = _rand_bpe_served()
    with pytest.raises(KGFormatError, match="missing"):
        build_kg_directory_index(tmp_path, served, SpanSyntax())
    (tmp_path / "entity_labels.jsonl").write_text(json.dumps(["E7", "Ba", "label"]) + "\n", encoding="utf-8")
    (tmp_path / "relation_labels.jsonl").write_text(json.dumps(["P1", "author", "label"]) + "\n", encoding="utf-8")
    np.save(tmp_path / "triples.npy", np.zeros((0, 3), dtype=np.int32))
    with pytest.raises(KGFormatError, match="Q<number>"):
        build_kg_directory_index(tmp_path, served, SpanSyntax())


def test_directory_index_command_saves_what_the_builder_returns(tmp_path):
    import gzip
    import json
    from pathlib import Path

    from xgraph_b200.index import build_kg_directory_index, load_kg_index, main
    from xgraph_b200.syntax import SpanSyntax

    golden = Path(__file__).parent / "golden"
    with gzip.open(golden / "worlds.json.gz", "rt", encoding="utf-8") as f:
        (tmp_path / "tokenizer.json").write_text(json.load(f)["rand_bpe"]["tokenizer"], encoding="utf-8")
    main(["--kg", str(golden / "kg_directory_toy"), "--tokenizer", str(tmp_path / "tokenizer.json"),
          "--out", str(tmp_path / "index"), "--unique-aliases"])
    saved = load_kg_index(tmp_path / "index")
    built = build_kg_directory_index(golden / "kg_directory_toy", _rand_bpe_served(), SpanSyntax(), unique_aliases=True)
    assert saved.base_fingerprint == built.base_fingerprint
    for name in ("adjacency_offsets", "edge_relations", "edge_objects", "sitelinks"):
        np.testing.assert_array_equal(getattr(saved, name), getattr(built, name))
    assert saved.relations.owner_ids == built.relations.owner_ids
