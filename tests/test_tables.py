"""Packed adjacency tables: relation runs, folded first rows, and the engine's relation
lookup over them (run through the host seam), against the index's own edge lists."""

import numpy as np
import pytest

from xgraph_b200.index import build_kg_index_arrays
from xgraph_b200.synthetic import synthetic_tokenizer, synthetic_world
from xgraph_b200.syntax import SpanSyntax
from xgraph_b200.tables import pack_tables

from .seam import SeamEngine


@pytest.fixture(scope="module")
def hub_world():
    # Zipf subjects: a few hubs carry edges under most of the 80 relations, so lookups go
    # through the pivot rounds as well as the short scans.
    syntax = SpanSyntax()
    world = synthetic_world(11, 300, 80, 6000, zipf=1.3)
    served = synthetic_tokenizer(world, 257, syntax)
    index = build_kg_index_arrays(world.entities, world.relations, world.triples, served, syntax)
    return index, served, syntax


def _array(tables, name, dtype, count):
    off = getattr(tables.layout, name)
    return np.frombuffer(tables.blob, dtype=dtype, count=count, offset=off)


def test_relation_runs_and_folded_first_rows(hub_world):
    index, served, syntax = hub_world
    tables = pack_tables(index, served, syntax, escapes=True)
    offsets = np.asarray(index.adjacency_offsets, dtype=np.int64)
    rel = np.asarray(index.edge_relations)
    obj = np.asarray(index.edge_objects)
    entities = len(offsets) - 1
    run_off = _array(tables, "run_off", np.int32, entities + 1)
    runs_total = int(run_off[-1])
    runs = _array(tables, "runs", np.int32, 2 * (runs_total + 1)).reshape(-1, 2)
    run_rel = _array(tables, "run_rel", np.int32, runs_total)
    assert runs[-1, 0] == np.iinfo(np.int32).max and runs[-1, 1] == len(rel)
    assert (run_rel == runs[:-1, 0]).all()
    assert max(np.diff(run_off)) > 16  # the pivot rounds are exercised
    for e in range(entities):
        a, b = offsets[e], offsets[e + 1]
        want = sorted(set(rel[a:b].tolist()))
        got = runs[run_off[e]:run_off[e + 1]]
        assert got[:, 0].tolist() == want
        for (r, start), nxt in zip(got, runs[run_off[e] + 1:run_off[e + 1] + 1, 1]):
            assert (rel[start:nxt] == r).all() and (start == a or rel[start - 1] != r)
    owners = np.asarray(index.labels.owners, dtype=np.int64)
    first = _array(tables, "edge_first", np.int32, len(obj)).view(np.uint32)
    degree = np.diff(offsets)
    for i in range(0, len(obj), 7):
        o = owners[obj[i]]
        rows = np.flatnonzero(owners == o)
        assert first[i] & 0x7FFFFFFF == rows.min()
        assert bool(first[i] >> 31) == (degree[o] == 0)


def test_relation_slice_matches_edge_lists(hub_world):
    index, served, syntax = hub_world
    seam = SeamEngine(index, served, syntax, 1)
    offsets = np.asarray(index.adjacency_offsets, dtype=np.int64)
    rel = np.asarray(index.edge_relations)
    relations = len(index.relations.owner_ids)
    checked = 0
    for e in range(len(offsets) - 1):
        a, b = int(offsets[e]), int(offsets[e + 1])
        mine = rel[a:b]
        for r in range(-1, relations + 1):
            lo = int(np.searchsorted(mine, r, "left"))
            hi = int(np.searchsorted(mine, r, "right"))
            first, last, n = seam.relation_slice(e, r)
            assert n == b - a
            if lo == hi:
                assert first == last, (e, r)
            else:
                assert (first, last) == (lo, hi), (e, r)
            checked += 1
    assert checked > 10000


def test_byte_table_is_the_token_byte_view():
    """ServedTokenizer.byte_table (the device label build's vocabulary) holds every id's
    bytes and its class: special ids, ids without bytes, and the rest."""
    from tests.conftest import golden_worlds, world

    for name in golden_worlds():
        _, served, _ = world(name)
        offsets, data, kind = served.byte_table()
        assert len(offsets) == len(kind) + 1 and offsets[-1] == len(data)
        for t in range(len(kind)):
            b = served.token_bytes(t)
            if t in served.special_ids:
                assert kind[t] == 1
            elif b is None:
                assert kind[t] == 2
            else:
                assert kind[t] == 0 and bytes(data[offsets[t]:offsets[t + 1]]) == b


def test_label_exclusion_test_equals_the_syntax_rule():
    """The compiled exclusion test of the label build equals SpanSyntax.excludes."""
    from xgraph_b200.index import _excluder
    from xgraph_b200.syntax import PRESETS, SpanSyntax

    labels = ["Marie Curie", "a ⟧ b", "x · y", "q ⁇", "earlier: x", "later:x", "same:", "p |q", "[[x]]", "a|b",
              "</kg>", "【x", 'say "x"', " ⟦", "plain", "ear lier:", "", " "]
    for syntax in [SpanSyntax(), *PRESETS.values(), SpanSyntax(operators=(), operand_separator="")]:
        excludes = _excluder(syntax)
        for label in labels:
            assert excludes(label) == syntax.excludes(label), (syntax, label)
