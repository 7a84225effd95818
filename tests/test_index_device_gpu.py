"""The device-side index build (xg_build_label_rows, xg_build_adjacency) against the host
build.

The reference builds a KG index on the host (src/xgraph/index.py:167-233 label rows,
403-516 edges); the library's device build must give the same arrays: label rows admitted
under exact-v1 and sorted as (token sequence, owner) tuples, with the same excluded labels
and reasons; CSR offsets per subject entity, edge relations and object label rows sorted
by (subject, relation, object row) without duplicates, and the same count of unwritable
triples (subject or object without label rows, relation without a relation row).  Equal
arrays give equal index fingerprints.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def both(entities, relations, triples, served, syntax, sitelinks=None):
    from xgraph_b200.index import build_kg_index_arrays

    host = build_kg_index_arrays(entities, relations, triples, served, syntax, sitelinks=sitelinks)
    device = build_kg_index_arrays(entities, relations, triples, served, syntax, sitelinks=sitelinks, device="cuda")
    return host, device


def assert_same_labels(host, device):
    for name, dtype in (("tokens", np.int32), ("offsets", np.int64), ("owners", np.int32)):
        a, b = np.asarray(getattr(host, name)), np.asarray(getattr(device, name))
        np.testing.assert_array_equal(a, b, err_msg=name)
        assert b.dtype == dtype, name
    assert host.owner_ids == device.owner_ids
    assert host.excluded == device.excluded


def assert_same(host, device):
    assert_same_labels(host.labels, device.labels)
    assert_same_labels(host.relations, device.relations)
    np.testing.assert_array_equal(host.adjacency_offsets, device.adjacency_offsets)
    np.testing.assert_array_equal(host.edge_relations, device.edge_relations)
    np.testing.assert_array_equal(host.edge_objects, device.edge_objects)
    assert host.adjacency_offsets.dtype == device.adjacency_offsets.dtype == np.int64
    assert host.edge_relations.dtype == device.edge_relations.dtype == np.int32
    assert host.edge_objects.dtype == device.edge_objects.dtype == np.int32
    assert host.unwritable_triples == device.unwritable_triples
    assert host.base_fingerprint == device.base_fingerprint


@pytest.mark.parametrize("zipf", [None, 1.3])
def test_device_adjacency_equals_host_on_synthetic_worlds(zipf):
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.synthetic import synthetic_tokenizer, synthetic_world

    syntax = SpanSyntax()
    world = synthetic_world(11, 3000, 80, 60000, labels=(1, 3), zipf=zipf)
    served = synthetic_tokenizer(world, 4000, syntax)
    host, device = both(world.entities, world.relations, world.triples, served, syntax, world.sitelinks)
    assert len(host.edge_objects) > len(world.triples) // 2
    assert_same(host, device)


def test_device_adjacency_equals_host_at_the_path_benchmark_size():
    from xgraph_b200.synthetic import build_workload

    host = build_workload(3)
    device = build_workload(3, device="cuda")
    assert_same(host.index, device.index)


def test_unwritable_triples_duplicates_and_empty_kg():
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.synthetic import synthetic_tokenizer, synthetic_world

    syntax = SpanSyntax()
    served = synthetic_tokenizer(synthetic_world(5, 300, 10, 900), 2000, syntax)
    entities = [("a", ["Alpha"]), ("b", ["Beta", "Bee"]), ("c", [f"bad {syntax.closer} label"]), ("d", [])]
    relations = [("r", ["likes"]), ("q", [f"no {syntax.opener}"])]
    triples = np.array([
        (0, 0, 1), (0, 0, 1), (1, 0, 0),  # a duplicate collapses
        (0, 0, 2), (2, 0, 0), (3, 0, 0),  # subject or object without label rows
        (0, 1, 1),                        # relation without a relation row
    ])
    host, device = both(entities, relations, triples, served, syntax)
    assert host.unwritable_triples == 4
    assert list(host.edge_objects) == [1, 2, 0]
    assert_same(host, device)
    empty_host, empty_device = both(entities, relations, np.zeros((0, 3), dtype=np.int64), served, syntax)
    assert len(empty_device.edge_objects) == 0 and not empty_device.adjacency_offsets.any()
    assert_same(empty_host, empty_device)


def test_out_of_range_position_is_a_value_error():
    """The check kernel tests every position against its bound before it reads anything
    indexed by it, and the call fails with XG_EINVAL (ValueError)."""
    from xgraph_b200.index import _adjacency_device, label_rows
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.synthetic import synthetic_tokenizer, synthetic_world

    syntax = SpanSyntax()
    served = synthetic_tokenizer(synthetic_world(5, 300, 10, 900), 2000, syntax)
    labels = label_rows([("a", ["Alpha"]), ("b", ["Beta"])], served, syntax)
    writable = np.ones(1, dtype=bool)
    with pytest.raises(ValueError, match="out of range"):
        _adjacency_device(labels, writable, np.array([0]), np.array([0]), np.array([2]), 2, "cuda")


def test_kg_directory_builds_the_same_index_on_the_device():
    from pathlib import Path

    from tests.conftest import world
    from xgraph_b200.index import build_kg_directory_index
    from xgraph_b200.syntax import SpanSyntax

    _, served, _ = world("rand_bpe")
    kg = Path(__file__).parent / "golden" / "kg_directory_toy"
    host = build_kg_directory_index(kg, served, SpanSyntax())
    device = build_kg_directory_index(kg, served, SpanSyntax(), device="cuda")
    assert_same(host, device)


def test_device_label_admission_gives_the_host_reasons():
    """Crafted encodings through the device build: a special token, an empty encoding, an
    id without known bytes (outside the vocabulary), bytes that do not round-trip, and
    admitted labels (one sharing a prefix with another, one a prefix of another); statuses
    and rows equal the host admission (_exact_v1_error) and the host sort."""
    from xgraph_b200.index import ADMISSION_REASONS, _exact_v1_error, _label_rows_device, _sorted_rows
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.synthetic import synthetic_tokenizer, synthetic_world

    syntax = SpanSyntax()
    served = synthetic_tokenizer(synthetic_world(5, 300, 10, 900), 2000, syntax)
    special = min(served.special_ids)
    labels = ["Alpha", "Alphabet", "Beta", "Gamma", "Delta", "Alp", "Epsilon"]
    encoded = [served.encode(syntax.label_prefix + label) for label in labels]
    encoded[2] = encoded[2] + [special]                 # a special token
    encoded[3] = []                                     # an empty encoding
    encoded[4] = encoded[4] + [served.vocab_size + 7]   # an id without bytes
    encoded[6] = list(reversed(encoded[6])) if len(encoded[6]) > 1 else encoded[0]  # bytes differ
    pairs = [(label, position) for position, label in enumerate(labels)]
    tokens, offsets, owners, status = _label_rows_device(pairs, encoded, len(labels), served, syntax, "cuda")
    host_status = []
    for (label, _), ids in zip(pairs, encoded):
        reason = _exact_v1_error(label, ids, served, syntax)
        host_status.append(0 if reason is None else next(k for k, v in ADMISSION_REASONS.items() if v == reason))
    assert status.tolist() == host_status == [0, 0, 1, 2, 3, 0, 4]
    kept = [(encoded[i], i) for i in range(len(labels)) if host_status[i] == 0]
    order = _sorted_rows(kept)
    assert owners.tolist() == [kept[i][1] for i in order]
    assert tokens.tolist() == [t for i in order for t in kept[i][0]]
    assert offsets.tolist() == [0, *np.cumsum([len(kept[i][0]) for i in order]).tolist()]


def test_device_label_rows_equal_host_on_the_golden_worlds():
    """Every golden world's label and relation rows, built on the device, equal the host's
    (which equal the reference's)."""
    from tests.conftest import golden_worlds, world
    from xgraph_b200.index import label_rows
    from xgraph_b200.syntax import SpanSyntax

    syntax = SpanSyntax()
    for name in golden_worlds():
        kg, served, _ = world(name)
        for items in (kg.entities, kg.relations):
            assert_same_labels(label_rows(items, served, syntax), label_rows(items, served, syntax, device="cuda"))
