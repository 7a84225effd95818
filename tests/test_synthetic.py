"""The synthetic workload generators (CPU): exact vocabulary sizes, the index they build,
and constrained stream sampling run against the host seam of the engine logic, checked
token by token with the oracle."""

from __future__ import annotations

import itertools

import numpy as np


def test_config1_world_and_byte_tokenizer():
    from xgraph_b200.synthetic import build_workload

    w = build_workload(1, 1)
    assert w.served.vocab_size == 256
    assert w.index.labels.num_rows == 1000 - len(w.index.labels.excluded)
    assert len(w.index.relations.owner_ids) == 20


def test_bpe_tokenizer_has_exact_size():
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.synthetic import synthetic_tokenizer, synthetic_world

    world = synthetic_world(5, 300, 10, 900)
    served = synthetic_tokenizer(world, 2000, SpanSyntax())
    assert served.vocab_size == 2000
    assert served.special_ids


def test_sampled_streams_are_oracle_valid_on_the_seam():
    import torch

    from oracle.oracle import Oracle
    from tests.seam import SeamEngine
    from xgraph_b200.index import build_kg_index_arrays
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.synthetic import sample_streams, synthetic_tokenizer, synthetic_world

    syntax = SpanSyntax()
    world = synthetic_world(9, 400, 12, 2000, labels=(1, 3))
    served = synthetic_tokenizer(world, 1500, syntax)
    index = build_kg_index_arrays(world.entities, world.relations, world.triples, served, syntax,
                                  sitelinks=world.sitelinks)
    options = {"paths": True, "committed_paths": True}
    rows, steps = 6, 120
    seam = SeamEngine(index, served, syntax, rows, **options)
    seam.begin = _begin_adapter(seam)
    tokens, counts, _ = sample_streams(seam, served, syntax, world, rows, steps, seed=4, device="cpu")
    oracle = Oracle(index, served, syntax, **options)
    opened = 0
    for r in range(rows):
        state = oracle.initial_state()
        for k, token in enumerate(tokens[r].tolist()):
            assert len(oracle.allowed(state)) == int(counts[r, k])
            state = oracle.advance(state, token)
            opened += state.phase.value == "span"
    assert opened > rows * steps // 10  # the walk spends real time inside spans


def _begin_adapter(seam):
    plain = seam.begin

    def begin(slot):
        if hasattr(slot, "tolist"):
            for s in slot.tolist():
                plain(int(s))
        else:
            plain(int(slot))

    return begin


def test_request_edits_are_pair_replacements_the_versions_apply():
    """The seeded per-request edits (the versions benchmark configuration) are the
    reference's pair-replacement edits (src/xgraph/kgversions.py:203-216): in the built
    version every touched (subject, relation) pair holds exactly the label rows of its
    edits' objects (none when the pair was emptied), and untouched pairs keep the base
    KG's objects."""
    from xgraph_b200.index import build_kg_index_arrays
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.synthetic import object_sets, request_edits, synthetic_tokenizer, synthetic_world

    syntax = SpanSyntax()
    world = synthetic_world(21, 400, 12, 3000, labels=(1, 2))
    served = synthetic_tokenizer(world, 1500, syntax)
    index = build_kg_index_arrays(world.entities, world.relations, world.triples, served, syntax)
    pairs = object_sets(world)
    assert request_edits(world, pairs, np.random.default_rng(0), 0) == []
    edits = request_edits(world, pairs, np.random.default_rng(3), 120)
    view = build_kg_versions(index, {"r": edits}).view(index, "r")
    entity_at = {e: k for k, (e, _) in enumerate(world.entities)}
    rows_of: dict[int, list[int]] = {}
    for row, owner in enumerate(index.labels.owners):
        rows_of.setdefault(int(owner), []).append(row)
    touched: dict[tuple[str, str], set[str]] = {}
    emptied = 0
    for s, r, o in edits:
        touched.setdefault((s, r), set())
        if o is None:
            emptied += 1
        else:
            touched[(s, r)].add(o)
    assert touched and emptied
    for (s, r), objects in touched.items():
        if not rows_of.get(entity_at[s]):
            continue  # a subject without label rows: the edit is unwritable
        expected = {row for o in objects for row in rows_of.get(entity_at[o], [])}
        assert set(view.object_rows(s, r)) == expected, (s, r)
    relation_id = [r for r, _ in world.relations]
    for (s, r), objects in list(itertools.islice(pairs.items(), 200)):
        sid, rid = world.entities[s][0], relation_id[r]
        if (sid, rid) in touched or not rows_of.get(s):
            continue
        expected = {row for o in objects for row in rows_of.get(o, [])}
        assert set(view.object_rows(sid, rid)) == expected, (sid, rid)


def test_seam_masks_equal_the_oracle_at_the_ordinary_benchmark_size():
    """The kernel logic compiled for the host (tests/seam.py) on the ordinary benchmark
    configuration's world (20 k entities, 50 relations, 100 k triples, a 32,000-id BPE):
    three constrained streams of 40 tokens sampled under its own masks, and at every step
    the full allowed set equals the oracle's."""
    from oracle.oracle import Oracle
    from tests.conftest import unpack
    from tests.seam import SeamEngine
    from xgraph_b200.synthetic import build_workload, sample_streams

    w = build_workload(2)
    rows, steps = 3, 40
    seam = SeamEngine(w.index, w.served, w.syntax, rows, **w.config.options)
    seam.begin = _begin_adapter(seam)
    record = {(r, k) for r in range(rows) for k in range(steps + 1)}
    tokens, _, recorded = sample_streams(seam, w.served, w.syntax, w.world, rows, steps, seed=12,
                                         device="cpu", record=record)
    oracle = Oracle(w.index, w.served, w.syntax, **w.config.options)
    spans = 0
    for r in range(rows):
        state = oracle.initial_state()
        for k in range(steps + 1):
            words = np.asarray(recorded[(r, k)]).astype(np.uint32)
            assert unpack(words, w.served.vocab_size) == set(oracle.allowed(state)), (r, k)
            if k < steps:
                state = oracle.advance(state, int(tokens[r, k]))
                spans += state.phase.value == "span"
    assert spans > rows * steps // 10


def test_seam_masks_equal_the_oracle_at_the_path_benchmark_size():
    """The same at the path benchmark configuration (100 k entities with 1-3 labels, 1 M
    triples, paths with committed paths, V = 128,256): two streams of 60 tokens, the full
    allowed set compared with the oracle's at every fourth step (a 128 k-wide scan each)."""
    from oracle.oracle import Oracle
    from tests.conftest import unpack
    from tests.seam import SeamEngine
    from xgraph_b200.synthetic import build_workload, sample_streams

    w = build_workload(3)
    rows, steps = 2, 60
    seam = SeamEngine(w.index, w.served, w.syntax, rows, **w.config.options)
    seam.begin = _begin_adapter(seam)
    record = {(r, k) for r in range(rows) for k in range(0, steps + 1, 4)}
    tokens, _, recorded = sample_streams(seam, w.served, w.syntax, w.world, rows, steps, seed=13,
                                         device="cpu", record=record)
    oracle = Oracle(w.index, w.served, w.syntax, **w.config.options)
    spans = 0
    for r in range(rows):
        state = oracle.initial_state()
        for k in range(steps + 1):
            if (r, k) in recorded:
                words = np.asarray(recorded[(r, k)]).astype(np.uint32)
                assert unpack(words, w.served.vocab_size) == set(oracle.allowed(state)), (r, k)
            if k < steps:
                state = oracle.advance(state, int(tokens[r, k]))
                spans += state.phase.value == "span"
    assert spans > rows * steps // 10


def test_seam_masks_equal_the_oracle_with_per_request_kg_versions():
    """The versions configuration on the host-compiled kernel logic: three requests, each
    with 0-256 seeded add/remove edits as its own KG version, V = 151,936, paths with
    committed paths, on a 2 k-entity world (so the edits meet the walks): every sixth
    step's full allowed set equals the oracle's for the request's version, and the same
    streams replayed on the base KG mask some step differently."""
    from oracle.oracle import Oracle
    from tests.conftest import unpack
    from tests.seam import SeamEngine
    from xgraph_b200.index import build_kg_index_arrays
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.synthetic import (object_sets, request_edits, sample_streams, synthetic_tokenizer,
                                       synthetic_world)

    syntax = SpanSyntax()
    world = synthetic_world(505, 2_000, 40, 20_000, labels=(1, 3))
    served = synthetic_tokenizer(world, 151_936, syntax)
    index = build_kg_index_arrays(world.entities, world.relations, world.triples, served, syntax,
                                  sitelinks=world.sitelinks)
    rng = np.random.default_rng(55)
    rows, steps, every = 3, 48, 6
    pairs = object_sets(world)
    edits = {f"request-{i}": request_edits(world, pairs, rng, int(rng.integers(0, 257))) for i in range(rows)}
    names = list(edits)
    options = {"paths": True, "committed_paths": True}
    seam = SeamEngine(index, served, syntax, rows, versions=build_kg_versions(index, edits), **options)
    seam.begin = _begin_adapter(seam)
    record = {(r, k) for r in range(rows) for k in range(steps + 1)}
    tokens, _, recorded = sample_streams(seam, served, syntax, world, rows, steps, seed=56, device="cpu",
                                         record=record, versions=names)
    # the same streams on the base KG mask some step differently: the versions are read
    base = SeamEngine(index, served, syntax, rows, **options)
    for r in range(rows):
        base.begin(r)
    differs = 0
    host_tokens = np.asarray(tokens)
    for k in range(steps + 1):
        masks = base.masks()
        differs += sum(not np.array_equal(masks[r], np.asarray(recorded[(r, k)]).astype(np.uint32)) for r in range(rows))
        if k < steps:
            base.advance(host_tokens[:, k])
    assert differs > 0
    oracle = Oracle(index, served, syntax, versions=edits, **options)
    for r in range(rows):
        state = oracle.initial_state(names[r])
        for k in range(steps + 1):
            if k % every == 0:
                words = np.asarray(recorded[(r, k)]).astype(np.uint32)
                assert unpack(words, served.vocab_size) == set(oracle.allowed(state)), (r, k)
            if k < steps:
                state = oracle.advance(state, int(host_tokens[r, k]))


def test_arrival_schedule_serves_every_request_in_ragged_batches():
    """The versions configuration's continuous batching: Poisson arrivals, geometric lengths,
    first come first served into at most `rows` slots; a slot is never shared, a request
    holds its slot for exactly its length, and the batch starts full."""
    from xgraph_b200.synthetic import CONFIGS, arrival_schedule

    cfg = CONFIGS[5]
    steps = 400
    a = arrival_schedule(cfg, steps, seed=5)
    assert len(a.live[0]) == cfg.rows and all(len(live) <= cfg.rows for live in a.live)
    owner = {}
    for k in range(steps):
        for slot, r in a.admitted[k]:
            assert a.slot[r] == slot and a.start[r] == k >= a.arrival[r]
        for slot in a.live[k]:
            r = next(r for r in range(len(a.slot)) if a.slot[r] == slot and a.start[r] <= k < a.start[r] + a.length[r])
            owner.setdefault((slot, r), 0)
            owner[(slot, r)] += 1
    for (slot, r), held in owner.items():
        assert held == min(a.length[r], steps - a.start[r])
    lengths = np.array(a.length)
    assert 150 < lengths.mean() < 350 and lengths.max() <= cfg.lengths[1]
    rate = (len(a.arrival) - cfg.rows) / (steps - 1)
    assert 0.35 < rate < 0.65  # 2,000 req/s over 8 GPUs at a 2 ms step: 0.5 per step
