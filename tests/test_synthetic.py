"""The synthetic workload generators (CPU): exact vocabulary sizes, the index they build,
and constrained stream sampling run against the host seam of the engine logic, checked
token by token with the oracle."""

from __future__ import annotations

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
