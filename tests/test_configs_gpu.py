"""The serving step (sync_apply) at the benchmark configurations, against the oracle.

Streams are constrained decodes sampled on the GPU under the engine's own masks
(xgraph_b200.synthetic.sample_streams, as bench.py makes them); a fresh engine then
replays them the way the serving step runs, one sync_apply launch per step over the
token history in place (the reference's serving loop: src/xgraph/vllm.py:607-631 over
csrc/engine.cu:2057-2074, 2562-2587).  At full size, on every row at every step:

* the apply contract (csrc/engine.cu:2340-2346, 2562-2587): a column keeps its logit bit
  for bit or becomes -inf, nothing else;
* the whole -inf pattern equals the allowed set of the host seam (tests/seam.py: the same
  per-row logic compiled by g++ as a sequential library, independent of the CUDA build,
  itself pinned to the reference's golden walks) advanced over the same tokens.

Against the oracle (oracle/oracle.py, the restatement of src/xgraph/oracle.py), advanced
over the same tokens: the device state's public projection at every step of the checked
rows (tests/agreement.py, as the reference's agreement harness,
tests/test_engine.py:1588-1730), and the kept columns as a set equal to Oracle.allowed —
at every step of every row for config 1 (V = 256), at seeded sampled steps for configs 2
(V = 32,000), 3 and 4 (V = 128,256; config 4 is 1 M entities with 10 M Zipf-distributed
triples, 512 rows), where each allowed set is a V-wide scan on the host.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.agreement import assert_agrees, engine_state, expected_state
from tests.conftest import state_record

pytestmark = pytest.mark.gpu

# config, rows replayed, steps, whole allowed sets checked against the oracle (None: every
# row at every step); the state projections are checked at every step of every row
CASES = [(1, 16, 64, None), (2, 64, 160, 48), (3, 256, 160, 64), (4, 512, 128, 48)]


def projection(states: dict, row: int, view, need_sets: bool) -> dict:
    """engine_state, without the subject/relation sets where the comparison does not read
    them (enumerating a wide subject range over a 100 k-entity index is slow on the host)."""
    if need_sets:
        return engine_state(states, row, view)
    from xgraph_b200.engine import closed_span

    field = {name: int(values[row]) for name, values in states.items()}
    closed = closed_span(view, states, row)
    return {**field, "subjects": set(), "relations": set(),
            "last": None if closed.kind == "none" else (closed.kind, closed.entity_ids, closed.triples),
            "resolved": closed.resolved}


_ORACLE = {}


def _oracle_init(index, served, syntax, options):
    from oracle.oracle import Oracle

    _ORACLE["oracle"] = Oracle(index, served, syntax, **options)


def _allowed_after(job):
    """The oracle's allowed set after `tokens` (a row's stream up to the checked step)."""
    oracle = _ORACLE["oracle"]
    state = oracle.initial_state()
    for token in job:
        state = oracle.advance(state, int(token))
    return sorted(oracle.allowed(state))


def oracle_allowed_sets(workload, syntax, options, prefixes: list, workers: int) -> list:
    """The oracle's allowed sets after each token prefix, on spawned CPU workers (started
    with spawn: a forked child of a CUDA process can hang)."""
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    with ctx.Pool(workers, initializer=_oracle_init,
                  initargs=(workload.index, workload.served, syntax, options)) as pool:
        return pool.map(_allowed_after, prefixes, chunksize=1)


@pytest.mark.parametrize("config, rows, steps, sampled_sets", CASES)
def test_sync_apply_agrees_with_oracle_at_benchmark_config(config, rows, steps, sampled_sets):
    """GPU-sampled streams replayed through the fused step one token at a time.  Every row at
    every step: each column keeps its logit bit for bit or becomes -inf, the -inf pattern is
    exactly the complement of the host seam's mask after the same tokens, and the state
    projection equals the oracle's (the oracle advanced over every token of every row);
    whole allowed sets (the -inf pattern) equal the oracle's at seeded (row, step) samples
    (every row and step at the toy size), computed on spawned workers."""
    import os

    import torch

    from oracle.oracle import Oracle
    from tests.seam import SeamEngine
    from xgraph_b200.engine import Engine
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.synthetic import build_workload, sample_streams

    w = build_workload(config)
    syntax = SpanSyntax()
    options = dict(w.config.options)
    paths = options.get("paths", False)
    vocab = w.served.vocab_size
    sampler = Engine(w.index, w.served, syntax, rows, **options)
    tokens, _, _ = sample_streams(sampler, w.served, syntax, w.world, rows, steps, seed=100 + config)
    del sampler

    rng = np.random.default_rng(200 + config)
    if sampled_sets is None:
        sampled = {(r, k) for r in range(rows) for k in range(steps + 1)}
    else:
        picks = rng.choice(rows * (steps + 1), size=sampled_sets, replace=False).tolist()
        sampled = {(p // (steps + 1), p % (steps + 1)) for p in picks}

    dtype = getattr(torch, w.config.dtype)
    bits = torch.int16 if dtype.itemsize == 2 else torch.int32
    gen = torch.Generator(device="cuda").manual_seed(300 + config)
    source = (torch.randn((rows, vocab), generator=gen, device="cuda") * 2.0).to(dtype)
    engine = Engine(w.index, w.served, syntax, rows, **options)
    engine.reset()
    slots = torch.arange(rows, dtype=torch.int32, device="cuda")
    engine.begin(slots)
    host_tokens = tokens.cpu().numpy()
    seam = SeamEngine(w.index, w.served, syntax, rows, **options)
    for r in range(rows):
        seam.begin(r)
    prompt = torch.zeros(rows, dtype=torch.int32, device="cuda")
    states_at, kept_at = [], {}
    spans = 0
    for k in range(steps + 1):  # total length k: the state after k tokens, the mask for token k
        total = torch.full((rows,), k, dtype=torch.int32, device="cuda")
        logits = source.clone()
        engine.sync_apply(slots, tokens, prompt, total, logits)
        blocked = torch.isneginf(logits)
        same = logits.view(bits) == source.view(bits)
        assert bool((blocked | same).all()), ("a column is neither its logit nor -inf", k)
        if k > 0:
            seam.advance(host_tokens[:, k - 1])
        seam_allowed = np.unpackbits(seam.masks().view(np.uint8), axis=1, bitorder="little")[:, :vocab]
        host_blocked = blocked.cpu().numpy()
        mismatch = np.flatnonzero((host_blocked[:, :vocab] == seam_allowed.astype(bool)).any(axis=1))
        assert mismatch.size == 0, ("-inf pattern differs from the host seam's mask", config, k, mismatch[:8].tolist())
        assert host_blocked[:, vocab:].all()
        states = engine.states_host(rows)
        states_at.append(states)
        spans += int((states["phase"] == 1).sum())
        for r in range(rows):
            if (r, k) in sampled:
                kept_at[(r, k)] = np.flatnonzero((~blocked[r]).cpu().numpy()).tolist()
    assert engine.errors() == 0 and engine.faults() == 0
    assert spans > rows * steps // 10  # the replay spends real time inside spans

    order = sorted(kept_at)
    workers = max(1, min(os.cpu_count() or 1, 8 if config >= 4 else 16, len(order)))
    allowed = oracle_allowed_sets(w, syntax, options, [host_tokens[r, :k] for r, k in order], workers)
    for (r, k), want in zip(order, allowed, strict=True):
        assert kept_at[(r, k)] == want, ("allowed set", config, r, k)

    oracle = Oracle(w.index, w.served, syntax, **options)
    for r in range(rows):
        state = oracle.initial_state()
        for k in range(steps + 1):
            where = (config, r, k)
            expected = expected_state(state_record(state), w.index, syntax)
            need_sets = expected["phase"] == 1 and expected.get("segment", 0) != 0 and not paths
            assert_agrees(expected, projection(states_at[k], r, w.index, need_sets), paths, where)
            if k < steps:
                state = oracle.advance(state, int(host_tokens[r, k]))


def test_sync_apply_with_per_request_kg_versions():
    """Continuous batching with KG versions (the benchmark's versions configuration):
    every request carries 0-256 seeded add/remove-triple edits as its own KG version
    (registered when the engine is built), V = 151,936, path mode with committed paths.
    Each slot serves one request, then is re-begun mid-replay for a second request with
    another version (begin + set_version at admission, as the reference's serving loop
    does).  The world is 2 k entities and 20 k triples rather than 1 M / 10 M: a request's
    ~100-200 edited subjects are then a fair share of the subjects its spans name (on a
    large world the walks almost never meet an edited subject, and the versions would go
    unread), and the oracle builds each checked request's version graphs; the device path
    reads versions the same way at any size.  Checked as above: the apply contract and agreement with the
    sampling engine (each request sampled in its own row under its version) on every row
    at every step; state projections and sampled allowed sets against the oracle holding
    the checked requests' versions; and the same replay on the base KG masks some rows
    differently (the versions are read)."""
    import torch

    from oracle.oracle import Oracle
    from xgraph_b200.engine import Engine
    from xgraph_b200.index import build_kg_index_arrays
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.synthetic import (object_sets, request_edits, sample_streams, synthetic_tokenizer,
                                       synthetic_world)

    syntax = SpanSyntax()
    world = synthetic_world(505, 2_000, 40, 20_000, labels=(1, 3))
    served = synthetic_tokenizer(world, 151_936, syntax)
    assert served.vocab_size == 151_936
    index = build_kg_index_arrays(world.entities, world.relations, world.triples, served, syntax,
                                  sitelinks=world.sitelinks)
    rng = np.random.default_rng(505)
    slots, steps = 32, 160
    pairs = object_sets(world)
    edits = {f"request-{i}": request_edits(world, pairs, rng, int(rng.integers(0, 257))) for i in range(2 * slots)}
    names = list(edits)
    versions = build_kg_versions(index, edits)
    options = {"paths": True, "committed_paths": True}
    vocab = served.vocab_size

    sampler = Engine(index, served, syntax, 2 * slots, versions=versions, **options)
    tokens, counts, _ = sample_streams(sampler, served, syntax, world, 2 * slots, steps, seed=505, versions=names)
    del sampler
    # slot j serves request j for switch[j] tokens, then request slots + j
    switch = np.clip(rng.geometric(1 / 60, size=slots), 8, steps - 8)
    history = torch.zeros((slots, steps), dtype=torch.int32, device="cuda")
    for j in range(slots):
        history[j, : switch[j]] = tokens[j, : switch[j]]
        history[j, switch[j]:] = tokens[slots + j, : steps - switch[j]]

    gen = torch.Generator(device="cuda").manual_seed(606)
    source = (torch.randn((slots, vocab), generator=gen, device="cuda") * 2.0).to(torch.bfloat16)
    engine = Engine(index, served, syntax, slots, versions=versions, **options)
    engine.reset()
    rows = torch.arange(slots, dtype=torch.int32, device="cuda")
    engine.begin(rows)
    for j in range(slots):
        engine.set_version(j, names[j])
    checked = sorted(rng.choice(slots, size=4, replace=False).tolist())
    sampled = {j: {int(rng.integers(0, switch[j])), int(rng.integers(switch[j], steps + 1))} for j in checked}
    base = Engine(index, served, syntax, slots, **options)  # the same replay on the base KG
    base.reset()
    base.begin(rows)
    states_at, kept_at = [], {}
    differs = 0
    switch_t = torch.from_numpy(switch).to("cuda")
    request_of = torch.arange(slots, device="cuda")
    for k in range(steps + 1):
        restarted = [j for j in range(slots) if switch[j] == k]
        if restarted:
            engine.begin(torch.tensor(restarted, dtype=torch.int32, device="cuda"))
            base.begin(torch.tensor(restarted, dtype=torch.int32, device="cuda"))
            for j in restarted:
                engine.set_version(j, names[slots + j])
        prompt = torch.full((slots,), k, dtype=torch.int32, device="cuda")
        total = torch.full((slots,), k, dtype=torch.int32, device="cuda")
        logits = source.clone()
        engine.sync_apply(rows, history, prompt, total, logits)
        unversioned = source.clone()
        base.sync_apply(rows, history, prompt, total, unversioned)
        differs += int((torch.isneginf(unversioned) != torch.isneginf(logits)).any(1).sum())
        blocked = torch.isneginf(logits)
        same = logits.view(torch.int16) == source.view(torch.int16)
        assert bool((blocked | same).all()), ("a column is neither its logit nor -inf", k)
        second = k >= switch_t
        expected = torch.where(second, counts[request_of + slots, (k - switch_t).clamp(min=0)],
                               counts[request_of, min(k, steps)])
        assert torch.equal((~blocked).sum(1, dtype=torch.int32), expected), ("kept columns", k)
        states = engine.states_host(slots)
        states_at.append({name: values[checked].copy() for name, values in states.items()})
        for j in checked:
            if k in sampled[j]:
                kept_at[(j, k)] = np.flatnonzero((~blocked[j]).cpu().numpy())
    assert engine.errors() == 0
    assert differs > 0  # the versions changed some rows' masks in this replay

    host_history = history.cpu().numpy()
    for n, j in enumerate(checked):
        first, later = names[j], names[slots + j]
        oracle = Oracle(index, served, syntax, versions={first: edits[first], later: edits[later]}, **options)
        state = oracle.initial_state(first)
        for k in range(steps + 1):
            if k == switch[j]:
                state = oracle.initial_state(later)
            where = ("versions", j, k)
            view = versions.view(index, state.version)
            expected_fields = expected_state(state_record(state), index, syntax)
            got = projection({name: values[n: n + 1] for name, values in states_at[k].items()}, 0, view, False)
            assert_agrees(expected_fields, got, True, where)
            if (j, k) in kept_at:
                assert set(kept_at[(j, k)].tolist()) == set(oracle.allowed(state)), ("allowed set", where)
            if k < steps:
                state = oracle.advance(state, int(host_history[j, k]))
