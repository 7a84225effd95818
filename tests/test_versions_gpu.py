"""KG versions registered while the engine runs (Engine.add_version / drop_version through
xg_add_version / xg_drop_version), and the versions configuration at its stated size.

The reference builds every version into the engine up front (src/xgraph/engine.py
versions=); here a request's version is added when it arrives, read by the kernels from the
engine's version arena (csrc/engine.cu:477-491 is the reference's per-version edge read, the
layout of src/xgraph/kgversions.py:14-21), and dropped when it leaves.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import case_versions, golden_masks, golden_walks, unpack
from tests.test_engine_gpu import engine_for

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["toy_committed", "bpe_committed", "bpe_ordinary", "crowd_committed"])
def test_versions_added_at_run_time_equal_versions_built_in(name):
    """Versions added after construction (in another order, after a dropped one) give every
    golden walk's masks, exactly as the same versions built into the engine."""
    import torch

    from tests.test_admission_gpu import admissions_of, assert_same_slots
    from xgraph_b200.engine import Engine
    from xgraph_b200.syntax import SpanSyntax

    case = next(c for c in golden_walks() if c["name"] == name)
    sequences = case["sequences"]
    n = len(sequences)
    built, index, served = engine_for(case)
    edits = case_versions(case)
    added = Engine(index, served, SpanSyntax(), n, **{k: v for k, v in case["options"].items()})
    scratch = added.add_version("scratch", [next(iter(edits.values()))[0]])
    for version in reversed(list(edits)):
        added.add_version(version, edits[version])
    added.drop_version("scratch")
    assert added.add_version("reused", []) == scratch  # a dropped number is reused
    for engine in (built, added):
        engine.reset()
        engine.admit(admissions_of(sequences))
    assert_same_slots(built, added, n, same_numbers=False)
    memory = added.memory_host(n)
    for k, seq in enumerate(sequences):  # each slot reads the number its version was added under
        assert memory[k, 3] == (added._version_number(seq["version"]))
    for step in range(len(sequences[0]["tokens"])):
        added.fill_mask()
        masks = added.mask_host().view(np.uint32)
        for k in range(n):
            assert unpack(masks[k], served.vocab_size) == unpack(golden_masks()[f"{name}/{k}"][step], served.vocab_size)
        added.advance(np.array([seq["tokens"][step] for seq in sequences], dtype=np.int32))
    assert added.errors() == 0 and added.faults() == 0
    for version in edits:  # closed spans resolve against the added versions' views
        assert added.view(version).labels is index.labels
    with pytest.raises(ValueError):
        added.add_version(next(iter(edits)), [])  # the name is taken
    added.drop_version(next(iter(edits)))
    with pytest.raises(ValueError):
        added.set_version(0, next(iter(edits)))
    del torch


def test_versions_configuration_at_full_size():
    """The versions configuration as benchmarked: 1 M entities, 10 M Zipf triples,
    V = 151,936, path mode with committed paths, requests arriving on the Poisson schedule
    into a ragged batch, each with its own KG version added when it arrives.  Each request's
    edits delete every relation of the first path subject its base-KG walk names (so the
    version changes what it may write) plus 0-256 seeded random edits.  Replayed through the
    fused step with the admissions folded in, checked against the oracle holding exactly
    those requests' versions (state projections at every step, whole allowed sets at seeded
    steps), and the same streams on the base KG must mask some rows differently."""
    import torch

    from oracle.oracle import Oracle
    from tests.agreement import assert_agrees, expected_state
    from tests.conftest import state_record
    from tests.test_configs_gpu import projection
    from xgraph_b200.engine import ADMISSION_INTS, Engine
    from xgraph_b200.synthetic import (CONFIGS, arrival_schedule, build_workload, object_sets, request_edits,
                                       sample_streams)

    w = build_workload(5)
    cfg = w.config
    assert w.served.vocab_size == 151_936 and w.index.labels.num_rows >= 1_000_000
    steps = 96
    sched = arrival_schedule(cfg, steps, seed=5)
    requests = [r for r in range(len(sched.arrival)) if sched.slot[r] >= 0]
    names = [f"request-{r}" for r in requests]
    n = len(requests)
    # pass 1: base-KG walks, to find the first path subject each request names
    base = Engine(w.index, w.served, w.syntax, n, **cfg.options)
    tokens, _, _ = sample_streams(base, w.served, w.syntax, w.world, n, steps, seed=11)
    first_subject: dict[int, int] = {}
    base.reset()
    base.begin(torch.arange(n, dtype=torch.int32, device="cuda"))
    owners = np.asarray(w.index.labels.owners)
    for k in range(steps):
        states = base.states_host(n)
        for j in range(n):
            if j not in first_subject and states["phase"][j] == 1 and states["segment"][j] == 1:
                first_subject[j] = int(owners[states["subj_lo"][j]])
        base.advance(tokens[:, k].contiguous())
    pairs = object_sets(w.world)
    rng = np.random.default_rng(55)
    entity_ids = w.index.labels.owner_ids
    relation_ids = w.index.relations.owner_ids
    edits = {}
    for j, name in enumerate(names):
        own = request_edits(w.world, pairs, rng, int(rng.integers(0, cfg.max_edits + 1)))
        if j in first_subject:
            e = first_subject[j]
            rels, _ = w.index.edges_at(e)
            own += [(entity_ids[e], relation_ids[int(r)], None) for r in np.unique(rels)]
        edits[name] = own
    # pass 2: each request's walk under its own version, added at run time
    sampler = Engine(w.index, w.served, w.syntax, n, **cfg.options)
    for name in names:
        sampler.add_version(name, edits[name])
    tokens, counts, _ = sample_streams(sampler, w.served, w.syntax, w.world, n, steps, seed=11, versions=names)
    assert sampler.errors(n) == 0
    del sampler, base
    # the replay: ragged rows, admissions (with versions) folded into each step's launch
    rows = cfg.rows
    engine = Engine(w.index, w.served, w.syntax, rows, **cfg.options)
    plain = Engine(w.index, w.served, w.syntax, rows, **cfg.options)  # base KG: the same streams
    numbers = [engine.add_version(name, edits[name]) for name in names]
    history = torch.zeros((rows, steps), dtype=torch.int32, device="cuda")
    host = tokens.cpu().numpy()
    joins = [[] for _ in range(steps)]
    for j, r in enumerate(requests):
        slot, k0 = sched.slot[r], sched.start[r]
        m = min(sched.length[r], steps - k0)
        history[slot, k0: k0 + m] = torch.from_numpy(host[j, :m])
        joins[k0].append((slot, j))
    prompt = [torch.full((rows,), k, dtype=torch.int32, device="cuda") for k in range(steps)]
    total = [torch.full((rows,), k + 1, dtype=torch.int32, device="cuda") for k in range(steps)]
    for e in (engine, plain):
        e.reset()
    gen = torch.Generator(device="cuda").manual_seed(3)
    checked = [j for j in range(n) if j in first_subject][:3] or [0]
    oracle = Oracle(w.index, w.served, w.syntax, versions={names[j]: edits[names[j]] for j in checked}, **cfg.options)
    states = {j: oracle.initial_state(names[j]) for j in checked}
    slot_of = {j: sched.slot[requests[j]] for j in range(n)}
    start_of = {j: sched.start[requests[j]] for j in range(n)}
    rng = np.random.default_rng(7)
    differ = 0
    for k in range(steps):
        live = sched.live[k]
        records = np.zeros((len(joins[k]), ADMISSION_INTS), dtype=np.int32)
        base_records = np.zeros_like(records)
        for i, (slot, j) in enumerate(joins[k]):
            records[i, :3] = (slot, 1, numbers[j])
            base_records[i, :3] = (slot, 1, 0)
        slots = torch.tensor(live, dtype=torch.int32, device="cuda")
        logits = (torch.randn((len(live), cfg.vocab), generator=gen, device="cuda") * 2).to(torch.bfloat16)
        a, b = logits.clone(), logits.clone()
        engine.sync_apply(slots, history, prompt[k], total[k], a, admissions=records if len(records) else None)
        plain.sync_apply(slots, history, prompt[k], total[k], b, admissions=base_records if len(records) else None)
        blocked_a = torch.isneginf(a.float())
        # the apply contract on every live row: kept columns bit-identical
        kept = ~blocked_a
        assert torch.equal(a.view(torch.int16)[kept], logits.view(torch.int16)[kept]), k
        differ += int((blocked_a != torch.isneginf(b.float())).any(1).sum())
        got = engine.states_host(rows)
        for j in checked:
            slot, pos = slot_of[j], k - start_of[j]
            if pos < 0 or pos >= sched.length[requests[j]]:
                continue
            states[j] = oracle.advance(states[j], int(host[j, pos]))
            where = (names[j], k)
            assert_agrees(expected_state(state_record(states[j]), w.index, w.syntax),
                          projection(got, slot, engine.view(names[j]), False), True, where)
            if rng.random() < 0.08:
                row = live.index(slot)
                allowed = set(np.flatnonzero(~blocked_a[row, : cfg.vocab].cpu().numpy()).tolist())
                assert allowed == set(oracle.allowed(states[j])), ("allowed set", where)
    assert engine.errors(rows) == 0 and engine.faults() == 0
    assert differ > 0, "no row's mask read its request's version"
    assert int(counts[:, 1:].min()) >= 0 and CONFIGS[5].rows == rows
