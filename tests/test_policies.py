"""apply_mask's logit policies, release and escape bias (the reference's csrc/engine.cu:
2416-2552; its tests/test_engine.py:2487-2581, 2694-2735, 4198-4250).

Which rows and tokens they touch is defined through the oracle, as the reference's tests
define it: a released row may write the allowed tokens after which the escape marker is
being typed or complete; the biased tokens are those of them that end every other branch
(no label, separator or closer left), where the marker has not started.  The policy
fixture (tests/golden/make_policy_cases.py) holds those sets as the reference Oracle
computed them in the reference's own test worlds.  CPU: the oracle reproduces the fixture,
and the engine's per-row logic (core.cuh, host seam) reproduces it and agrees with the
oracle at every step of every golden walk.  GPU: the logits the kernels write (apply_mask,
the sync_apply step and draft rows) against the fixture and against a float64 restatement
of the allowed mass."""

from __future__ import annotations

import gzip
import json
import math
from functools import cache

import numpy as np
import pytest

from tests.conftest import GOLDEN, golden_walks, make_oracle, start_state, unpack, world


@cache
def policy_cases():
    with gzip.open(GOLDEN / "policy_cases.json.gz", "rt", encoding="utf-8") as f:
        return json.load(f)


@cache
def policy_world(name: str):
    """(index, served tokenizer, syntax) of a fixture world."""
    from tokenizers import Tokenizer

    from xgraph_b200 import Entity, KnowledgeGraph, ServedTokenizer, SpanSyntax, build_kg_index
    from xgraph_b200.kg import Relation

    w = policy_cases()["worlds"][name]
    served = ServedTokenizer(Tokenizer.from_str(w["tokenizer"]))
    syntax = SpanSyntax(**w["syntax"])
    kg = KnowledgeGraph(tuple(Entity(i, tuple(ls)) for i, ls in w["entities"]),
                        tuple(Relation(i, tuple(ls)) for i, ls in w["relations"]),
                        tuple(tuple(t) for t in w["triples"]))
    return build_kg_index(kg, served, syntax), served, syntax


def policy_sets(oracle, state, pieces) -> tuple[set, set]:
    """(released, committing) tokens of an oracle state, as the reference's tests define
    them; only allowed tokens whose bytes are a piece of the escape marker can be released,
    so only those are advanced."""
    from oracle.oracle import Phase

    released, commits = set(), set()
    for token in oracle.allowed(state) & pieces:
        after = oracle.advance(state, token)
        if after.phase is Phase.ESCAPED or (after.phase is Phase.SPAN and after.escaping):
            released.add(token)
            if after.phase is Phase.ESCAPED or (
                    after.typed is None and after.separating is None and after.closing is None):
                commits.add(token)
    return released, commits


def escape_pieces(served, syntax) -> set[int]:
    """Tokens whose bytes occur in the escape marker (a superset of every released set)."""
    marker = syntax.escape.encode("utf-8")
    return {t for t in range(served.vocab_size) if (b := served.token_bytes(t)) and b in marker}


def expected_policy(case) -> tuple[set, set]:
    """(released, biased) tokens of a fixture case: the bias only where the marker has not
    started."""
    return set(case["released"]), set() if case["escaping"] else set(case["commits"])


# ------------------------------------------------------------------------------------ CPU

def test_oracle_reproduces_the_policy_cases():
    from oracle.oracle import Oracle

    for case in policy_cases()["cases"]:
        index, served, syntax = policy_world(case["world"])
        oracle = Oracle(index, served, syntax)
        state = oracle.initial_state()
        for token in case["tokens"]:
            state = oracle.advance(state, token)
        assert sorted(oracle.allowed(state)) == case["allowed"], case["test"]
        released, commits = policy_sets(oracle, state, escape_pieces(served, syntax))
        assert (sorted(released), sorted(commits)) == (case["released"], case["commits"]), case["test"]
        if "expected_bias" in case:  # the reference test's own expectation
            assert commits == set(case["expected_bias"])


def test_seam_reproduces_the_policy_cases():
    from tests.seam import SeamEngine

    for case in policy_cases()["cases"]:
        index, served, syntax = policy_world(case["world"])
        seam = SeamEngine(index, served, syntax, 1)
        seam.begin(0)
        for token in case["tokens"]:
            seam.advance([token])
        assert sorted(unpack(seam.masks()[0], served.vocab_size)) == case["allowed"], case["test"]
        pos, commits, released = seam.escape_policy(0)
        want_released, want_bias = expected_policy(case)
        assert (pos >= 0) == bool(want_released), case["test"]
        assert released == want_released and commits == want_bias, case["test"]


@pytest.mark.parametrize("name", [c["name"] for c in golden_walks() if c["options"].get("escapes", True)])
def test_seam_policy_agrees_with_the_oracle_on_every_golden_walk(name):
    """At every step of every sequence inside a span: the released set and the committing
    tokens of the engine's logic equal the oracle's (most span steps of every walk release,
    and most of those bias)."""
    seen = seam_policy_walk(name)
    assert seen["span"] > 0 and seen["released"] > 0 and seen["biased"] > 0, seen


def seam_policy_walk(name: str) -> dict:
    from oracle.oracle import Phase
    from tests.test_seam_golden import seam_for
    from xgraph_b200.syntax import SpanSyntax

    case = next(c for c in golden_walks() if c["name"] == name)
    seam, _ = seam_for(case)
    oracle = make_oracle(case)
    _, served, _ = world(case["world"])
    pieces = escape_pieces(served, SpanSyntax())
    sequences = case["sequences"]
    states = []
    for k, seq in enumerate(sequences):
        seam.begin(k)
        seam.set_version(k, seq["version"])
        if seq["anchor"]:
            seam.anchor(k, seq["anchor"])
        if seq["opened"]:
            seam.open_span(k)
        states.append(start_state(oracle, seq))
    seen = {"span": 0, "released": 0, "biased": 0}
    steps = len(sequences[0]["tokens"])
    for step in range(steps + 1):
        for k, state in enumerate(states):
            pos, commits, released = seam.escape_policy(k)
            if state.phase is not Phase.SPAN:
                assert pos == -1 and not commits, (name, k, step)
                continue
            want_released, want_commits = policy_sets(oracle, state, pieces)
            if state.escaping:
                want_commits = set()
            assert released == want_released, (name, k, step)
            assert (pos >= 0) == bool(want_released), (name, k, step)
            assert commits == want_commits, (name, k, step)
            seen["span"] += 1
            seen["released"] += bool(released)
            seen["biased"] += bool(commits)
        if step < steps:
            tokens = [seq["tokens"][step] for seq in sequences]
            seam.advance(tokens)
            states = [oracle.advance(s, t) for s, t in zip(states, tokens)]
    return seen


def test_release_needs_escapes_and_a_mass_below_one():
    """The reference's constructor checks (src/xgraph/engine.py:765-768), raised before any
    device work."""
    from xgraph_b200.engine import Engine, EngineUnavailable

    index, served, syntax = policy_world("toy")
    try:
        with pytest.raises(ValueError, match="escape"):
            Engine(index, served, syntax, 1, escapes=False, release_top=True)
        with pytest.raises(ValueError, match="escape"):
            Engine(index, served, syntax, 1, escapes=False, release_mass=0.5)
        for mass in (-0.1, 1.0, 2.0):
            with pytest.raises(ValueError, match="release_mass"):
                Engine(index, served, syntax, 1, release_mass=mass)
    except EngineUnavailable:
        pytest.skip("the engine library is not built")


def release_reference(logits: np.ndarray, allowed: set[int], vocab: int, log_mass: float, top: bool) -> tuple[bool, float]:
    """Float64 restatement of the reference's release test (csrc/engine.cu:2479-2552): the
    row's log allowed mass over the served vocabulary, and whether the row is released."""
    x = logits[:vocab].astype(np.float64)
    best = x.max()
    if not math.isfinite(best):
        return False, 0.0
    e = np.exp(x - best)
    ok = np.zeros(vocab, dtype=bool)
    ok[list(allowed)] = True
    mass = math.log(e[ok].sum()) - math.log(e.sum()) if ok.any() else -math.inf
    top_allowed = bool(ok[int(np.argmax(x))])
    return (top and not top_allowed) or mass < log_mass, mass


def test_release_reference_matches_the_reference_tests_mass():
    """The restatement on the reference test's own logits (tests/test_engine.py:2527-2533):
    three tenths of the probability on the allowed set."""
    allowed = {3, 5, 7}
    vocab = 20
    logits = np.full(vocab, -1e4, dtype=np.float32)
    logits[sorted(allowed)] = math.log(0.3 / 3)
    logits[11] = math.log(0.7)
    released, mass = release_reference(logits, allowed, vocab, math.log(0.5), False)
    assert released and mass == pytest.approx(math.log(0.3), abs=1e-6)
    assert not release_reference(logits, allowed, vocab, math.log(0.2), False)[0]
    assert release_reference(logits, allowed, vocab, -math.inf, True)[0]
    logits[11] = -1e4
    assert not release_reference(logits, allowed, vocab, -math.inf, True)[0]


# ------------------------------------------------------------------------------------ GPU

def begin_walk(engine, tokens_per_slot: dict[int, list[int]]):
    """Begin the slots and sync each over its tokens (history rows on the GPU)."""
    import torch

    slots = sorted(tokens_per_slot)
    width = max(8, max(len(t) for t in tokens_per_slot.values()))
    history = torch.zeros((engine.max_sequences, width), dtype=torch.int32, device="cuda")
    total = torch.zeros(engine.max_sequences, dtype=torch.int32, device="cuda")
    for slot, tokens in tokens_per_slot.items():
        if tokens:
            history[slot, : len(tokens)] = torch.tensor(tokens, dtype=torch.int32)
        total[slot] = len(tokens)
    device_slots = torch.tensor(slots, dtype=torch.int32, device="cuda")
    engine.begin(device_slots)
    engine.sync(device_slots, history, torch.zeros_like(total), total)
    return history, total


def kept(logits_row, vocab: int) -> set[int]:
    import torch

    return set(torch.nonzero(~torch.isneginf(logits_row[:vocab].float())).flatten().tolist())


@pytest.mark.gpu
@pytest.mark.parametrize("world_name", ["bias_plain", "bias_shared"])
@pytest.mark.parametrize("bias", [-3.0, -0.5])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_escape_bias_logits(world_name, bias, dtype):
    """After the opener, every allowed logit keeps its value except the committing tokens',
    which gain the bias (16-bit: rounded to nearest); grown, reused and grown row counts
    across a CTA boundary, with padding so that the logits stride differs from the
    vocabulary (the reference's tests/test_engine.py:4198-4235)."""
    import torch

    from xgraph_b200.engine import Engine

    index, served, syntax = policy_world(world_name)
    case = next(c for c in policy_cases()["cases"] if c["world"] == world_name)
    biased, allowed = set(case["expected_bias"]), set(case["allowed"])
    engine = Engine(index, served, syntax, 1, escape_bias=bias)
    begin_walk(engine, {0: case["tokens"]})
    torch_dtype = getattr(torch, dtype)
    vocab = served.vocab_size
    for rows in (1, 3, 2, 129):
        bases = [(1.25, 3.5, -1.75)[row % 3] for row in range(rows)]
        storage = torch.tensor([[b] * (vocab + 3) for b in bases], device="cuda").to(torch_dtype)
        logits = storage[:, :vocab]
        engine.apply_mask(logits, torch.zeros(rows, dtype=torch.int32, device="cuda"))
        expected = torch.tensor(
            [[(b + bias if t in biased else b) if t in allowed else -math.inf for t in range(vocab)] for b in bases],
            dtype=torch.float32).to(torch_dtype)  # the sum in fp32, rounded once to the logits' type
        assert torch.equal(logits.cpu(), expected)
        assert torch.equal(storage[:, vocab:].cpu(), torch.tensor([[b] * 3 for b in bases]).to(torch_dtype))
    assert engine.faults() == 0


@pytest.mark.gpu
@pytest.mark.parametrize(
    ("release", "favourite", "released"),
    [
        ({"release_top": True}, "disallowed", True),
        ({"release_top": True}, "allowed", False),
        ({"release_mass": 0.5}, "disallowed", True),  # the allowed mass is about 0.3
        ({"release_mass": 0.2}, "disallowed", False),
        ({}, "disallowed", False),
    ],
)
@pytest.mark.parametrize("path", ["apply_mask", "sync_apply", "drafts"])
def test_rows_with_high_rejected_mass_are_released_to_the_escape(release, favourite, released, path):
    """The reference's tests/test_engine.py:2498-2546 on its toy world: a row inside a span
    with three tenths of its probability on the allowed set, the rest on one token, is
    released (to the escape marker's next tokens) or not; a row in free text never is.
    Through apply_mask, the fused sync_apply step and draft rows at offset 0."""
    import torch

    from xgraph_b200.engine import Engine

    index, served, syntax = policy_world("toy")
    span, _, free = [c for c in policy_cases()["cases"] if c["world"] == "toy"]
    assert span["text"].endswith("Marie") and free["phase"] == "FREE"
    engine = Engine(index, served, syntax, 2, **release)
    vocab = served.vocab_size
    allowed = set(span["allowed"])
    disallowed = next(t for t in range(vocab) if t not in allowed)
    logits = torch.full((2, vocab), -1e4, device="cuda")
    logits[:, sorted(allowed)] = math.log(0.3 / len(allowed))
    top = disallowed if favourite == "disallowed" else min(allowed)
    logits[:, top] = math.log(0.7) if favourite == "disallowed" else math.log(0.7 + 0.3 / len(allowed))
    slots = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    if path == "sync_apply":
        history, total = begin_walk(engine, {0: [], 1: []})
        for slot, case in ((0, span), (1, free)):
            history[slot, : len(case["tokens"])] = torch.tensor(case["tokens"], dtype=torch.int32)
            total[slot] = len(case["tokens"])
        engine.sync_apply(slots, history, torch.zeros_like(total), total, logits)
    else:
        begin_walk(engine, {0: span["tokens"], 1: free["tokens"]})
        if path == "drafts":
            zero = torch.zeros(2, dtype=torch.int32, device="cuda")
            engine.apply_mask(logits, slots, local_pos=zero, input_ids=zero)
        else:
            engine.apply_mask(logits, slots)
    expected = set(span["released"]) if released else allowed
    assert kept(logits[0], vocab) == expected
    assert (expected and expected != allowed) or not released
    assert kept(logits[1], vocab) == set(free["allowed"])  # free text is never released
    # the slot's recorded mask is the ordinary one: release is per call
    engine.fill_mask()
    assert unpack(engine.mask_host().view(np.uint32)[0], vocab) == allowed
    assert engine.faults() == 0


@pytest.mark.gpu
def test_a_started_escape_marker_is_released_to_its_continuation():
    """The reference's tests/test_engine.py:2559-2581: after the opener, "Bra" and the first
    two bytes of the escape marker (which also continue the label "Bra⁄"), a released row
    keeps only the byte that completes the marker."""
    import torch

    from xgraph_b200.engine import Engine

    index, served, syntax = policy_world("hand")
    case = next(c for c in policy_cases()["cases"] if c["world"] == "hand")
    assert case["escaping"] and len(case["allowed"]) == 2
    engine = Engine(index, served, syntax, 1, release_top=True)
    begin_walk(engine, {0: case["tokens"]})
    vocab = served.vocab_size
    logits = torch.zeros((1, vocab), device="cuda")
    logits[0, next(t for t in range(vocab) if t not in case["allowed"])] = 50.0
    engine.apply_mask(logits, torch.zeros(1, dtype=torch.int32, device="cuda"))
    assert kept(logits[0], vocab) == set(case["released"])
    assert engine.faults() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["toy_ordinary", "bpe_paths", "crowd_committed", "bytes_derivation"])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("path", ["apply_mask", "sync_apply"])
def test_release_and_bias_agree_with_the_oracle_along_golden_walks(name, dtype, path):
    """Every step of a golden walk, every sequence, random logits whose allowed columns are
    lifted by a random amount per row (so that the allowed mass spreads over (0, 1)): the
    row the kernels write equals the one built from the oracle's allowed, released and
    committing sets and the float64 mass of the biased logits.  Rows whose mass lies within
    1e-4 of the threshold (where float32 sums may round either way) may take either side.
    Through advance + apply_mask (the row kernel), and through one fused sync_apply step per
    token (rows already in a span take their mass while the state machine runs)."""
    import torch

    from oracle.oracle import Phase
    from tests.conftest import case_index, case_options, case_versions
    from xgraph_b200.engine import Engine
    from xgraph_b200.kgversions import build_kg_versions
    from xgraph_b200.syntax import SpanSyntax

    case = next(c for c in golden_walks() if c["name"] == name)
    _, served, _ = world(case["world"])
    index = case_index(case)
    edits = case_versions(case)
    versions = build_kg_versions(index, edits) if edits else None
    bias, threshold = -0.75, 0.35
    engine = Engine(index, served, SpanSyntax(), len(case["sequences"]), versions=versions,
                    release_mass=threshold, escape_bias=bias, **case_options(case))
    oracle = make_oracle(case)
    pieces = escape_pieces(served, SpanSyntax())
    sequences = case["sequences"]
    n, vocab = len(sequences), served.vocab_size
    slots = torch.arange(n, dtype=torch.int32, device="cuda")
    engine.begin(slots)
    states = []
    for k, seq in enumerate(sequences):
        if seq["version"] is not None:
            engine.set_version(k, seq["version"])
        if seq["anchor"]:
            engine.anchor(k, seq["anchor"])
        if seq["opened"]:
            engine.open_span(k)
        states.append(start_state(oracle, seq))
    rng = np.random.default_rng(7)
    torch_dtype = getattr(torch, dtype)
    seen = {"released": 0, "kept": 0, "near": 0, "biased": 0}
    steps = len(sequences[0]["tokens"])
    history = torch.tensor([seq["tokens"] for seq in sequences], dtype=torch.int32, device="cuda")
    zeros = torch.zeros(n, dtype=torch.int32, device="cuda")
    for step in range(steps + 1):
        allowed = [oracle.allowed(state) for state in states]
        raw = rng.normal(0.0, 2.0, (n, vocab)).astype(np.float32)
        for k in range(n):
            raw[k, sorted(allowed[k])] += rng.uniform(-1.0, 9.0)
        logits = torch.from_numpy(raw).to(torch_dtype)
        before = logits.float().numpy()
        device = logits.cuda()
        if path == "sync_apply":  # the step's token (the previous one) consumed in the same launch
            engine.sync_apply(slots, history, zeros, torch.full_like(zeros, step), device)
        else:
            engine.apply_mask(device, slots)
        got = device.cpu().float().numpy()
        for k, state in enumerate(states):
            released, commits = policy_sets(oracle, state, pieces) if state.phase is Phase.SPAN else (set(), set())
            if state.escaping:
                commits = set()
            row = before[k].copy()
            for t in commits:  # the bias in fp32, rounded once to the logits' type
                row[t] = torch.tensor(float(np.float32(row[t]) + np.float32(bias))).to(torch_dtype).float().item()
            outcomes = [False]
            if released:
                release, mass = release_reference(row, allowed[k], vocab, math.log(threshold), False)
                near = abs(mass - math.log(threshold)) < 1e-4
                outcomes = [False, True] if near else [release]
                seen["near"] += near
            matches = []
            for outcome in outcomes:
                keep = sorted(released if outcome else allowed[k])
                want = np.full(vocab, -np.inf, dtype=np.float32)
                want[keep] = row[keep]
                matches.append(np.array_equal(got[k], want))
            assert any(matches), (name, step, k, outcomes)
            seen["released"] += outcomes == [True]
            seen["kept"] += bool(released) and outcomes == [False]
            seen["biased"] += bool(commits)
        if step < steps:
            tokens = [seq["tokens"][step] for seq in sequences]
            if path == "apply_mask":
                engine.advance(np.array(tokens, dtype=np.int32))
            states = [oracle.advance(s, t) for s, t in zip(states, tokens)]
    assert engine.faults() == 0
    assert seen["released"] > 0 and seen["kept"] > 0 and seen["biased"] > 0, seen


_WORKER = {}


def _policy_worker_init(index, served, syntax, options):
    from oracle.oracle import Oracle

    _WORKER["oracle"] = Oracle(index, served, syntax, **options)
    _WORKER["pieces"] = escape_pieces(served, syntax)


def _policy_sets_after(prefix):
    """The oracle after a token prefix: (allowed, released, committing, in a span, the
    escape marker started)."""
    from oracle.oracle import Phase

    oracle = _WORKER["oracle"]
    state = oracle.initial_state()
    for token in prefix:
        state = oracle.advance(state, int(token))
    span = state.phase is Phase.SPAN
    released, commits = policy_sets(oracle, state, _WORKER["pieces"]) if span else (set(), set())
    return sorted(oracle.allowed(state)), sorted(released), sorted(commits), span, bool(state.escaping)


@pytest.mark.gpu
def test_policies_agree_with_the_oracle_at_the_path_benchmark_size():
    """paths-100k (config 3: 100 k entities, 1 M triples, V = 128,256), 64 rows of GPU-sampled
    streams replayed through the fused step one token per step with release (0.35) and
    escape bias (-0.75) on, bf16 logits.  Every row at every step keeps each column's logit
    bit for bit, takes exactly the biased value, or becomes -inf.  At 48 seeded (row, step)
    samples, 40 of them inside spans, the written row equals the one built from the
    oracle's allowed, released and committing sets and a float64 mass of the biased logits
    (the sampled rows' allowed columns lifted by a seeded amount so that masses spread
    around the threshold; either side within 1e-4 of it)."""
    import multiprocessing as mp

    import torch

    from xgraph_b200.engine import Engine
    from xgraph_b200.synthetic import build_workload, sample_streams

    rows, steps, bias, threshold = 64, 96, -0.75, 0.35
    w = build_workload(3)
    syntax, options, vocab = w.syntax, dict(w.config.options), w.served.vocab_size
    sampler = Engine(w.index, w.served, syntax, rows, **options)
    tokens, _, _ = sample_streams(sampler, w.served, syntax, w.world, rows, steps, seed=103)
    slots = torch.arange(rows, dtype=torch.int32, device="cuda")
    prompt = torch.zeros(rows, dtype=torch.int32, device="cuda")
    # which (row, step) pairs are in a span: a replay without the policies
    sampler.reset()
    sampler.begin(slots)
    phases = []
    for k in range(steps + 1):
        sampler.sync(slots, tokens, prompt, torch.full((rows,), k, dtype=torch.int32, device="cuda"))
        phases.append(sampler.states_host(rows)["phase"].copy())
    del sampler
    rng = np.random.default_rng(17)
    span_pairs = [(r, k) for k in range(steps + 1) for r in range(rows) if phases[k][r] == 1]
    free_pairs = [(r, k) for k in range(steps + 1) for r in range(rows) if phases[k][r] != 1]
    picks = [span_pairs[i] for i in rng.choice(len(span_pairs), 40, replace=False)]
    picks += [free_pairs[i] for i in rng.choice(len(free_pairs), 8, replace=False)]
    host_tokens = tokens.cpu().numpy()
    with mp.get_context("spawn").Pool(8, initializer=_policy_worker_init,
                                      initargs=(w.index, w.served, syntax, options)) as pool:
        expected = dict(zip(picks, pool.map(_policy_sets_after, [host_tokens[r, :k] for r, k in picks],
                                            chunksize=1)))
    engine = Engine(w.index, w.served, syntax, rows, release_mass=threshold, escape_bias=bias, **options)
    engine.reset()
    engine.begin(slots)
    seen = {"released": 0, "kept": 0, "near": 0, "biased": 0, "free": 0}
    for k in range(steps + 1):
        raw = rng.normal(0.0, 2.0, (rows, vocab)).astype(np.float32)
        for (r, kk), (allowed, *_rest) in expected.items():
            if kk == k:
                raw[r, allowed] += rng.uniform(4.0, 14.0)
        before_t = torch.from_numpy(raw).to(torch.bfloat16)
        logits = before_t.cuda()
        engine.sync_apply(slots, tokens, prompt, torch.full((rows,), k, dtype=torch.int32, device="cuda"), logits)
        got = logits.cpu()
        before = before_t.float().numpy()
        got_f = got.float().numpy()
        biased = torch.tensor(before + np.float32(bias)).to(torch.bfloat16).float().numpy()
        ok = (got.view(torch.int16) == before_t.view(torch.int16)).numpy() | np.isneginf(got_f) | (got_f == biased)
        assert ok.all(), ("a column is neither its logit, its biased logit nor -inf", k)
        for (r, kk), (allowed, released, commits, span, escaping) in expected.items():
            if kk != k:
                continue
            commits = set() if escaping else set(commits)
            row = before[r].copy()
            for t in commits:
                row[t] = biased[r, t]
            outcomes = [False]
            if released:
                release, mass = release_reference(row, set(allowed), vocab, math.log(threshold), False)
                near = abs(mass - math.log(threshold)) < 1e-4
                outcomes = [False, True] if near else [release]
                seen["near"] += near
            matches = []
            for outcome in outcomes:
                keep = sorted(released if outcome else allowed)
                want = np.full(vocab, -np.inf, dtype=np.float32)
                want[keep] = row[keep]
                matches.append(np.array_equal(got_f[r], want))
            assert any(matches), (r, k, outcomes, span)
            seen["released"] += outcomes == [True]
            seen["kept"] += bool(released) and outcomes == [False]
            seen["biased"] += bool(commits)
            seen["free"] += not span
    assert engine.errors() == 0 and engine.faults() == 0
    assert seen["released"] > 0 and seen["kept"] > 0 and seen["biased"] > 0 and seen["free"] == 8, seen
