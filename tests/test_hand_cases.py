"""The reference's hand-worked oracle cases (its tests/test_oracle.py:2491-2556: opener split
across tokens, a token completing the opener before its end, end of text only outside
spans, the closer only after a complete label, one token serving a label and the closer or
the escape marker, the closer ending at a token boundary, escapes), as golden walks the
reference Oracle recorded (tests/golden/make_hand_cases.py).  The oracle (CPU) and the CUDA
engine through the C ABI (GPU) must reproduce every state and every allowed set."""

from __future__ import annotations

import gzip
import json
from functools import cache

import numpy as np
import pytest

from tests.conftest import GOLDEN, state_record, unpack


@cache
def hand():
    with gzip.open(GOLDEN / "hand_cases.json.gz", "rt", encoding="utf-8") as f:
        return json.load(f)


def hand_world():
    from tokenizers import Tokenizer

    from xgraph_b200 import Entity, KnowledgeGraph, ServedTokenizer, SpanSyntax, build_kg_index

    data = hand()
    served = ServedTokenizer(Tokenizer.from_str(data["tokenizer"]))
    syntax = SpanSyntax(**data["syntax"])
    kg = KnowledgeGraph(tuple(Entity(i, tuple(labels)) for i, labels in data["entities"]), (), ())
    return build_kg_index(kg, served, syntax), served, syntax


def test_the_walks_pin_what_the_reference_tests_assert():
    """The fixture holds the situations the reference's tests name (a sanity check of the
    recorded walks themselves)."""
    data = hand()
    probe = data["probes"]
    by_test = {}
    for w in data["walks"]:
        by_test.setdefault(w["test"], []).append(w)
    assert by_test["test_opener_split_across_tokens_opens_a_span"][0]["final"]["phase"] == "span"
    assert probe["âŁ¦y"] not in by_test["test_token_that_completes_the_opener_before_its_end_is_not_allowed"][0]["allowed"][0]
    eos = probe["<|endoftext|>"]
    walk = by_test["test_end_of_text_is_allowed_only_outside_spans"][0]
    assert eos in walk["allowed"][0] and eos not in walk["allowed"][1] and eos not in walk["final_allowed"]
    walk = by_test["test_closer_is_allowed_only_after_a_complete_label"][0]
    assert probe["âŁ§"] not in walk["allowed"][1] and probe["âŁ§"] in walk["allowed"][2]
    assert probe["âŁ§"] not in walk["final_allowed"]
    short, long = by_test["test_a_token_can_both_continue_a_label_and_start_the_closer"]
    assert short["final"]["last_span"]["entity_ids"] == ["Q1"] and long["final"]["last_span"]["entity_ids"] == ["Q2"]
    walk = by_test["test_closer_must_end_at_a_token_boundary"][0]
    assert probe["âŁ§y"] not in walk["final_allowed"]
    assert by_test["test_escape_turns_the_rest_of_the_span_into_free_text"][0]["final"]["phase"] == "escaped"


def test_oracle_reproduces_the_hand_walks():
    from oracle.oracle import Oracle

    index, served, syntax = hand_world()
    oracle = Oracle(index, served, syntax)
    for w in hand()["walks"]:
        state = oracle.initial_state()
        for k, token in enumerate(w["tokens"]):
            assert state_record(state) == w["states"][k], (w["pieces"], k)
            assert sorted(oracle.allowed(state)) == w["allowed"][k], (w["pieces"], k)
            state = oracle.advance(state, token)
        assert state_record(state) == w["final"], w["pieces"]
        assert sorted(oracle.allowed(state)) == w["final_allowed"], w["pieces"]


@pytest.mark.gpu
def test_engine_reproduces_the_hand_walks():
    """Every step's mask (one slot per walk, all walks advanced together, finished walks
    re-begun) and the final closed spans, through the C ABI."""
    import torch

    from tests.agreement import assert_agrees, engine_state, expected_state
    from xgraph_b200.engine import Engine

    index, served, syntax = hand_world()
    walks = hand()["walks"]
    n = len(walks)
    engine = Engine(index, served, syntax, n)
    engine.reset()
    engine.begin(torch.arange(n, dtype=torch.int32, device="cuda"))
    longest = max(len(w["tokens"]) for w in walks)
    for k in range(longest + 1):
        engine.fill_mask()
        masks = engine.mask_host().view(np.uint32)
        states = engine.states_host()
        for j, w in enumerate(walks):
            if k > len(w["tokens"]):
                continue
            record = w["states"][k] if k < len(w["tokens"]) else w["final"]
            allowed = w["allowed"][k] if k < len(w["tokens"]) else w["final_allowed"]
            assert sorted(unpack(masks[j], served.vocab_size)) == allowed, (w["pieces"], k)
            assert_agrees(expected_state(record, index, syntax), engine_state(states, j, index), False,
                          (w["pieces"], k))
        if k < longest:
            step = [w["tokens"][k] if k < len(w["tokens"]) else w["tokens"][-1] for w in walks]
            done = [j for j, w in enumerate(walks) if k >= len(w["tokens"])]
            engine.advance(np.array(step, dtype=np.int32))
            if done:  # walks already finished are begun again (their checks are over)
                engine.begin(torch.tensor(done, dtype=torch.int32, device="cuda"))
    assert engine.faults() == 0
