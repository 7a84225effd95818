"""The oracle restatement against the reference Oracle's own walks (golden vectors).

Every state along every golden walk, and every allowed set, must equal what the
reference's src/xgraph/oracle.py produced on the same KG, tokenizer, options and tokens.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import (
    golden_masks,
    golden_walks,
    make_oracle,
    start_state,
    state_record,
    unpack,
    world,
)

CASES = [case["name"] for case in golden_walks()]


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_walks(name):
    case = next(c for c in golden_walks() if c["name"] == name)
    oracle = make_oracle(case)
    vocab = world(case["world"])[1].vocab_size
    masks = golden_masks()
    for k, sequence in enumerate(case["sequences"]):
        state = start_state(oracle, sequence)
        expected_masks = masks[f"{name}/{k}"]
        for step, (token, expected) in enumerate(zip(sequence["tokens"], sequence["states"], strict=True)):
            assert state_record(state) == expected, (name, k, step)
            allowed = oracle.allowed(state)
            assert allowed == unpack(expected_masks[step], vocab), (name, k, step)
            state = oracle.advance(state, token)
        assert state_record(state) == sequence["final"], (name, k, "final")


def test_golden_walks_cover_every_closing_kind():
    kinds = set()
    for case in golden_walks():
        for sequence in case["sequences"]:
            for st in sequence["states"]:
                span = st["last_span"]
                if span is None:
                    continue
                if not span["resolved"]:
                    kinds.add("unresolved")
                elif span["triples"]:
                    kinds.add("fact")
                elif len(span["labels"]) > 1:
                    kinds.add("path")
                else:
                    kinds.add("entity")
                if st["answer_complete"]:
                    kinds.add("answer_complete")
    assert kinds == {"unresolved", "fact", "path", "entity", "answer_complete"}


def test_mask_fixture_words_match_vocabulary():
    for case in golden_walks():
        vocab = world(case["world"])[1].vocab_size
        for k in range(len(case["sequences"])):
            assert golden_masks()[f"{case['name']}/{k}"].shape[1] == (vocab + 31) // 32
            assert golden_masks()[f"{case['name']}/{k}"].dtype == np.uint32
