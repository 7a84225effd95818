"""Golden fixture of apply_mask's logit policies (release and escape bias), recorded with
the reference itself.

Run in a container that holds the reference checkout (imported read-only, no bytecode):

    python tests/golden/make_policy_cases.py --reference <reference checkout>

policy_cases.json.gz records, from the reference's own test worlds and its Oracle:
- the escape-bias worlds of its tests/test_engine_cpu.py:247-264 (an escape marker
  "abcdefghij" every prefix of which is a token, beside a label that shares none, or two,
  of those prefixes), with the tokens its tests expect the bias on after the opener;
- the span situations of its tests/test_engine.py:2487-2546, 2559-2581 and 2694-2735 (the
  toy world inside a span, mid-label and after a complete label, and in free text; the hand
  world after the escape marker has started beside a label).
For every walk it stores the tokens, the Oracle's allowed set after them, the released set
(the allowed tokens after which the escape marker is being typed or complete,
tests/test_engine.py:2487-2495) and the committing set (those of them that end every other
branch: no label, separator or closer left, tests/test_engine.py:2718-2726), as the
reference's tests define them.
"""

from __future__ import annotations

import argparse
import gzip
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent

TOY_TEXTS = [" She met ⟦ Marie", " She met ⟦ Marie Curie", " She met"]
HAND_PIECES = ["âŁ¦", "Bra", "âģ"]
BIAS_ESCAPE = "abcdefghij"


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True, help="the reference checkout")
    args = parser.parse_args()
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(args.reference / "src"), str(args.reference)]

    from tests.conftest import (  # the reference's own tests package
        TOY_ENTITIES, TOY_RELATIONS, TOY_TEXT, TOY_TRIPLES, byte_level_tokenizer, train_byte_level_bpe)
    from tests.test_engine_cpu import escape_bias_world
    from tests.test_oracle import HAND_ENTITIES, HAND_SYNTAX, MERGES
    from xgraph.index import build_kg_index
    from xgraph.kg import Entity, KnowledgeGraph, Relation
    from xgraph.oracle import Oracle, Phase
    from xgraph.syntax import SpanSyntax
    from xgraph.tokenizer import ServedTokenizer

    def sets(oracle, state):
        allowed = oracle.allowed(state)
        released, commits = set(), set()
        for token in allowed:
            after = oracle.advance(state, token)
            if after.phase is Phase.ESCAPED or (after.phase is Phase.SPAN and after.escaping):
                released.add(token)
                if after.phase is Phase.ESCAPED or (
                    after.typed is None and after.separating is None and after.closing is None
                ):
                    commits.add(token)
        return {"allowed": sorted(allowed), "released": sorted(released), "commits": sorted(commits),
                "phase": state.phase.name, "escaping": state.escaping is not None and len(state.escaping) > 0}

    def walk(oracle, tokens, state=None):
        state = oracle.initial_state() if state is None else state
        for token in tokens:
            state = oracle.advance(state, token)
        return state

    def syntax_record(syntax):
        return {"opener": syntax.opener, "label_prefix": syntax.label_prefix, "separator": syntax.separator,
                "closer": syntax.closer, "escape": syntax.escape}

    worlds, cases = {}, []
    # the escape-bias worlds: the expected tokens are the reference tests' own
    merges = [(BIAS_ESCAPE[: k - 1], BIAS_ESCAPE[k - 1]) for k in range(2, len(BIAS_ESCAPE) + 1)]
    for shared in (False, True):
        index, served, syntax, expected = escape_bias_world(shared)
        name = f"bias_{'shared' if shared else 'plain'}"
        # the world escape_bias_world builds (its labels), checked against its index
        entities = [["item", ["abacus" if shared else "Atlas"]]] + ([["other", ["az"]]] if shared else [])
        rebuilt = build_kg_index(KnowledgeGraph(tuple(Entity(i, tuple(ls)) for i, ls in entities), (), ()),
                                 served, syntax)
        assert rebuilt.labels.num_rows == index.labels.num_rows
        worlds[name] = {"tokenizer": byte_level_tokenizer(merges).to_str(), "entities": entities,
                        "relations": [], "triples": [], "syntax": syntax_record(syntax)}
        oracle = Oracle(index, served, syntax)
        tokens = served.encode(syntax.opener)
        record = sets(oracle, walk(oracle, tokens))
        assert set(record["commits"]) == expected, (name, record["commits"], expected)
        cases.append({"world": name, "tokens": tokens, "test": "test_escape_bias_covers_more_than_eight_prefix_tokens",
                      "expected_bias": sorted(expected), **record})
    # the toy world (the reference's toy_kg and toy_tokenizer fixtures)
    labels = [label for _, labels in TOY_ENTITIES + TOY_RELATIONS for label in labels]
    toy_tokenizer = train_byte_level_bpe(labels + list(TOY_TEXT), vocab_size=400)  # the toy_tokenizer fixture
    served = ServedTokenizer(toy_tokenizer)
    kg = KnowledgeGraph(entities=tuple(Entity(id=i, labels=ls) for i, ls in TOY_ENTITIES),
                        relations=tuple(Relation(id=i, labels=ls) for i, ls in TOY_RELATIONS),
                        triples=TOY_TRIPLES)
    worlds["toy"] = {"tokenizer": toy_tokenizer.to_str(), "entities": [[i, list(ls)] for i, ls in TOY_ENTITIES],
                     "relations": [[i, list(ls)] for i, ls in TOY_RELATIONS],
                     "triples": [list(t) for t in TOY_TRIPLES], "syntax": syntax_record(SpanSyntax())}
    oracle = Oracle(build_kg_index(kg, served, SpanSyntax()), served, SpanSyntax())
    for text in TOY_TEXTS:
        tokens = served.encode(text)
        cases.append({"world": "toy", "tokens": tokens, "text": text,
                      "test": "test_rows_with_high_rejected_mass_are_released_to_the_escape",
                      **sets(oracle, walk(oracle, tokens))})
    # the hand world: the escape marker started beside the label "Bra⁄"
    hand_tokenizer = byte_level_tokenizer(MERGES)
    served = ServedTokenizer(hand_tokenizer)
    worlds["hand"] = {"tokenizer": hand_tokenizer.to_str(), "entities": [[e.id, list(e.labels)] for e in HAND_ENTITIES],
                      "relations": [], "triples": [], "syntax": syntax_record(HAND_SYNTAX)}
    oracle = Oracle(build_kg_index(KnowledgeGraph(entities=HAND_ENTITIES), served, HAND_SYNTAX), served, HAND_SYNTAX)
    tokens = [hand_tokenizer.token_to_id(p) for p in HAND_PIECES]
    record = sets(oracle, walk(oracle, tokens))
    assert record["released"] == [hand_tokenizer.token_to_id("ĩ")], record
    cases.append({"world": "hand", "tokens": tokens, "test": "test_a_started_escape_marker_is_released_to_its_continuation",
                  **record})
    with gzip.open(HERE / "policy_cases.json.gz", "wt", encoding="utf-8") as f:
        json.dump({"worlds": worlds, "cases": cases}, f, separators=(",", ":"))
    for c in cases:
        print(c["world"], c["test"], len(c["allowed"]), "allowed,", len(c["released"]), "released,",
              len(c["commits"]), "committing")


if __name__ == "__main__":
    main()
