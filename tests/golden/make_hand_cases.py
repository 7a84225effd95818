"""Golden fixture of the reference's hand-worked oracle cases (tests/test_oracle.py:2491-2556
of the reference: an opener split across tokens, a token that completes the opener before
its end, end of text only outside spans, the closer only after a complete label, one token
serving a label and the closer or the escape marker, the closer ending at a token boundary,
the escape marker turning the span into free text).

Run in a container that holds the reference checkout (imported read-only, no bytecode):

    python tests/golden/make_hand_cases.py --reference <reference checkout>

The hand world is the reference's own (its `hand` fixture, tests/test_oracle.py:854-890:
a byte-level tokenizer with nine hand-picked merges, the labels "Bra", "Bra⟩" and "Bra⁄",
no label prefix, escape marker "⁇").  Each walk below replays, through the reference
Oracle, one token sequence those tests walk (named after the test), recording at every
step the reference state and its whole allowed set; hand_cases.json.gz holds the world and
the walks.
"""

from __future__ import annotations

import argparse
import gzip
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent

# (test of the reference's tests/test_oracle.py it pins, token pieces of the walk)
WALKS = [
    ("test_opener_at_the_end_of_a_token_opens_a_span", ["x", "xâŁ¦"]),
    ("test_opener_split_across_tokens_opens_a_span", ["âŁ", "¦"]),
    ("test_opener_split_across_tokens_opens_a_span", ["â", "Ł", "¦"]),
    ("test_token_that_completes_the_opener_before_its_end_is_not_allowed", ["x"]),
    ("test_end_of_text_is_allowed_only_outside_spans", ["âŁ¦", "Bra"]),
    ("test_end_of_text_is_allowed_only_outside_spans", ["âŁ¦", "â", "ģ", "ĩ"]),
    ("test_closer_is_allowed_only_after_a_complete_label", ["âŁ¦", "Bra", "âŁ"]),
    ("test_a_token_can_both_continue_a_label_and_start_the_closer", ["âŁ¦", "Bra", "âŁ", "§"]),
    ("test_a_token_can_both_continue_a_label_and_start_the_closer", ["âŁ¦", "Bra", "âŁ", "©", "âŁ§"]),
    ("test_a_token_can_both_continue_a_label_and_start_the_escape_marker", ["âŁ¦", "Bra", "âģ", "ĩ"]),
    ("test_a_token_can_both_continue_a_label_and_start_the_escape_marker", ["âŁ¦", "Bra", "âģ", "Ħ", "âŁ§"]),
    ("test_closer_must_end_at_a_token_boundary", ["âŁ¦", "Bra"]),
    ("test_escape_turns_the_rest_of_the_span_into_free_text", ["âŁ¦", "Bra", "â", "ģ", "ĩ", "x", "y", "Br"]),
]
# single tokens whose allowance the reference tests probe after a walk prefix
PROBES = ["âŁ¦y", "âŁ§y", "âŁ§", "âģ", "<|endoftext|>"]


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True, help="the reference checkout")
    args = parser.parse_args()
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(args.reference / "src"), str(args.reference)]
    sys.path.insert(0, str(HERE))
    from make_golden import state_record  # noqa: E402  (the state encoding the other walks use)

    from tests.conftest import byte_level_tokenizer  # the reference's own tests package
    from tests.test_oracle import HAND_ENTITIES, HAND_SYNTAX, MERGES
    from xgraph.index import build_kg_index
    from xgraph.kg import KnowledgeGraph
    from xgraph.oracle import Oracle
    from xgraph.tokenizer import ServedTokenizer

    tokenizer = byte_level_tokenizer(MERGES)
    served = ServedTokenizer(tokenizer)
    oracle = Oracle(build_kg_index(KnowledgeGraph(entities=HAND_ENTITIES), served, HAND_SYNTAX), served, HAND_SYNTAX)
    walks = []
    for test, pieces in WALKS:
        tokens = [tokenizer.token_to_id(p) for p in pieces]
        assert None not in tokens, pieces
        state = oracle.initial_state()
        states, allowed = [], []
        for token in tokens:
            states.append(state_record(state))
            allowed.append(sorted(oracle.allowed(state)))
            state = oracle.advance(state, token)
        walks.append({"test": test, "pieces": pieces, "tokens": tokens, "states": states, "allowed": allowed,
                      "final": state_record(state), "final_allowed": sorted(oracle.allowed(state))})
    fixture = {
        "tokenizer": tokenizer.to_str(),
        "entities": [[e.id, list(e.labels)] for e in HAND_ENTITIES],
        "syntax": {"opener": HAND_SYNTAX.opener, "label_prefix": HAND_SYNTAX.label_prefix,
                   "separator": HAND_SYNTAX.separator, "closer": HAND_SYNTAX.closer, "escape": HAND_SYNTAX.escape},
        "probes": {p: tokenizer.token_to_id(p) for p in PROBES},
        "walks": walks,
    }
    with gzip.open(HERE / "hand_cases.json.gz", "wt", encoding="utf-8") as f:
        json.dump(fixture, f, separators=(",", ":"))
    print(f"{len(walks)} hand walks, vocabulary {served.vocab_size}")


if __name__ == "__main__":
    main()
