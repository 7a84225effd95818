"""Golden fixture of the weaker relation supports, recorded with the reference itself.

Run in a container that holds the reference checkout (imported read-only, no bytecode):

    python tests/golden/make_relation_cases.py --reference <reference checkout>

relation_cases.json.gz holds walks of the reference Oracle in path mode with committed
paths and relations="vocabulary" or "successor" (src/xgraph/oracle.py:67-79, 865-871,
1066-1077, 1138-1147, 1599-1605, 1809-1822): relation segments admit every relation
(vocabulary), or after the first relation only the successors of the preceding label's
relations in the walk's KG version (successor); no path is executed, a closed plan is
unresolved and the next span is its answer.  Every step records the reference state
(make_golden.state_record) and its whole allowed set.  Walks on four golden worlds of
worlds.json.gz (two of them with two KG versions each, the walks alternating base and
versions):

- path walks: the text of a span naming a start entity with triples and 1-4 random
  relation labels, written token by token; where the text's next token is not allowed the
  walk writes the closer if it may, else a random allowed token;
- random walks: the make_golden sampler (spans, separators, closers, escapes).
"""

from __future__ import annotations

import argparse
import gzip
import json
import os
import random
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
STEPS = 48
WORLDS = (("toy", True), ("rand_bpe", True), ("rand_dense", False), ("crowd", False))


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True, help="the reference checkout")
    args = parser.parse_args()
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(args.reference / "src"), str(args.reference)]
    sys.path.insert(0, str(HERE))
    from make_golden import _edits, _kg, _tokenizer, state_record  # noqa: E402

    from xgraph.index import build_kg_index
    from xgraph.oracle import Oracle, Phase, Segment
    from xgraph.syntax import SpanSyntax

    with gzip.open(HERE / "worlds.json.gz", "rt", encoding="utf-8") as f:
        worlds = json.load(f)

    cases = []
    for world_name, versioned in WORLDS:
        world = worlds[world_name]
        served, syntax = _tokenizer(world["tokenizer"]), SpanSyntax()
        as_tuple = (world["entities"], world["relations"], world["triples"], None, None)
        index = build_kg_index(_kg(as_tuple), served, syntax)
        edits = _edits(as_tuple, sum(map(ord, world_name)) + 3) if versioned else {}
        names = [None, *edits]
        ents = {e: labels for e, labels in world["entities"] if labels}
        rel_labels = [label for _, labels in world["relations"] for label in labels]
        subjects = sorted({s for s, _, _ in world["triples"] if s in ents})
        opener = served.encode(" " + syntax.opener)
        closer, separator = served.encode(syntax.closer), served.encode(syntax.separator)
        escape = served.encode(syntax.escape)
        regular = [t for t in range(served.vocab_size) if t not in served.special_ids]
        for mode in ("vocabulary", "successor"):
            oracle = Oracle(index, served, syntax, paths=True, committed_paths=True, relations=mode,
                            versions=edits or None)
            rng = random.Random(sum(map(ord, world_name + mode)))
            walks = []
            for n in range(12):
                version = names[n % len(names)]
                state = oracle.initial_state(version)
                if n < 8:  # a path walk
                    start = rng.choice(ents[rng.choice(subjects)])
                    hops = [rng.choice(rel_labels) for _ in range(rng.randint(1, 4))]
                    text = (" " + syntax.opener + syntax.label_prefix + start
                            + "".join(syntax.separator + syntax.label_prefix + r for r in hops) + syntax.closer)
                    queue, free = list(served.encode(text)), False
                else:
                    queue, free = [], True
                tokens, states, allowed_at = [], [], []
                for _ in range(STEPS):
                    allowed = oracle.allowed(state)
                    states.append(state_record(state))
                    allowed_at.append(sorted(allowed))
                    if free and not queue:
                        p = rng.random()
                        in_span = state.phase is Phase.SPAN
                        if state.phase is Phase.FREE and p < 0.3:
                            queue = list(opener)
                        elif in_span and separator[0] in allowed and p < 0.6:
                            queue = list(separator)
                        elif in_span and closer[0] in allowed and p < 0.85 and (
                                state.segment is not Segment.SUBJECT or rng.random() < 0.5):
                            queue = list(closer)
                        elif in_span and p > 0.97:
                            queue = list(escape)
                        elif state.phase is Phase.ESCAPED and p < 0.45:
                            queue = list(closer)
                    if queue and queue[0] in allowed:
                        token = queue.pop(0)
                    elif queue and not free and closer[0] in allowed:
                        queue = list(closer)
                        token = queue.pop(0)
                    else:
                        queue = []
                        pool = sorted(allowed & set(regular)) or sorted(allowed)
                        token = rng.choice(pool)
                    tokens.append(token)
                    state = oracle.advance(state, token)
                walks.append({"version": version, "tokens": tokens, "states": states, "allowed": allowed_at,
                              "final": state_record(state), "final_allowed": sorted(oracle.allowed(state))})
            cases.append({"world": world_name, "mode": mode,
                          "versions": {k: [list(e) for e in v] for k, v in edits.items()}, "walks": walks})
    plans = sum(1 for c in cases for w in c["walks"] for s in [*w["states"], w["final"]]
                if s["last_span"] and not s["last_span"]["resolved"] and s["last_span"]["labels"])
    relation_states = sum(1 for c in cases for w in c["walks"] for s in w["states"]
                          if s["phase"] == "span" and s["segment"] == "relation")
    with gzip.open(HERE / "relation_cases.json.gz", "wt", encoding="utf-8") as f:
        json.dump({"cases": cases}, f, separators=(",", ":"))
    print(f"{sum(len(c['walks']) for c in cases)} walks, {relation_states} relation-segment states, "
          f"{plans} states after a closed plan")


if __name__ == "__main__":
    main()
