"""Golden fixture of residual-goal STOP, recorded with the reference itself.

Run in a container that holds the reference checkout (imported read-only, no bytecode):

    python tests/golden/make_stop_cases.py --reference <reference checkout>

stop_cases.json.gz holds walks of the reference Oracle with paths, committed paths and
stop="residual-goal" (src/xgraph/oracle.py:1081-1111, 1608-1635), each under its own
question, recording at every step the reference state (make_golden.state_record) and its
whole allowed set; and for every question the reference's STOP table
(src/xgraph/stopping.py:74-133: answer-head relations, relevant question words, each
relation's covered words).

- Path walks on three golden worlds (the reference's toy KG and two seeded random KGs of
  worlds.json.gz): a question asks for the last relation of a path the KG holds ("Which
  <relation> has <start>?" or "What is the <relation> of <start>?"), the walk writes that
  path in a span token by token, and where the text's next token is not allowed (STOP
  forces the closer) it writes the closer instead; random tokens follow.
- Random walks on the same worlds under a question (the make_golden sampler).
- The reference's own STOP tests' worlds (tests/test_engine.py:3930-3967, 3970-4000): a
  STOP that overrides an escape marker already started beside a longer relation label,
  and questions of 33 and 64 relevant words (the high word bits).
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
STEPS = 40


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True, help="the reference checkout")
    args = parser.parse_args()
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(args.reference / "src"), str(args.reference)]
    sys.path.insert(0, str(HERE))
    from make_golden import _kg, _tokenizer, state_record  # noqa: E402

    from tests.conftest import byte_level_tokenizer  # the reference's own tests package
    from xgraph.index import build_kg_index
    from xgraph.kg import Entity, KnowledgeGraph, Relation
    from xgraph.oracle import Oracle, Phase
    from xgraph.stopping import RelationTerms
    from xgraph.syntax import SpanSyntax

    with gzip.open(HERE / "worlds.json.gz", "rt", encoding="utf-8") as f:
        worlds = json.load(f)

    def table(terms, question):
        goal = terms.for_question(question)
        return {"head": sorted(goal.head), "words": list(goal.words),
                "coverage": sorted([r, m] for r, m in goal.coverage.items())}

    def record_walk(oracle, served, syntax, question, tokens, rng, fallback_closer=True, extra=8):
        """The walk over `tokens` (a token not allowed there: the closer if allowed, else a
        random allowed token), then `extra` random allowed tokens."""
        state = oracle.initial_state(question=question)
        closer = served.encode(syntax.closer)
        walked, states, allowed_at = [], [], []
        queue = list(tokens)
        steps = len(tokens) + extra
        for _ in range(steps):
            allowed = oracle.allowed(state)
            states.append(state_record(state))
            allowed_at.append(sorted(allowed))
            if queue and queue[0] in allowed:
                token = queue.pop(0)
            elif queue and fallback_closer and closer[0] in allowed:
                queue = list(closer)
                token = queue.pop(0)
            else:
                queue = []
                regular = sorted(t for t in allowed if t not in served.special_ids) or sorted(allowed)
                token = rng.choice(regular)
            walked.append(token)
            state = oracle.advance(state, token)
        return {"question": question, "tokens": walked, "states": states, "allowed": allowed_at,
                "final": state_record(state), "final_allowed": sorted(oracle.allowed(state))}

    cases = []
    for world_name in ("toy", "rand_bpe", "rand_dense"):
        world = worlds[world_name]
        served, syntax = _tokenizer(world["tokenizer"]), SpanSyntax()
        index = build_kg_index(_kg((world["entities"], world["relations"], world["triples"], None, None)),
                               served, syntax)
        oracle = Oracle(index, served, syntax, paths=True, committed_paths=True, stop="residual-goal")
        terms = RelationTerms.from_index(index, served)
        rng = random.Random(sum(map(ord, world_name)) + 5)
        ents = {e: labels for e, labels in world["entities"]}
        rels = {r: labels for r, labels in world["relations"]}
        outgoing: dict[str, list[tuple[str, str]]] = {}
        for s, r, o in world["triples"]:
            outgoing.setdefault(s, []).append((r, o))
        walks, tables = [], {}
        subjects = sorted(s for s in outgoing if ents.get(s))
        for k in range(14):
            start = rng.choice(subjects)
            hops, at = [], start
            for _ in range(rng.randint(1, 3)):
                if at not in outgoing:
                    break
                r, o = rng.choice(outgoing[at])
                hops.append(r)
                at = o
            asked = rels[hops[-1]][0]
            name = ents[start][0]
            question = (f"Which {asked} has {name}?" if k % 2 == 0 else f"What is the {asked} of {name}?")
            text = (" " + syntax.opener + syntax.label_prefix + name
                    + "".join(syntax.separator + syntax.label_prefix + rels[r][0] for r in hops) + syntax.closer)
            walks.append(record_walk(oracle, served, syntax, question, served.encode(text), rng))
            tables[question] = table(terms, question)
        for k in range(4):  # random walks under a question
            start, hop = rng.choice(subjects), rng.choice(outgoing[rng.choice(subjects)])[0]
            question = f"Which {rels[hop][0]} has {ents[start][0]}?"
            tokens = [rng.randrange(served.vocab_size) for _ in range(STEPS)]
            walks.append(record_walk(oracle, served, syntax, question, tokens, rng, fallback_closer=False, extra=0))
            tables[question] = table(terms, question)
        cases.append({"world": world_name, "walks": walks, "tables": tables})

    # the reference tests' STOP worlds
    served = byte_level_tokenizer([])
    from xgraph.tokenizer import ServedTokenizer

    plain = ServedTokenizer(served)
    syntax = SpanSyntax(opener="[", label_prefix="", closer="]", separator="/", escape="ry?")
    kg = KnowledgeGraph(
        entities=(Entity("Q1", ("Seed",)), Entity("Q2", ("End",))),
        relations=(Relation("P1", ("count",)), Relation("P2", ("country",))),
        triples=(("Q1", "P1", "Q2"), ("Q1", "P2", "Q2"), ("Q2", "P1", "Q1")),
    )
    index = build_kg_index(kg, plain, syntax)
    oracle = Oracle(index, plain, syntax, paths=True, committed_paths=True, stop="residual-goal")
    question = "Which country has Seed?"
    walk = record_walk(oracle, plain, syntax, question, plain.encode("[Seed/country"), random.Random(3), extra=4)
    cases.append({"world": "escape", "tokenizer": served.to_str(),
                  "kg": {"entities": [["Q1", ["Seed"]], ["Q2", ["End"]]],
                         "relations": [["P1", ["count"]], ["P2", ["country"]]],
                         "triples": [["Q1", "P1", "Q2"], ["Q1", "P2", "Q2"], ["Q2", "P1", "Q1"]]},
                  "syntax": {"opener": "[", "label_prefix": "", "closer": "]", "separator": "/", "escape": "ry?"},
                  "walks": [walk], "tables": {question: table(RelationTerms.from_index(index, plain), question)}})
    for word_count in (33, 64):
        syntax = SpanSyntax()
        words = [f"item{i:03}" for i in range(word_count - 1)]
        start = " ".join(words)
        kg_json = {"entities": [["Q1", [start]], ["Q2", ["End"]], ["Q3", ["Tail"]]],
                   "relations": [["P1", ["country"]], ["P2", ["zulu", "border country", *words]]],
                   "triples": [["Q1", "P1", "Q2"], ["Q2", "P2", "Q3"], ["Q3", "P1", "Q1"]]}
        kg = KnowledgeGraph(
            entities=tuple(Entity(i, tuple(ls)) for i, ls in kg_json["entities"]),
            relations=tuple(Relation(i, tuple(ls)) for i, ls in kg_json["relations"]),
            triples=tuple(tuple(t) for t in kg_json["triples"]),
        )
        index = build_kg_index(kg, plain, syntax)
        oracle = Oracle(index, plain, syntax, paths=True, committed_paths=True, stop="residual-goal")
        question = f"Which country has the zulu of {start}?"
        text = f" {syntax.opener} {start} · country · zulu{syntax.closer}"
        walk = record_walk(oracle, plain, syntax, question, plain.encode(text), random.Random(word_count), extra=2)
        cases.append({"world": f"words{word_count}", "tokenizer": served.to_str(), "kg": kg_json,
                      "syntax": {"opener": syntax.opener, "label_prefix": syntax.label_prefix,
                                 "closer": syntax.closer, "separator": syntax.separator, "escape": syntax.escape},
                      "walks": [walk], "tables": {question: table(RelationTerms.from_index(index, plain), question)}})
    forced = sum(1 for c in cases for w in c["walks"] for s in w["states"]
                 if s["phase"] == Phase.SPAN.value and s["segment"] == "relation")
    with gzip.open(HERE / "stop_cases.json.gz", "wt", encoding="utf-8") as f:
        json.dump({"cases": cases}, f, separators=(",", ":"))
    print(f"{sum(len(c['walks']) for c in cases)} walks, {forced} relation-label states")


if __name__ == "__main__":
    main()
