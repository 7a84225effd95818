"""Golden fixture of expressions (date and value comparisons), recorded with the reference.

Run in a container that holds the reference checkout (imported read-only, no bytecode):

    python tests/golden/make_expression_cases.py --reference <reference checkout>

expression_cases.json.gz holds walks of the reference Oracle in path mode with committed
paths and expressions=True (src/xgraph/oracle.py:104-133, 1048-1130, 1669-1737, 1830-1905):
`⟦ earlier: A | B · r1 · r2⟧` compares the earliest dates the two operands' best starts
reach (`later:` the latest), `⟦ same: A | B · r⟧` gives the verdict entity of whether the
two reaches share a value; the result binds the answer span after it.  Every step records
the reference state (make_golden.state_record plus the expression fields) and its whole
allowed set.  Per golden world (toy, rand_bpe, rand_dense, crowd): a seeded date for about
half of the entities that are objects of triples (years 1890-1895, day, month or year
precision, stored with or without the month and day), the index built with those dates and,
on all worlds but rand_dense, with the verdict entities; two worlds carry two KG versions
each, the walks alternating base and versions:

- comparison walks: the text of a comparison with a random operator, two start labels of
  entities with an edge of one relation, that relation's label and sometimes one more
  random relation label, written token
  by token; where the text's next token is not allowed the walk writes the closer if it
  may, else a random allowed token; then random tokens;
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
STEPS = 56
WORLDS = (("toy", True, True), ("rand_bpe", True, True), ("rand_dense", False, False), ("crowd", False, True))


def seeded_dates(world, rng: random.Random) -> dict[str, list]:
    """[year, month, day, precision] for about half the objects of the world's triples."""
    objects = sorted({o for _, _, o in world["triples"]})
    out = {}
    for entity in objects:
        if rng.random() < 0.5:
            continue
        year, month, day = rng.randint(1890, 1895), rng.randint(1, 12), rng.randint(1, 28)
        kind = rng.random()
        if kind < 0.45:
            out[entity] = [year, month, day, "day"]
        elif kind < 0.7:
            out[entity] = [year, month, None, "month"]
        elif kind < 0.85:
            out[entity] = [year, None, None, "year"]
        else:  # stored at year precision with its month and day kept (1 January)
            out[entity] = [year, 1, 1, "year"]
    return out


def expression_record(state_record, state) -> dict:
    """make_golden.state_record plus the expression fields of the state and its last span."""
    record = state_record(state)
    record["operating"] = None if state.operating is None else state.operating.hex()
    record["operator"] = state.operator
    record["starts"] = [list(s) for s in state.starts]
    record["ranks_b"] = sorted([list(x) for x in state.ranks_b])
    if state.last_span is not None:
        record["last_span"]["operator"] = state.last_span.operator
        record["last_span"]["operands"] = list(state.last_span.operands)
    return record


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True, help="the reference checkout")
    args = parser.parse_args()
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(args.reference / "src"), str(args.reference)]
    sys.path.insert(0, str(HERE))
    from make_golden import _edits, _kg, _tokenizer, state_record  # noqa: E402

    from xgraph.expressions import Date
    from xgraph.index import build_kg_index
    from xgraph.oracle import Oracle, Phase, Segment
    from xgraph.syntax import SpanSyntax

    with gzip.open(HERE / "worlds.json.gz", "rt", encoding="utf-8") as f:
        worlds = json.load(f)

    cases = []
    for world_name, versioned, verdicts in WORLDS:
        world = worlds[world_name]
        served, syntax = _tokenizer(world["tokenizer"]), SpanSyntax()
        as_tuple = (world["entities"], world["relations"], world["triples"], None, None)
        rng = random.Random(sum(map(ord, world_name)) * 7 + 1)
        dates = seeded_dates(world, rng)
        index = build_kg_index(_kg(as_tuple), served, syntax,
                               dates={e: Date(*d) for e, d in dates.items()}, verdicts=verdicts)
        edits = _edits(as_tuple, sum(map(ord, world_name)) + 5) if versioned else {}
        names = [None, *edits]
        oracle = Oracle(index, served, syntax, paths=True, committed_paths=True, expressions=True,
                        versions=edits or None)
        ents = {e: labels for e, labels in world["entities"] if labels}
        rel_names = {r: labels for r, labels in world["relations"] if labels}
        outgoing: dict[str, list[str]] = {}
        having: dict[str, set[str]] = {}
        for s, r, _ in world["triples"]:
            if r in rel_names and s in ents:
                outgoing.setdefault(s, []).append(r)
                having.setdefault(r, set()).add(s)
        subjects = sorted(outgoing)
        operators = syntax.operators if verdicts else syntax.operators[:2]
        opener = served.encode(" " + syntax.opener)
        closer, separator = served.encode(syntax.closer), served.encode(syntax.separator)
        escape = served.encode(syntax.escape)
        regular = [t for t in range(served.vocab_size) if t not in served.special_ids]
        walks = []
        for n in range(20):
            version = names[n % len(names)]
            state = oracle.initial_state(version)
            if n < 15:  # a comparison walk
                a = rng.choice(subjects)
                relation = rng.choice(outgoing[a])
                b = rng.choice(sorted(having[relation]))
                hops = [rng.choice(rel_names[relation])]
                if rng.random() < 0.3:
                    hops.append(rng.choice(rel_names[rng.choice(sorted(rel_names))]))
                text = (" " + syntax.opener + syntax.label_prefix + operators[n % len(operators)]
                        + syntax.label_prefix + rng.choice(ents[a]) + syntax.operand_separator
                        + syntax.label_prefix + rng.choice(ents[b])
                        + "".join(syntax.separator + syntax.label_prefix + r for r in hops) + syntax.closer)
                queue, free = list(served.encode(text)), False
            else:
                queue, free = [], True
            tokens, states, allowed_at = [], [], []
            for _ in range(STEPS):
                allowed = oracle.allowed(state)
                states.append(expression_record(state_record, state))
                allowed_at.append(sorted(allowed))
                if not queue:
                    free = True
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
                          "final": expression_record(state_record, state),
                          "final_allowed": sorted(oracle.allowed(state))})
        cases.append({"world": world_name, "verdicts": verdicts, "dates": dates,
                      "versions": {k: [list(e) for e in v] for k, v in edits.items()}, "walks": walks})
    closed = [s["last_span"] for c in cases for w in c["walks"] for s in [*w["states"], w["final"]]
              if s["last_span"] and s["last_span"].get("operator")]
    kinds = sorted({(s["operator"], len(s["entity_ids"])) for s in closed})
    with gzip.open(HERE / "expression_cases.json.gz", "wt", encoding="utf-8") as f:
        json.dump({"cases": cases}, f, separators=(",", ":"))
    print(f"{sum(len(c['walks']) for c in cases)} walks, {len(closed)} states after a comparison, "
          f"(operator, result size) seen: {kinds}")


if __name__ == "__main__":
    main()
