"""Golden fixture of offline path execution, recorded with the reference itself.

Run in a container that holds the reference checkout (imported read-only, no bytecode):

    python tests/golden/make_matched_cases.py --reference <reference checkout>

matched_cases.json.gz holds paths written without the engine, `start · r1 · ... · rk`, and
what the reference's MatchedExecutor (src/xgraph/programs.py:368-1130, path mode with
committed paths executed after decoding) makes of each: the entities reached in
best-connected order, the answer delivered and the plan path mode would write.  The paths
run on four golden worlds of worlds.json.gz (the reference's toy KG, two seeded random KGs
with homonyms, aliases and quoted labels, and the crowded KG whose starts and frontiers
overflow every 64-entry cap) under several executor settings (committed or union paths,
degree or sitelink start rank, unquoted starts, KG versions with add / remove edits):

- paths walked along the KG's own edges, 1-4 relations, with random labels and aliases;
- entity spans (no relation), starts that name nothing, relations the frontier lacks,
  relation labels cut short, and walks longer than the 8-relation cap;
- with strip_quotes, every other start wrapped in quotation marks;
- anchored paths and entity spans (see anchored_of), each recorded with whether the
  executor fell back to every anchor entity, and an anchor naming no entity (recorded with
  the reference's error).

Every path also records the executor's live frontier: `starts`, `frontier` (after its
relations) and `frontier_relations`, the `derivations` of the entities it resolves to, and
`execute_set` (reached, uncapped reached, cap events; and with endpoint witnesses;
src/xgraph/programs.py:486-736), and its execution with relation repair.
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
SETTINGS = {
    "committed": {"committed_paths": True},
    "sitelinks": {"committed_paths": True, "start_rank": "sitelinks"},
    "union": {"committed_paths": False},
    "unquoted": {"committed_paths": True, "unquoted_starts": True},
    "stripped": {"committed_paths": True, "strip_quotes": True},
}
PLAN = [("toy", ("committed", "sitelinks", "union", "stripped")),
        ("rand_bpe", ("committed", "sitelinks", "union", "unquoted", "stripped")),
        ("rand_dense", ("committed", "union")),
        ("crowd", ("committed", "sitelinks"))]


def paths_of(world, rng: random.Random, count: int) -> list[tuple[str, list[str]]]:
    """Seeded written paths over one world (see the module docstring)."""
    ents = {e: labels for e, labels in world["entities"] if labels}
    rels = {r: labels for r, labels in world["relations"] if labels}
    outgoing: dict[str, list[tuple[str, str]]] = {}
    for s, r, o in world["triples"]:
        if r in rels:
            outgoing.setdefault(s, []).append((r, o))
    subjects = sorted(s for s in outgoing if s in ents)
    out = []
    for k in range(count):
        start = rng.choice(subjects)
        name = rng.choice(ents[start])
        kind = k % 8
        hops, at = [], start
        length = 10 if kind == 7 else rng.randint(1, 4)
        for _ in range(length):
            if at not in outgoing:
                break
            r, o = rng.choice(outgoing[at])
            hops.append(rng.choice(rels[r]))
            at = o
        if kind == 3:
            hops = []                                   # an entity span
        elif kind == 4:
            name = "Nobody Here"                        # a start naming nothing
        elif kind == 5 and hops:
            hops[-1] = rng.choice(rels[rng.choice(sorted(rels))])  # a relation the frontier may lack
        elif kind == 6 and hops and len(hops[-1]) > 2:
            hops[-1] = hops[-1][: len(hops[-1]) // 2]   # a relation label cut short
        out.append((name, hops))
    return out


def anchored_of(world, rng: random.Random, count: int) -> list[tuple[str, list[str], list[str]]]:
    """Seeded anchored paths: walks as in paths_of (some of them entity spans) written from
    one label of the start entity, with an anchor that is the start entity, the start and
    another entity, another entity the same label names (a homonym, where there is one), or
    an entity the label does not name (the executor then starts from every anchor entity);
    and one anchor naming no entity with labels."""
    ents = {e: labels for e, labels in world["entities"] if labels}
    rels = {r: labels for r, labels in world["relations"] if labels}
    named: dict[str, list[str]] = {}
    for e, labels in ents.items():
        for label in labels:
            named.setdefault(label, []).append(e)
    outgoing: dict[str, list[tuple[str, str]]] = {}
    for s, r, o in world["triples"]:
        if r in rels:
            outgoing.setdefault(s, []).append((r, o))
    subjects = sorted(s for s in outgoing if s in ents)
    everyone = sorted(ents)
    out = []
    for k in range(count):
        start = rng.choice(subjects)
        name = rng.choice(ents[start])
        hops, at = [], start
        for _ in range(0 if k % 6 == 5 else rng.randint(1, 3)):
            if at not in outgoing:
                break
            r, o = rng.choice(outgoing[at])
            hops.append(rng.choice(rels[r]))
            at = o
        kind = k % 4
        if kind == 0:
            anchor = [start]
        elif kind == 1:
            anchor = [start, rng.choice(everyone)]
        elif kind == 2:
            others = [e for e in named[name] if e != start]
            anchor = [rng.choice(others)] if others else [start]
        else:
            anchor = [rng.choice([e for e in everyone if e not in named[name]])]
        out.append((name, hops, anchor))
    out.append((rng.choice(ents[rng.choice(subjects)]), [], ["Q999999999"]))
    return out


def live(executor, start, relations, anchor, version) -> dict:
    """The executor's view of the path's live frontier: its starts, the capped frontier after
    its relations, the relations that frontier offers with their edge counts, and the
    derivations of the entities it resolves to."""
    return {"starts": list(executor.starts(start, anchor, version)),
            "frontier": list(executor.frontier(start, relations, anchor, version)),
            "frontier_relations": [list(x) for x in executor.frontier_relations(start, relations, anchor, version)],
            "derivations": [list(x) for x in executor.derivations(start, relations, anchor, version)],
            "execute_set": executor.execute_set(start, relations, anchor, version),
            "witnesses": witnessed(executor, start, relations, anchor, version),
            "repaired": repaired(executor, start, relations, anchor, version)}


def repaired(executor, start, relations, anchor, version):
    """execute with repair: reached, answer and plan."""
    path = executor.execute(start, relations, anchor=anchor, version=version, repair=True)
    return {"reached": list(path.reached), "answer": path.answer,
            "plan": None if path.plan is None else list(path.plan)}


def witnessed(executor, start, relations, anchor, version):
    """execute_set with witnesses, or the error it raises (an entity id whose tail is no
    number cannot rank a chain)."""
    try:
        return executor.execute_set(start, relations, anchor, version, witnesses=True)
    except ValueError as error:
        return {"error": str(error)}


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True, help="the reference checkout")
    args = parser.parse_args()
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(args.reference / "src"), str(args.reference)]
    sys.path.insert(0, str(HERE))
    from make_golden import _edits, _kg, _tokenizer  # noqa: E402

    from xgraph.index import build_kg_index
    from xgraph.kgversions import build_kg_versions
    from xgraph.programs import MatchedExecutor
    from xgraph.syntax import SpanSyntax

    with gzip.open(HERE / "worlds.json.gz", "rt", encoding="utf-8") as f:
        worlds = json.load(f)
    cases, all_edits = [], {}
    for world_name, settings in PLAN:
        world = worlds[world_name]
        served, syntax = _tokenizer(world["tokenizer"]), SpanSyntax()
        as_tuple = (world["entities"], world["relations"], world["triples"], None, None)
        index = build_kg_index(_kg(as_tuple), served, syntax, sitelinks=world["sitelinks"])
        edits = _edits(as_tuple, sum(map(ord, world_name)))
        all_edits[world_name] = {name: [list(e) for e in v] for name, v in edits.items()}
        versions = build_kg_versions(index, edits)
        rng = random.Random(sum(map(ord, world_name)) * 31 + 7)
        written = paths_of(world, rng, 64)
        anchored = anchored_of(world, rng, 24)
        for setting in settings:
            executor = MatchedExecutor(index, served, versions=versions, **SETTINGS[setting])
            for n, (start, relations) in enumerate(written):
                version = (None, "v0", "v1")[n % 3] if world_name != "crowd" else None
                if setting == "stripped" and n % 2 == 0:  # a start written in quotation marks
                    start = ('"{}"', "\u201c{}\u201d", "'{}'", "\u00ab {} \u00bb")[n // 2 % 4].format(start)
                path = executor.execute(start, relations, version=version)
                cases.append({"world": world_name, "setting": setting, "start": start,
                              "relations": relations, "version": version,
                              "reached": list(path.reached), "answer": path.answer,
                              "plan": None if path.plan is None else list(path.plan), "stripped": path.stripped,
                              **live(executor, start, relations, None, version)})
            for n, (start, relations, anchor) in enumerate(anchored):
                version = (None, "v0", "v1")[n % 3] if world_name != "crowd" else None
                case = {"world": world_name, "setting": setting, "start": start, "relations": relations,
                        "version": version, "anchor": anchor}
                try:
                    path = executor.execute(start, relations, anchor=anchor, version=version)
                except ValueError as error:
                    cases.append({**case, "error": str(error)})
                    continue
                # the executor's fallback: the start label names none of the anchor's entities
                fallback = not executor._written_starts(start, anchor)
                cases.append({**case, "fallback": fallback, "reached": list(path.reached),
                              "answer": path.answer, "plan": None if path.plan is None else list(path.plan),
                              **live(executor, start, relations, anchor, version)})
    with gzip.open(HERE / "matched_cases.json.gz", "wt", encoding="utf-8") as f:
        json.dump({"settings": SETTINGS, "edits": all_edits, "cases": cases}, f)
    empty = sum(1 for c in cases if not c.get("reached"))
    print(f"{len(cases)} cases ({empty} empty)")


if __name__ == "__main__":
    main()
