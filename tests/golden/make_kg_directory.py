"""Write a toy KG directory (the reference's "gate" layout) and the index the reference's
own directory builder makes from it, so that the tests can check this library's reader
against it (src/xgraph/wikidata.py:859-1037).

Run in a container that holds the reference checkout (imported read-only, no bytecode):

    python tests/golden/make_kg_directory.py --reference <reference checkout>

From the rand_bpe world of worlds.json.gz it writes, next to this script:
  kg_directory_toy/        entity_labels.jsonl and relation_labels.jsonl (one JSON list
                           [id, label, "label" | "alias"] per line), triples.npy (int32
                           item/property numbers), sitelink_counts.npy ([item, count] rows)
  kg_directory_toy_index/  the reference's build_index output (its on-disk index format)
  kg_directory_toy_index_unique/  the same with unique_aliases
Item numbers are spread out (Q10, Q13, ...), a few triples name items or properties that
have no label rows, and the relation rows hold an alias-only property, an alias that is
another property's label and an alias two properties share, so the position lookup, the
unwritable count and the relation-name rules are exercised.
"""

from __future__ import annotations

import argparse
import gzip
import json
import shutil
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True, help="the reference checkout")
    args = parser.parse_args()
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(args.reference / "src"), str(args.reference)]
    from tokenizers import Tokenizer
    from xgraph.syntax import SpanSyntax
    from xgraph.tokenizer import ServedTokenizer
    from xgraph.wikidata import build_index

    with gzip.open(HERE / "worlds.json.gz", "rt", encoding="utf-8") as f:
        world = json.load(f)["rand_bpe"]
    item = {e: 10 + 3 * k for k, (e, _) in enumerate(world["entities"])}
    prop = {r: 5 + 2 * k for k, (r, _) in enumerate(world["relations"])}
    kg = HERE / "kg_directory_toy"
    out = HERE / "kg_directory_toy_index"
    for path in (kg, out):
        if path.exists():
            shutil.rmtree(path)
    kg.mkdir()
    with (kg / "entity_labels.jsonl").open("w", encoding="utf-8") as f:
        for e, labels in world["entities"]:
            for k, label in enumerate(labels):
                f.write(json.dumps([f"Q{item[e]}", label, "label" if k == 0 else "alias"]) + "\n")
    with (kg / "relation_labels.jsonl").open("w", encoding="utf-8") as f:
        for r, labels in world["relations"]:
            for k, label in enumerate(labels):
                f.write(json.dumps([f"P{prop[r]}", label, "label" if k == 0 else "alias"]) + "\n")
        f.write(json.dumps(["P3", "unused alias", "alias"]) + "\n")  # a property with no label
        first, second, third = (f"P{prop[r]}" for r, _ in world["relations"][:3])
        label_of_second = world["relations"][1][1][0]
        f.write(json.dumps([first, label_of_second.upper(), "alias"]) + "\n")  # another property's label
        f.write(json.dumps([second, "shared name", "alias"]) + "\n")  # an alias two properties share
        f.write(json.dumps([third, "shared name", "alias"]) + "\n")
    triples = [(item[s], prop[r], item[o]) for s, r, o in world["triples"]]
    triples += [(99999, prop[world["relations"][0][0]], item[world["entities"][0][0]]),
                (item[world["entities"][1][0]], 3, item[world["entities"][2][0]]),
                (item[world["entities"][3][0]], 77, 88888)]
    np.save(kg / "triples.npy", np.array(triples, dtype=np.int32))
    counts = sorted((item[e], int(n)) for e, n in world["sitelinks"].items())
    np.save(kg / "sitelink_counts.npy", np.array(counts, dtype=np.int64))
    served = ServedTokenizer(Tokenizer.from_str(world["tokenizer"]))
    build_index(kg, served, SpanSyntax(), out)
    unique = HERE / "kg_directory_toy_index_unique"
    if unique.exists():
        shutil.rmtree(unique)
    build_index(kg, served, SpanSyntax(), unique, unique_aliases=True)
    print("wrote", kg, out, "and", unique)


if __name__ == "__main__":
    main()
