"""Save the toy world's KG index with the reference's own builder and writer, so that the
tests can check that this library reads the reference's on-disk index format (one .npy
file per array plus kg-index.json, src/xgraph/index.py:731-903).

Run in a container that holds the reference checkout (imported read-only, no bytecode):

    python tests/golden/make_reference_index.py --reference <reference checkout>

It writes reference_index_toy/ next to this script from worlds.json.gz.
"""

from __future__ import annotations

import argparse
import gzip
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True, help="the reference checkout")
    args = parser.parse_args()
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(args.reference / "src"), str(args.reference)]
    from tokenizers import Tokenizer
    from xgraph.index import build_kg_index, save_kg_index
    from xgraph.kg import Entity, KnowledgeGraph, Relation
    from xgraph.syntax import SpanSyntax
    from xgraph.tokenizer import ServedTokenizer

    with gzip.open(HERE / "worlds.json.gz", "rt", encoding="utf-8") as f:
        world = json.load(f)["toy"]
    kg = KnowledgeGraph(
        tuple(Entity(i, tuple(ls)) for i, ls in world["entities"]),
        tuple(Relation(i, tuple(ls)) for i, ls in world["relations"]),
        tuple(tuple(t) for t in world["triples"]),
    )
    served = ServedTokenizer(Tokenizer.from_str(world["tokenizer"]))
    index = build_kg_index(kg, served, SpanSyntax(), sitelinks=world["sitelinks"])
    save_kg_index(index, HERE / "reference_index_toy")
    print("wrote", HERE / "reference_index_toy")


if __name__ == "__main__":
    main()
