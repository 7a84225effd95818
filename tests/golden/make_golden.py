"""Generate the golden vectors that pin the oracle to the reference implementation.

Run in a container that holds the reference checkout (it is imported read-only,
without writing bytecode):

    python tests/golden/make_golden.py --reference <reference checkout>

It writes three fixtures next to this script:

- worlds.json.gz: each world's KG (entities, relations, triples), its tokenizer
  (serialized tokenizer.json) and sitelink counts;
- index.npz: the reference's compiled index arrays of every world (label rows,
  relation rows, adjacency) and the version tables of every versioned case;
- walks.json.gz + masks.npz: seeded random walks through the reference Oracle in
  every engine mode: per step the token taken, the reference state before it
  (every in-scope field) and, in masks.npz, its allowed set as packed uint32 words.

The walks are biased toward whole spans (open, separate, close, escape now and then)
so that every phase, segment, branch and closing kind is visited.
"""

from __future__ import annotations

import argparse
import gzip
import json
import os
import random
import sys
from concurrent.futures import ProcessPoolExecutor
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

SYLLABLES = [
    "ka", "lo", "mi", "ra", "ne", "to", "su", "vi", "da", "pe", "zu", "ho", "ri", "an",
    "el", "or", "ul", "ba", "co", "fe", "ga", "ju", "ly", "qu", "wen", "ish",
]
WORDS = ["born", "in", "part", "of", "capital", "member", "author", "river", "near", "made"]


def _name(rng: random.Random, words: int) -> str:
    out = []
    for _ in range(words):
        word = "".join(rng.choice(SYLLABLES) for _ in range(rng.randint(1, 3)))
        out.append(word.capitalize())
    return " ".join(out)


def random_world(seed: int, entities: int, relations: int, triples: int, quoted: bool):
    """A seeded KG with homonyms, labels that prefix other labels, aliases, quoted labels,
    multibyte labels and a few isolated entities."""
    rng = random.Random(seed)
    names: list[str] = []
    ents = []
    for n in range(entities):
        if names and rng.random() < 0.15:
            label = rng.choice(names)  # homonym
        elif names and rng.random() < 0.12:
            label = rng.choice(names) + " " + _name(rng, 1)  # continues another label
        else:
            label = _name(rng, rng.randint(1, 2))
        if quoted and rng.random() < 0.08:
            label = rng.choice(['"', "«", "“"]) + label
        if rng.random() < 0.05:
            label = label + " Ł"
        names.append(label)
        labels = [label]
        if rng.random() < 0.2:
            labels.append(_name(rng, 1))  # alias
        ents.append((f"E{n}", labels))
    rels = []
    rel_names: list[str] = []
    for n in range(relations):
        if rel_names and rng.random() < 0.2:
            label = rng.choice(rel_names)  # shared relation label
        elif rel_names and rng.random() < 0.2:
            label = rng.choice(rel_names) + " " + rng.choice(WORDS)  # prefixed relation label
        else:
            label = " ".join(rng.sample(WORDS, rng.randint(1, 2)))
        rel_names.append(label)
        rels.append((f"R{n}", [label]))
    trip = set()
    for _ in range(triples):
        s = rng.randrange(entities - 3)  # the last three entities stay isolated
        trip.add((f"E{s}", f"R{rng.randrange(relations)}", f"E{rng.randrange(entities)}"))
    sitelinks = {f"E{n}": rng.randrange(0, 5) for n in range(entities)}
    return ents, rels, sorted(trip), sitelinks


def crowded_world():
    """Caps: a hub with 70 objects under one relation, 70 homonymous starts with triples,
    and an entity with 70 aliases, so that frontiers, starts and reached rows overflow 64."""
    ents = [("H", ["Hub"]), ("G", ["Goal"]), ("A", ["Alias Owner"] + [f"Al{k:02d}" for k in range(70)])]
    rels = [("r", ["to"]), ("t", ["then"]), ("u", ["also"])]
    trip = []
    for k in range(70):
        ents.append((f"B{k}", [f"Bee {k:02d}"]))
        ents.append((f"T{k}", ["Twin"]))
        trip.append(("H", "r", f"B{k}"))
        trip.append((f"T{k}", "r", f"B{(k * 7) % 70}"))
        trip.append((f"T{k}", "u", "A"))
    trip += [("B64", "t", "G"), ("B3", "t", "G"), ("B69", "u", "H"), ("A", "r", "G"), ("G", "t", "H")]
    sitelinks = {e: (k * 13) % 7 for k, (e, _) in enumerate(ents)}
    return ents, rels, sorted(trip), sitelinks


def load_reference(root: Path):
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(root / "src"), str(root)]
    import xgraph  # noqa: F401

    return root


def tokenizers_for(world, kind: str):
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers

    alphabet = sorted(pre_tokenizers.ByteLevel.alphabet())
    if kind == "bytes":
        tok = Tokenizer(models.BPE({c: i for i, c in enumerate(alphabet)}, []))
        tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
        tok.decoder = decoders.ByteLevel()
        tok.add_special_tokens(["<|endoftext|>"])
        return tok
    ents, rels, _, _ = world
    corpus = [label for _, labels in ents + rels for label in labels]
    corpus += ["⟦ " + label + " · " + rels[0][1][0] + "⟧ ⟦ ⁇ text⟧" for _, (label, *_) in ents[:50]]
    tok = Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(
        vocab_size=int(kind), special_tokens=["<|endoftext|>"],
        initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False,
    )
    tok.train_from_iterator(corpus, trainer=trainer)
    return tok


def build_worlds(root: Path) -> dict:
    """name -> (entities, relations, triples, sitelinks, tokenizer json)."""
    sys.path.insert(0, str(root / "tests"))
    from tests.conftest import TOY_ENTITIES, TOY_RELATIONS, TOY_TEXT, TOY_TRIPLES, train_byte_level_bpe

    worlds = {}
    toy_ents = [(i, list(ls)) for i, ls in TOY_ENTITIES]
    toy_rels = [(i, list(ls)) for i, ls in TOY_RELATIONS]
    labels = [label for _, ls in TOY_ENTITIES + TOY_RELATIONS for label in ls]
    toy_tok = train_byte_level_bpe(labels + list(TOY_TEXT), vocab_size=400)
    worlds["toy"] = (toy_ents, toy_rels, [list(t) for t in TOY_TRIPLES],
                     {i: n for n, (i, _) in enumerate(TOY_ENTITIES)}, toy_tok.to_str())
    for name, seed, size, quoted, tok_kind in (
        ("rand_bpe", 11, (60, 8, 220), True, "520"),
        ("rand_bytes", 12, (40, 6, 140), True, "bytes"),
        ("rand_dense", 13, (30, 5, 260), False, "420"),
    ):
        world = random_world(seed, *size, quoted)
        tok = tokenizers_for(world, tok_kind)
        ents, rels, trip, sitelinks = world
        worlds[name] = (ents, rels, [list(t) for t in trip], sitelinks, tok.to_str())
    crowd = crowded_world()
    tok = tokenizers_for(crowd, "600")
    worlds["crowd"] = (*crowd[:4], tok.to_str())
    return worlds


# (case name, world, engine options, versions?, anchors?, opened?)
CASES = [
    ("toy_ordinary", "toy", {}, False, False, False),
    ("toy_noescape", "toy", {"escapes": False}, False, False, False),
    ("toy_norepeat", "toy", {"repeats": False}, False, False, False),
    ("toy_derivation", "toy", {"derivation": True}, False, True, False),
    ("toy_paths", "toy", {"paths": True}, False, False, False),
    ("toy_committed", "toy", {"paths": True, "committed_paths": True}, True, True, False),
    ("toy_opened", "toy", {"paths": True, "committed_paths": True, "start_rank": "sitelinks"}, False, False, True),
    ("bpe_ordinary", "rand_bpe", {"unquoted_starts": True}, True, False, False),
    ("bpe_norepeat", "rand_bpe", {"repeats": False, "derivation": True}, True, True, False),
    ("bpe_paths", "rand_bpe", {"paths": True, "bound_escapes": False}, True, True, False),
    ("bpe_committed", "rand_bpe", {"paths": True, "committed_paths": True, "unquoted_starts": True}, True, True, False),
    ("bpe_sitelinks", "rand_bpe", {"paths": True, "committed_paths": True, "start_rank": "sitelinks", "end_after_answer": True}, True, True, False),
    ("bytes_ordinary", "rand_bytes", {}, False, False, False),
    ("bytes_paths", "rand_bytes", {"paths": True, "committed_paths": True}, True, True, True),
    ("bytes_derivation", "rand_bytes", {"derivation": True, "bound_escapes": False, "unquoted_starts": True}, False, True, False),
    ("dense_committed", "rand_dense", {"paths": True, "committed_paths": True, "end_after_answer": True}, True, False, False),
    ("dense_ordinary", "rand_dense", {"repeats": False}, True, False, True),
    ("crowd_union", "crowd", {"paths": True}, False, False, False),
    ("crowd_committed", "crowd", {"paths": True, "committed_paths": True}, True, True, True),
    ("crowd_derivation", "crowd", {"derivation": True}, False, False, False),
    ("crowd_sitelinks", "crowd", {"paths": True, "committed_paths": True, "start_rank": "sitelinks"}, False, False, False),
]
SEQUENCES, STEPS = 8, 160


def _tokenizer(tok_json: str):
    from tokenizers import Tokenizer
    from xgraph.tokenizer import ServedTokenizer

    return ServedTokenizer(Tokenizer.from_str(tok_json))


def _kg(world):
    from xgraph.kg import Entity, KnowledgeGraph, Relation

    ents, rels, trip, _, _ = world
    return KnowledgeGraph(
        tuple(Entity(i, tuple(ls)) for i, ls in ents),
        tuple(Relation(i, tuple(ls)) for i, ls in rels),
        tuple(tuple(t) for t in trip),
    )


def _edits(world, seed: int) -> dict:
    rng = random.Random(seed)
    ents, rels, trip, _, _ = world
    out = {}
    for v in range(2):
        edits = []
        for _ in range(6):
            s, r, _ = rng.choice(trip)
            kind = rng.random()
            if kind < 0.6:
                edits.append((s, r, rng.choice(ents)[0]))
            elif kind < 0.8:
                edits.append((s, r, None))
            else:
                edits.append((rng.choice(ents)[0], rng.choice(rels)[0], rng.choice(ents)[0]))
        out[f"v{v}"] = edits
    return out


def _closed(span):
    if span is None:
        return None
    return {
        "labels": [list(x) for x in span.labels], "entity_ids": list(span.entity_ids),
        "triples": [list(t) for t in span.triples], "resolved": span.resolved,
    }


def state_record(state) -> dict:
    """Every in-scope field of a reference OracleState, as JSON."""
    def hexed(b):
        return None if b is None else b.hex()

    return {
        "phase": state.phase.value, "tail": state.tail.hex(), "segment": state.segment.value,
        "subjects": sorted(state.subjects), "relations": sorted(state.relations),
        "written": [list(x) for x in state.written],
        "typed": None if state.typed is None else list(state.typed),
        "closing": hexed(state.closing), "closing_label": list(state.closing_label),
        "separating": hexed(state.separating), "separating_label": list(state.separating_label),
        "escaping": hexed(state.escaping), "last_span": _closed(state.last_span),
        "facts": [[list(x) for x in f] for f in state.facts],
        "reached": None if state.reached is None else sorted(state.reached),
        "ranks": sorted([list(x) for x in state.ranks]), "version": state.version,
        "answer_complete": state.answer_complete,
    }


def walk_case(args):
    root, worlds, case = args
    load_reference(Path(root))
    from xgraph.index import build_kg_index
    from xgraph.oracle import Oracle, Phase, Segment
    from xgraph.syntax import SpanSyntax

    name, world_name, options, versioned, anchored, opened = case
    world = worlds[world_name]
    served = _tokenizer(world[4])
    syntax = SpanSyntax()
    sitelinks = world[3] if options.get("start_rank") == "sitelinks" else None
    index = build_kg_index(_kg(world), served, syntax, sitelinks=sitelinks)
    versions = _edits(world, sum(map(ord, name)) + 7) if versioned else None
    options = dict(options)
    if options.get("end_after_answer"):
        options["eos_token_ids"] = sorted(served.special_ids)
    oracle = Oracle(index, served, syntax, versions=versions, **options)
    rng = random.Random(sum(map(ord, name)))
    names = [None, *(versions or {})]
    opener = served.encode(" " + syntax.opener)
    closer, separator = served.encode(syntax.closer), served.encode(syntax.separator)
    escape = served.encode(syntax.escape)
    regular = [t for t in range(served.vocab_size) if t not in served.special_ids]
    delims = [d.encode() for d in (syntax.closer, syntax.separator, syntax.escape)]
    delimiter_like = {
        t for t in regular
        if any(d.startswith(served.token_bytes(t), k) for d in delims for k in range(len(d)))
    }
    sequences = []
    masks = []
    for seq in range(SEQUENCES):
        version = names[seq % len(names)]
        anchor = None
        if anchored and seq % 2 == 1:
            with_edges = sorted({t[0] for t in world[2]})
            anchor = rng.sample(with_edges, 2)
            state = oracle.anchored_state(anchor, version)
        else:
            state = oracle.initial_state(version)
        if opened and seq % 2 == 0:
            state = oracle.opened_state(state)
        queue: list[int] = []
        tokens, states, seq_masks = [], [], []
        for _ in range(STEPS):
            allowed = oracle.allowed(state)
            words = np.zeros((served.vocab_size + 31) // 32, dtype=np.uint32)
            for t in allowed:
                words[t >> 5] |= np.uint32(1 << (t & 31))
            seq_masks.append(words)
            states.append(state_record(state))
            if not queue:
                in_span = state.phase is Phase.SPAN
                p = rng.random()
                if state.phase is Phase.FREE and p < 0.3:
                    queue = list(opener)
                elif in_span and separator[0] in allowed and p < 0.6:
                    queue = list(separator)
                elif in_span and closer[0] in allowed and p < 0.85 and (
                    state.segment is not Segment.SUBJECT or rng.random() < 0.5
                ):
                    queue = list(closer)
                elif in_span and p > 0.97:
                    queue = list(escape)
                elif state.phase is Phase.ESCAPED and p < 0.45:
                    queue = list(closer)
            label_tokens = sorted(allowed - delimiter_like)
            if queue and queue[0] in allowed:
                token = queue.pop(0)
            elif state.phase is Phase.SPAN and label_tokens and rng.random() < 0.85:
                queue = []
                token = rng.choice(label_tokens)
            else:
                queue = []
                pool = sorted(allowed & set(regular)) or sorted(allowed)
                token = rng.choice(pool)
            tokens.append(token)
            state = oracle.advance(state, token)
        sequences.append({"version": version, "anchor": anchor, "opened": bool(opened and seq % 2 == 0),
                          "tokens": tokens, "states": states, "final": state_record(state)})
        masks.append(np.stack(seq_masks))
    record = {"name": name, "world": world_name, "options": options,
              "versions": {k: [list(e) for e in v] for k, v in (versions or {}).items()},
              "sequences": sequences}
    vt = None
    if versions:
        from xgraph.kgversions import build_kg_versions

        kv = build_kg_versions(index, versions)
        vt = {k: np.asarray(v) for k, v in kv.native_tables().items()}
    return record, masks, vt


def index_arrays(root: Path, worlds: dict) -> dict:
    load_reference(root)
    from xgraph.index import build_kg_index
    from xgraph.syntax import SpanSyntax

    out = {}
    for name, world in worlds.items():
        index = build_kg_index(_kg(world), _tokenizer(world[4]), SpanSyntax(), sitelinks=world[3])
        for part in ("labels", "relations"):
            rows = getattr(index, part)
            for field in ("tokens", "offsets", "owners"):
                out[f"{name}/{part}.{field}"] = np.asarray(getattr(rows, field))
        for field in ("adjacency_offsets", "edge_relations", "edge_objects", "sitelinks"):
            out[f"{name}/{field}"] = np.asarray(getattr(index, field))
        out[f"{name}/unwritable"] = np.array([index.unwritable_triples])
        out[f"{name}/excluded"] = np.array(
            [f"{e.owner_id}\t{e.label}\t{e.reason}" for e in index.labels.excluded], dtype=object
        ).astype(str)
    return out


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, required=True, help="the reference checkout")
    args = parser.parse_args()
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    root = load_reference(args.reference)
    worlds = build_worlds(root)
    arrays = index_arrays(root, worlds)
    with ProcessPoolExecutor(max_workers=8) as pool:
        results = list(pool.map(walk_case, [(str(root), worlds, c) for c in CASES]))
    walks = []
    masks = {}
    for (record, seq_masks, vt), case in zip(results, CASES, strict=True):
        walks.append(record)
        for k, m in enumerate(seq_masks):
            masks[f"{case[0]}/{k}"] = m
        if vt:
            for key, value in vt.items():
                arrays[f"{case[0]}/{key}"] = value
    with gzip.open(HERE / "worlds.json.gz", "wt", encoding="utf-8") as f:
        json.dump({k: {"entities": v[0], "relations": v[1], "triples": v[2], "sitelinks": v[3],
                       "tokenizer": v[4]} for k, v in worlds.items()}, f)
    with gzip.open(HERE / "walks.json.gz", "wt", encoding="utf-8") as f:
        json.dump(walks, f, separators=(",", ":"))
    np.savez_compressed(HERE / "masks.npz", **masks)
    np.savez_compressed(HERE / "index.npz", **arrays)
    print(f"{len(walks)} cases, {sum(len(w['sequences']) for w in walks)} sequences")


if __name__ == "__main__":
    main()
