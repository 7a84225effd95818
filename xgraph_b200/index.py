"""KG index: tokenized label rows, relation rows and CSR adjacency.

The tables and their order are the reference's (src/xgraph/index.py:51-101, 181-233,
236-300, 403-516), because the engine's row ranges and the oracle's states name rows
by position:

- one label row per distinct (item, label) pair, holding the tokens of
  ``label_prefix + label``; blank labels, labels holding span syntax, and labels whose
  encoding does not round-trip to their exact bytes (exact-v1) are excluded;
- rows sorted as token tuples, a row that ends sorting before the rows that continue
  it, ties broken by item position; so a typed token prefix selects one contiguous row
  range, and inside it every token column is sorted;
- adjacency: for every writable triple, one edge per label row of the object, deduped,
  sorted by (subject, relation, object row), in CSR by subject position.

The build here is vectorised with numpy (lexsort on padded token columns, one int64
key per edge) so that million-entity graphs build in seconds; `build_kg_index_arrays`
takes numeric triples directly for graphs too large for Python tuples.
"""

from __future__ import annotations

import bisect
import hashlib
import json
import re
from collections.abc import Mapping, Sequence
from dataclasses import dataclass, field, replace
from pathlib import Path

import numpy as np

from .kg import Entity, KGFormatError, KnowledgeGraph, Relation, validate
from .syntax import SpanSyntax
from .tokenizer import ServedTokenizer

END = -1
"""Column value past a row's last token; sorts before every token id."""


class UnknownId(LookupError):
    """A query names an entity or relation the KG index does not hold."""


class IndexMismatch(ValueError):
    """The KG index, tokenizer, or KG-version base identity differs."""


@dataclass(frozen=True)
class ExcludedLabel:
    owner_id: str
    label: str
    reason: str


@dataclass(frozen=True)
class LabelIndex:
    """Sorted label rows: row r is ``tokens[offsets[r]:offsets[r+1]]``, naming
    ``owner_ids[owners[r]]``."""

    tokens: np.ndarray  # int32
    offsets: np.ndarray  # int64 [rows + 1]
    owners: np.ndarray  # int32 [rows]
    owner_ids: tuple[str, ...]
    tokenizer_fingerprint: str
    excluded: tuple[ExcludedLabel, ...]

    @property
    def num_rows(self) -> int:
        return len(self.owners)

    def row_tokens(self, row: int) -> tuple[int, ...]:
        a, b = int(self.offsets[row]), int(self.offsets[row + 1])
        return tuple(int(t) for t in self.tokens[a:b])

    def owner_id(self, row: int) -> str:
        return self.owner_ids[int(self.owners[row])]

    def token_at(self, row: int, depth: int) -> int:
        a, b = int(self.offsets[row]), int(self.offsets[row + 1])
        return int(self.tokens[a + depth]) if a + depth < b else END

    def prefix_range(self, prefix: Sequence[int]) -> tuple[int, int]:
        """Rows [lo, hi) whose tokens start with ``prefix`` (narrowed one column at a time)."""
        lo, hi = 0, self.num_rows
        for depth, token in enumerate(prefix):
            rows = range(lo, hi)

            def column(row: int, depth: int = depth) -> int:
                return self.token_at(row, depth)

            first = bisect.bisect_left(rows, token, key=column)
            last = bisect.bisect_right(rows, token, key=column)
            lo, hi = lo + first, lo + last
        return lo, hi


def _exact_v1_error(label: str, tokens: list[int], tokenizer, syntax: SpanSyntax) -> str | None:
    """exact-v1 label admission (src/xgraph/index.py:167-178): no special tokens, a
    nonempty encoding, known bytes for every token, and bytes equal to prefix + label."""
    if tokenizer.special_ids.intersection(tokens):
        return "label contains a special token"
    if not tokens:
        return "empty label encoding"
    pieces = [tokenizer.token_bytes(t) for t in tokens]
    if any(p is None for p in pieces):
        return "label contains a token with unknown bytes"
    if b"".join(pieces) != (syntax.label_prefix + label).encode("utf-8"):
        return "label bytes do not round-trip"
    return None


def _sorted_rows(rows: list[tuple[list[int], int]]) -> list[int]:
    """Permutation sorting (tokens, item) pairs as Python tuples would sort."""
    n = len(rows)
    if n == 0:
        return []
    lengths = np.fromiter((len(t) for t, _ in rows), dtype=np.int64, count=n)
    width = int(lengths.max())
    if width > 64:  # long labels: the plain tuple sort
        return sorted(range(n), key=lambda i: (tuple(rows[i][0]), rows[i][1]))
    padded = np.full((n, width), END, dtype=np.int64)
    flat = np.fromiter((t for toks, _ in rows for t in toks), dtype=np.int64, count=int(lengths.sum()))
    row_of = np.repeat(np.arange(n), lengths)
    col_of = np.arange(len(flat)) - np.repeat(np.cumsum(lengths) - lengths, lengths)
    padded[row_of, col_of] = flat
    items = np.fromiter((i for _, i in rows), dtype=np.int64, count=n)
    keys = [items] + [padded[:, c] for c in range(width - 1, -1, -1)]
    return np.lexsort(keys).tolist()


def _excluder(syntax: SpanSyntax):
    """SpanSyntax.excludes as one compiled test: a delimiter or the operand separator
    anywhere in the written label, or an operator at its start."""
    inner = [*syntax.delimiters, *([syntax.operand_separator] if syntax.operand_separator else [])]
    anywhere = re.compile("|".join(re.escape(d) for d in inner))
    starts = tuple(syntax.label_prefix + op for op in syntax.operators)
    prefix = syntax.label_prefix

    def excludes(label: str) -> bool:
        written = prefix + label
        return anywhere.search(written) is not None or (bool(starts) and written.startswith(starts))

    return excludes


ADMISSION_REASONS = {1: "label contains a special token", 2: "empty label encoding",
                     3: "label contains a token with unknown bytes", 4: "label bytes do not round-trip"}
"""Reasons of the exact-v1 admission failures, by the device build's status code."""


def label_rows(
    items: Sequence[Entity | Relation] | Sequence[tuple[str, Sequence[str]]],
    tokenizer: ServedTokenizer,
    syntax: SpanSyntax,
    device=None,
) -> LabelIndex:
    """The label index over these items' labels (src/xgraph/index.py:181-233).  With
    `device` (a CUDA device) the admission checks, the row sort and the row arrays run
    there (xg_build_label_rows); the tokenizer encodes on the host either way."""
    pairs: list[tuple[str, int]] = []
    excluded: list[ExcludedLabel] = []
    ids: list[str] = []
    excludes = _excluder(syntax)
    for position, item in enumerate(items):
        item_id, labels = (item.id, item.labels) if hasattr(item, "id") else item
        ids.append(item_id)
        seen: set[str] = set()
        for label in labels:
            if label in seen:
                continue
            seen.add(label)
            if not label.strip():
                excluded.append(ExcludedLabel(item_id, label, "blank label"))
            elif excludes(label):
                excluded.append(ExcludedLabel(item_id, label, "label contains span syntax"))
            else:
                pairs.append((label, position))
    encoded = tokenizer.encode_batch([syntax.label_prefix + label for label, _ in pairs])
    if device is not None:
        tokens, offsets, owners, status = _label_rows_device(pairs, encoded, len(ids), tokenizer, syntax, device)
        excluded.extend(ExcludedLabel(ids[pairs[i][1]], pairs[i][0], ADMISSION_REASONS[int(status[i])])
                        for i in np.flatnonzero(status))
        return LabelIndex(tokens=tokens, offsets=offsets, owners=owners, owner_ids=tuple(ids),
                          tokenizer_fingerprint=tokenizer.fingerprint, excluded=tuple(excluded))
    rows: list[tuple[list[int], int]] = []
    for (label, position), tokens in zip(pairs, encoded, strict=True):
        reason = _exact_v1_error(label, tokens, tokenizer, syntax)
        if reason:
            excluded.append(ExcludedLabel(ids[position], label, reason))
        else:
            rows.append((tokens, position))
    order = _sorted_rows(rows)
    lengths = np.array([len(rows[i][0]) for i in order], dtype=np.int64)
    offsets = np.zeros(len(order) + 1, dtype=np.int64)
    np.cumsum(lengths, out=offsets[1:])
    tokens = np.fromiter(
        (t for i in order for t in rows[i][0]), dtype=np.int32, count=int(offsets[-1])
    )
    owners = np.array([rows[i][1] for i in order], dtype=np.int32)
    return LabelIndex(
        tokens=tokens,
        offsets=offsets,
        owners=owners,
        owner_ids=tuple(ids),
        tokenizer_fingerprint=tokenizer.fingerprint,
        excluded=tuple(excluded),
    )


def _label_rows_device(pairs, encoded, owner_count: int, tokenizer: ServedTokenizer, syntax: SpanSyntax, device):
    """label_rows' admission and row arrays on a GPU (xg_build_label_rows): (tokens,
    offsets, owners, status per pair), the same arrays as the host build's."""
    import ctypes
    import itertools

    import torch

    from .engine import _check, load_library

    lib = load_library()
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError(f"the device label build needs a CUDA device, got {device}")
    n = len(pairs)
    lengths = np.fromiter(map(len, encoded), dtype=np.int64, count=n)
    token_off = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(lengths, out=token_off[1:])
    token_ids = np.fromiter(itertools.chain.from_iterable(encoded), dtype=np.int32, count=int(token_off[-1]))
    written = [(syntax.label_prefix + label).encode("utf-8") for label, _ in pairs]
    text_off = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(np.fromiter(map(len, written), dtype=np.int64, count=n), out=text_off[1:])
    text = np.frombuffer(bytearray(b"".join(written)), dtype=np.uint8)
    owners = np.fromiter((position for _, position in pairs), dtype=np.int32, count=n)
    vocab_off, vocab_bytes, vocab_kind = tokenizer.byte_table()
    with torch.cuda.device(device):
        def put(array, dtype):
            return torch.from_numpy(np.ascontiguousarray(array)).to(device=device, dtype=dtype)

        def ptr(t):
            return ctypes.c_void_p(t.data_ptr())

        d_token_off, d_ids = put(token_off, torch.int64), put(token_ids, torch.int32)
        d_text_off, d_text = put(text_off, torch.int64), put(text, torch.uint8)
        d_owners = put(owners, torch.int32)
        d_vocab_off, d_vocab_bytes = put(vocab_off, torch.int64), put(vocab_bytes, torch.uint8)
        d_kind = put(vocab_kind, torch.int8)
        status = torch.empty(max(n, 1), dtype=torch.int32, device=device)
        row_offsets = torch.empty(n + 1, dtype=torch.int64, device=device)
        row_tokens = torch.empty(max(len(token_ids), 1), dtype=torch.int32, device=device)
        row_owners = torch.empty(max(n, 1), dtype=torch.int32, device=device)
        rows, total = ctypes.c_int32(), ctypes.c_int64()
        stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        _check(lib.xg_build_label_rows(
            n, ptr(d_token_off), ptr(d_ids), len(token_ids), ptr(d_text_off), ptr(d_text), len(text), ptr(d_owners),
            owner_count, len(vocab_kind), ptr(d_vocab_off), ptr(d_vocab_bytes), len(vocab_bytes), ptr(d_kind),
            ptr(status), ptr(row_offsets), ptr(row_tokens), ptr(row_owners), ctypes.byref(rows), ctypes.byref(total),
            stream))
        r, t = rows.value, total.value
        return (row_tokens[:t].cpu().numpy(), row_offsets[: r + 1].cpu().numpy(), row_owners[:r].cpu().numpy(),
                status[:n].cpu().numpy())


def entity_row_lists(labels: LabelIndex) -> tuple[np.ndarray, np.ndarray]:
    """Each owner's rows in row order, as CSR: (offsets [owners + 1] int64, rows int32)."""
    owners = np.asarray(labels.owners, dtype=np.int64)
    count = len(labels.owner_ids)
    order = np.argsort(owners, kind="stable").astype(np.int32)
    offsets = np.zeros(count + 1, dtype=np.int64)
    np.cumsum(np.bincount(owners, minlength=count), out=offsets[1:])
    return offsets, order


@dataclass(frozen=True)
class KGIndex:
    """A source KG compiled for one served tokenizer and span syntax."""

    labels: LabelIndex
    relations: LabelIndex
    adjacency_offsets: np.ndarray  # int64 [entities + 1]
    edge_relations: np.ndarray  # int32 [edges]
    edge_objects: np.ndarray  # int32 [edges], object label rows
    unwritable_triples: int
    span_syntax: SpanSyntax = field(default_factory=SpanSyntax)
    sitelinks: np.ndarray | None = None
    date_entities: np.ndarray | None = None
    date_keys: np.ndarray | None = None
    verdicts: dict[str, str] | None = None
    expressions: bool = True
    base_fingerprint: str = ""

    @property
    def tokenizer_fingerprint(self) -> str:
        return self.labels.tokenizer_fingerprint

    def edges_at(self, entity: int) -> tuple[np.ndarray, np.ndarray]:
        a, b = int(self.adjacency_offsets[entity]), int(self.adjacency_offsets[entity + 1])
        return self.edge_relations[a:b], self.edge_objects[a:b]

    def _position(self, table: str, item: str, kind: str) -> int:
        cache = self.__dict__.get(table)
        if cache is None:
            owner_ids = self.labels.owner_ids if table == "_entity_at" else self.relations.owner_ids
            cache = {name: n for n, name in enumerate(owner_ids)}
            object.__setattr__(self, table, cache)
        if item not in cache:
            raise UnknownId(f"the KG index holds no {kind} {item!r}")
        return cache[item]

    def relations_of(self, subject: str) -> list[str]:
        relations, _ = self.edges_at(self._position("_entity_at", subject, "entity"))
        return [self.relations.owner_ids[r] for r in np.unique(relations)]

    def object_rows(self, subject: str, relation: str, lo: int = 0, hi: int | None = None) -> list[int]:
        relations, objects = self.edges_at(self._position("_entity_at", subject, "entity"))
        r = self._position("_relation_at", relation, "relation")
        a, b = np.searchsorted(relations, r, "left"), np.searchsorted(relations, r, "right")
        objects = objects[a:b]
        hi = self.labels.num_rows if hi is None else hi
        x, y = np.searchsorted(objects, lo, "left"), np.searchsorted(objects, hi, "left")
        return [int(o) for o in objects[x:y]]


def _fingerprint(index_parts: dict) -> str:
    digest = hashlib.sha256()
    for name in sorted(index_parts):
        value = index_parts[name]
        digest.update(name.encode())
        if isinstance(value, np.ndarray):
            digest.update(str((value.dtype.str, value.shape)).encode())
            digest.update(np.ascontiguousarray(value).tobytes())
        else:
            digest.update(json.dumps(value, sort_keys=True, default=str).encode())
    return digest.hexdigest()


def sitelink_array(counts, entities: int) -> np.ndarray:
    array = np.asarray(counts, dtype=np.int64).reshape(-1)
    if len(array) != entities:
        raise ValueError(
            f"a KG index needs one sitelink count per entity ({entities}), got {len(array)}"
        )
    if len(array) and int(array.min()) < 0:
        raise ValueError(f"sitelink counts cannot be negative, got {int(array.min())}")
    if len(array) and int(array.max()) > np.iinfo(np.int32).max:
        raise ValueError(f"a sitelink count of {int(array.max())} does not fit in int32")
    return array.astype(np.int32)


def _adjacency(
    labels: LabelIndex, writable_relations: np.ndarray, subjects: np.ndarray,
    relations: np.ndarray, objects: np.ndarray, entities: int,
) -> tuple[np.ndarray, np.ndarray, np.ndarray, int]:
    """CSR edges from position triples: one edge per object label row, deduped and sorted."""
    row_offsets, row_list = entity_row_lists(labels)
    row_counts = np.diff(row_offsets)
    ok = (row_counts[subjects] > 0) & (row_counts[objects] > 0) & writable_relations[relations]
    unwritable = int(len(subjects) - int(ok.sum()))
    s, r, o = subjects[ok].astype(np.int64), relations[ok].astype(np.int64), objects[ok]
    repeat = row_counts[o]
    starts = np.repeat(row_offsets[o], repeat)
    within = np.arange(int(repeat.sum()), dtype=np.int64) - np.repeat(np.cumsum(repeat) - repeat, repeat)
    rows = row_list[starts + within].astype(np.int64)
    s, r = np.repeat(s, repeat), np.repeat(r, repeat)
    n_rel = max(1, len(writable_relations))
    n_rows = max(1, labels.num_rows)
    if entities * n_rel * n_rows < (1 << 62):
        keys = np.unique((s * n_rel + r) * n_rows + rows)
        rows_out = keys % n_rows
        rel_out = (keys // n_rows) % n_rel
        subj_out = keys // (n_rows * n_rel)
    else:  # pragma: no cover - astronomically large indexes
        stacked = np.unique(np.stack([s, r, rows], axis=1), axis=0)
        subj_out, rel_out, rows_out = stacked[:, 0], stacked[:, 1], stacked[:, 2]
    offsets = np.zeros(entities + 1, dtype=np.int64)
    np.cumsum(np.bincount(subj_out, minlength=entities), out=offsets[1:])
    return offsets, rel_out.astype(np.int32), rows_out.astype(np.int32), unwritable


def _adjacency_device(
    labels: LabelIndex, writable_relations: np.ndarray, subjects: np.ndarray,
    relations: np.ndarray, objects: np.ndarray, entities: int, device,
) -> tuple[np.ndarray, np.ndarray, np.ndarray, int]:
    """_adjacency's arrays built on a GPU by the library's xg_build_adjacency (expand,
    radix sort, unique and CSR scan on the device), copied back to the host."""
    import ctypes

    import torch

    from .engine import _check, load_library

    lib = load_library()
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError(f"the device adjacency build needs a CUDA device, got {device}")
    row_offsets, row_list = entity_row_lists(labels)
    with torch.cuda.device(device):
        def put(array, dtype):
            return torch.from_numpy(np.ascontiguousarray(array)).to(device=device, dtype=dtype)

        s, r, o = put(subjects, torch.int32), put(relations, torch.int32), put(objects, torch.int32)
        offsets_in, rows_in = put(row_offsets, torch.int64), put(row_list, torch.int32)
        writable = put(np.asarray(writable_relations, dtype=np.uint8), torch.uint8)
        stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        edges, unwritable = ctypes.c_int64(), ctypes.c_int64()

        def ptr(t):
            return ctypes.c_void_p(t.data_ptr())

        head = (ptr(s), ptr(r), ptr(o), len(subjects), ptr(offsets_in), ptr(rows_in), entities, labels.num_rows,
                ptr(writable), len(writable_relations))
        _check(lib.xg_build_adjacency(*head, 0, None, None, None, ctypes.byref(edges), ctypes.byref(unwritable), stream))
        capacity = edges.value
        offsets = torch.empty(entities + 1, dtype=torch.int64, device=device)
        edge_rel = torch.empty(max(capacity, 1), dtype=torch.int32, device=device)
        edge_obj = torch.empty(max(capacity, 1), dtype=torch.int32, device=device)
        _check(lib.xg_build_adjacency(*head, capacity, ptr(offsets), ptr(edge_rel), ptr(edge_obj), ctypes.byref(edges),
                                      ctypes.byref(unwritable), stream))
        n = edges.value
        return (offsets.cpu().numpy(), edge_rel[:n].cpu().numpy(), edge_obj[:n].cpu().numpy(),
                int(unwritable.value))


def check_expressions(index: KGIndex) -> None:
    """Refuse an index expressions cannot run on (src/xgraph/index.py:686-704): one built
    for a span syntax without operators, one whose labels may hold expression syntax, one
    without the date table."""
    if not index.span_syntax.writes_expressions:
        raise ValueError("expressions need a KG index built for a span syntax with operators and an "
                         f"operand separator, not {index.span_syntax}")
    if not index.expressions:
        raise ValueError("the KG index was saved before labels holding expression syntax were excluded: rebuild it")
    if index.date_entities is None:
        raise ValueError("expressions need a KG index with the date table")


def build_kg_index_arrays(
    entities: Sequence[tuple[str, Sequence[str]]],
    relations: Sequence[tuple[str, Sequence[str]]],
    triples: np.ndarray,
    tokenizer: ServedTokenizer,
    syntax: SpanSyntax,
    sitelinks: np.ndarray | Sequence[int] | None = None,
    device=None,
    *,
    dates: tuple[np.ndarray, np.ndarray] | None = None,
    verdicts: dict[str, str] | None = None,
) -> KGIndex:
    """The KG index of entities and relations given as (id, labels) and triples given as
    an int (n, 3) array of (subject position, relation position, object position).
    `device` (a CUDA device): the edge arrays are built there by the library (the same
    arrays as the host build's); None builds everything on the host.  `dates`: the date
    table (xgraph_b200.dates.date_table); `verdicts`: the verdict entities by verdict,
    which the entities must already hold."""
    triples = np.asarray(triples, dtype=np.int64).reshape(-1, 3)
    if len(triples) and (
        triples.min() < 0
        or triples[:, 0].max() >= len(entities)
        or triples[:, 2].max() >= len(entities)
        or triples[:, 1].max() >= len(relations)
    ):
        raise KGFormatError("triples name entity or relation positions outside the KG")
    labels = label_rows(entities, tokenizer, syntax, device=device)
    relation_index = label_rows(relations, tokenizer, syntax, device=device)
    writable = np.zeros(len(relations), dtype=bool)
    writable[np.asarray(relation_index.owners, dtype=np.int64)] = True
    if device is None:
        offsets, edge_rel, edge_obj, unwritable = _adjacency(
            labels, writable, triples[:, 0], triples[:, 1], triples[:, 2], len(entities)
        )
    else:
        offsets, edge_rel, edge_obj, unwritable = _adjacency_device(
            labels, writable, triples[:, 0], triples[:, 1], triples[:, 2], len(entities), device
        )
    counts = None if sitelinks is None else sitelink_array(sitelinks, len(entities))
    parts = {
        "labels.tokens": labels.tokens, "labels.offsets": labels.offsets,
        "labels.owners": labels.owners, "labels.ids": list(labels.owner_ids),
        "relations.tokens": relation_index.tokens, "relations.offsets": relation_index.offsets,
        "relations.owners": relation_index.owners, "relations.ids": list(relation_index.owner_ids),
        "adjacency_offsets": offsets, "edge_relations": edge_rel, "edge_objects": edge_obj,
        "tokenizer": tokenizer.fingerprint, "syntax": repr(syntax),
        "sitelinks": counts if counts is not None else "none",
    }
    if dates is not None:
        parts["date_entities"], parts["date_keys"] = dates
    if verdicts is not None:
        parts["verdicts"] = verdicts
    return KGIndex(
        labels=labels,
        relations=relation_index,
        adjacency_offsets=offsets,
        edge_relations=edge_rel,
        edge_objects=edge_obj,
        unwritable_triples=unwritable,
        span_syntax=syntax,
        sitelinks=counts,
        date_entities=None if dates is None else dates[0],
        date_keys=None if dates is None else dates[1],
        verdicts=verdicts,
        base_fingerprint=_fingerprint(parts),
    )


def build_kg_index(
    kg: KnowledgeGraph,
    tokenizer: ServedTokenizer,
    syntax: SpanSyntax,
    sitelinks: Mapping[str, int] | None = None,
    dates=None,
    verdicts: bool = False,
    *,
    initial_case_aliases: bool = False,
) -> KGIndex:
    """The KG index of an in-memory KG (src/xgraph/index.py:403-516).  With dates (Date
    values by entity id) the index holds the date table of date comparisons; with verdicts
    the verdict entities (xgraph_b200.dates.VERDICTS, each labelled with its verdict) are
    appended to the KG's entities.  Initial-case aliases feed the reference's alias policy,
    which this engine does not implement; asking for them raises ValueError."""
    from .dates import VERDICTS, date_table

    if initial_case_aliases:
        raise ValueError("initial_case_aliases belongs to a policy this engine does not implement")
    validate(kg)
    if verdicts:
        taken = sorted(set(VERDICTS.values()) & {e.id for e in kg.entities})
        if taken:
            raise KGFormatError(f"the KG holds {taken}, the ids of the verdict entities")
        kg = KnowledgeGraph((*kg.entities, *(Entity(i, (v,)) for v, i in VERDICTS.items())), kg.relations,
                            kg.triples)
    entity_at = {e.id: n for n, e in enumerate(kg.entities)}
    relation_at = {r.id: n for n, r in enumerate(kg.relations)}
    triples = np.array(
        [(entity_at[s], relation_at[r], entity_at[o]) for s, r, o in kg.triples], dtype=np.int64
    ).reshape(-1, 3)
    counts = None
    if sitelinks is not None:
        counts = [sitelinks.get(e.id, 0) for e in kg.entities]
    table = None
    if dates is not None:
        unknown = sorted(set(dates) - set(entity_at))
        if unknown:
            raise KGFormatError(f"dates name entities the KG lacks: {unknown[:5]}")
        table = date_table({entity_at[e]: d for e, d in dates.items()})
    return build_kg_index_arrays(
        [(e.id, e.labels) for e in kg.entities],
        [(r.id, r.labels) for r in kg.relations],
        triples,
        tokenizer,
        syntax,
        sitelinks=counts,
        dates=table,
        verdicts=dict(VERDICTS) if verdicts else None,
    )


def relation_names(rows, unique_aliases: bool = False) -> dict[str, list[str]]:
    """Each property's names from relation label rows (property, label, kind), labels
    first (src/xgraph/wikidata.py:835-857): an alias that is, ignoring case, another
    property's label is dropped, and with unique_aliases so is an alias several
    properties share (a path naming it would follow every one of them)."""
    rows = [tuple(row) for row in rows]
    labels = {label.casefold(): prop for prop, label, kind in rows if kind == "label"}
    owners: dict[str, set[str]] = {}
    for prop, label, kind in rows:
        if kind != "label":
            owners.setdefault(label.casefold(), set()).add(prop)
    names: dict[str, list[str]] = {}
    for prop, label, kind in sorted(rows, key=lambda row: row[2] != "label"):
        if kind != "label" and labels.get(label.casefold(), prop) != prop:
            continue
        if kind != "label" and unique_aliases and len(owners[label.casefold()]) > 1:
            continue
        names.setdefault(prop, []).append(label)
    return names


KG_DIRECTORY_FILES = ("entity_labels.jsonl", "relation_labels.jsonl", "triples.npy")
SITELINK_COUNTS = "sitelink_counts.npy"


def build_kg_directory_index(
    kg: str | Path, tokenizer: ServedTokenizer, syntax: SpanSyntax, unique_aliases: bool = False, device=None,
) -> KGIndex:
    """The KG index of a KG directory in the reference's layout (src/xgraph/wikidata.py:
    859-1037): entity_labels.jsonl and relation_labels.jsonl hold one JSON list [id,
    label, "label" | "alias"] per line (items Q<n>, properties P<n>), triples.npy the
    (subject item, property, object item) numbers, sitelink_counts.npy (optional) [item,
    count] rows.  Entities are the items with a label row, in item-number order, each with
    its labels in file order; relations the properties relation_names keeps, in number
    order; a triple naming an item or property without one is unwritable, like a triple
    whose subject, object or relation has no label row.  The arrays equal the reference
    builder's; `device` builds the edge arrays on that GPU.  The directory's date tables
    and RDF ids are not read: an index for expressions takes its dates in memory
    (build_kg_index's `dates`) or from a saved index that holds them."""
    kg = Path(kg)
    for name in KG_DIRECTORY_FILES:
        if not (kg / name).is_file():
            raise KGFormatError(f"{kg} is not a KG directory: {name} is missing")

    def records(name: str) -> list[tuple]:
        with (kg / name).open(encoding="utf-8") as lines:
            return [tuple(json.loads(line)) for line in lines if line.strip()]

    def number(identifier: str, prefix: str) -> int:
        if not (isinstance(identifier, str) and identifier[:1] == prefix and identifier[1:].isdigit()):
            raise KGFormatError(f"{kg}: {identifier!r} is not a {prefix}<number> id")
        return int(identifier[1:])

    labels_of: dict[int, list[str]] = {}
    for identifier, label, _kind in records("entity_labels.jsonl"):
        labels_of.setdefault(number(identifier, "Q"), []).append(label)
    items = np.array(sorted(labels_of), dtype=np.int64)
    entities = [(f"Q{n}", labels_of[n]) for n in items.tolist()]
    names = relation_names(records("relation_labels.jsonl"), unique_aliases)
    properties = sorted(names, key=lambda p: number(p, "P"))
    relations = [(p, names[p]) for p in properties]
    numbers = np.array([number(p, "P") for p in properties], dtype=np.int64)

    def positions(known: np.ndarray, wanted: np.ndarray) -> np.ndarray:
        if not len(known):
            return np.full(len(wanted), -1, dtype=np.int64)
        at = np.minimum(np.searchsorted(known, wanted), len(known) - 1)
        return np.where(known[at] == wanted, at, -1)

    raw = np.asarray(np.load(kg / "triples.npy"), dtype=np.int64).reshape(-1, 3)
    found = np.stack([positions(items, raw[:, 0]), positions(numbers, raw[:, 1]), positions(items, raw[:, 2])], axis=1)
    known = (found >= 0).all(axis=1)
    sitelinks = None
    if (kg / SITELINK_COUNTS).is_file():
        table = np.asarray(np.load(kg / SITELINK_COUNTS), dtype=np.int64).reshape(-1, 2)
        order = np.argsort(table[:, 0], kind="stable")
        at = positions(table[order, 0], items)
        sitelinks = np.where(at >= 0, table[order, 1][np.maximum(at, 0)] if len(table) else 0, 0)
    index = build_kg_index_arrays(entities, relations, found[known], tokenizer, syntax, sitelinks=sitelinks,
                                  device=device)
    return replace(index, unwritable_triples=index.unwritable_triples + int((~known).sum()))


START_RANKS = ("degree", "sitelinks")


def check_start_rank(start_rank: str, index) -> str:
    if start_rank not in START_RANKS:
        raise ValueError(f"start_rank must be one of {START_RANKS}, got {start_rank!r}")
    if start_rank == "sitelinks":
        if index.sitelinks is None:
            raise ValueError("the sitelink rank needs a KG index with sitelink counts")
        sitelink_array(index.sitelinks, len(index.labels.owner_ids))
    return start_rank


def save_kg_index(index: KGIndex, directory: str | Path) -> None:
    """Write the index as one .npz of arrays plus a JSON header of ids and identity."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    arrays = {
        "labels_tokens": index.labels.tokens, "labels_offsets": index.labels.offsets,
        "labels_owners": index.labels.owners, "relations_tokens": index.relations.tokens,
        "relations_offsets": index.relations.offsets, "relations_owners": index.relations.owners,
        "adjacency_offsets": index.adjacency_offsets, "edge_relations": index.edge_relations,
        "edge_objects": index.edge_objects,
    }
    if index.sitelinks is not None:
        arrays["sitelinks"] = index.sitelinks
    if index.date_entities is not None:
        arrays["date_entities"], arrays["date_keys"] = index.date_entities, index.date_keys
    np.savez(directory / "kg-index.npz", **arrays)
    header = {
        "format": "xgraph-b200-index-1",
        "tokenizer_fingerprint": index.tokenizer_fingerprint,
        "span_syntax": {k: getattr(index.span_syntax, k) for k in index.span_syntax.__dataclass_fields__},
        "unwritable_triples": index.unwritable_triples,
        "labels": {"owner_ids": list(index.labels.owner_ids),
                   "excluded": [[e.owner_id, e.label, e.reason] for e in index.labels.excluded]},
        "relations": {"owner_ids": list(index.relations.owner_ids),
                      "excluded": [[e.owner_id, e.label, e.reason] for e in index.relations.excluded]},
        "base_fingerprint": index.base_fingerprint,
        "verdicts": index.verdicts,
    }
    (directory / "kg-index.json").write_text(json.dumps(header) + "\n", encoding="utf-8")


REFERENCE_INDEX_FORMAT = 1
"""The reference's saved-index layout (src/xgraph/index.py:711), which load_kg_index reads."""


def load_kg_index(directory: str | Path) -> KGIndex:
    """Read a KG index saved by save_kg_index, or by the reference's save_kg_index (one .npy
    file per array and kg-index.json, src/xgraph/index.py:731-903), with its date table and
    verdict entities.  A reference index that carries initial-case aliases (a policy this
    engine does not serve) is refused."""
    directory = Path(directory)
    header = json.loads((directory / "kg-index.json").read_text(encoding="utf-8"))
    if header.get("format") == REFERENCE_INDEX_FORMAT:
        return _load_reference_index(directory, header)
    if header.get("format") != "xgraph-b200-index-1":
        raise ValueError(f"{directory} holds no index of this library's or the reference's format")
    data = np.load(directory / "kg-index.npz")
    syntax = SpanSyntax(**header["span_syntax"])

    def part(name: str) -> LabelIndex:
        return LabelIndex(
            tokens=data[f"{name}_tokens"], offsets=data[f"{name}_offsets"],
            owners=data[f"{name}_owners"], owner_ids=tuple(header[name]["owner_ids"]),
            tokenizer_fingerprint=header["tokenizer_fingerprint"],
            excluded=tuple(ExcludedLabel(*e) for e in header[name]["excluded"]),
        )

    return KGIndex(
        labels=part("labels"), relations=part("relations"),
        adjacency_offsets=data["adjacency_offsets"], edge_relations=data["edge_relations"],
        edge_objects=data["edge_objects"], unwritable_triples=header["unwritable_triples"],
        span_syntax=syntax, sitelinks=data["sitelinks"] if "sitelinks" in data else None,
        date_entities=data["date_entities"] if "date_entities" in data else None,
        date_keys=data["date_keys"] if "date_keys" in data else None,
        verdicts=header.get("verdicts"), base_fingerprint=header["base_fingerprint"],
    )


def _load_reference_index(directory: Path, header: dict) -> KGIndex:
    """The reference's saved index (format 1) as this library's KGIndex; its recorded base
    fingerprint is kept when it has one, else this library's is computed."""
    if header.get("initial_case_aliases"):
        raise ValueError(f"{directory}: the index carries initial_case_aliases, which this engine does not serve")

    def array(name: str) -> np.ndarray:
        file = directory / f"{name}.npy"
        if not file.is_file():
            raise ValueError(f"{directory} misses {file.name}")
        return np.load(file)

    known = SpanSyntax.__dataclass_fields__
    syntax_fields = {k: tuple(v) if isinstance(v, list) else v for k, v in header.get("span_syntax", {}).items()
                     if k in known}
    syntax = SpanSyntax(**syntax_fields)

    def part(name: str) -> LabelIndex:
        return LabelIndex(
            tokens=array(f"{name}.tokens"), offsets=array(f"{name}.offsets"), owners=array(f"{name}.owners"),
            owner_ids=tuple(header[name]["owner_ids"]), tokenizer_fingerprint=header["tokenizer_fingerprint"],
            excluded=tuple(ExcludedLabel(*e) for e in header[name]["excluded"]),
        )

    labels, relations = part("labels"), part("relations")
    offsets, edge_rel, edge_obj = array("adjacency_offsets"), array("edge_relations"), array("edge_objects")
    sitelinks = array("sitelinks") if header.get("sitelinks") else None
    dates = (array("date_entities"), array("date_keys")) if header.get("dates") else None
    parts = {
        "labels.tokens": labels.tokens, "labels.offsets": labels.offsets, "labels.owners": labels.owners,
        "labels.ids": list(labels.owner_ids), "relations.tokens": relations.tokens,
        "relations.offsets": relations.offsets, "relations.owners": relations.owners,
        "relations.ids": list(relations.owner_ids), "adjacency_offsets": offsets, "edge_relations": edge_rel,
        "edge_objects": edge_obj, "tokenizer": header["tokenizer_fingerprint"], "syntax": repr(syntax),
        "sitelinks": sitelinks if sitelinks is not None else "none",
    }
    if dates is not None:
        parts["date_entities"], parts["date_keys"] = dates
    if header.get("verdicts") is not None:
        parts["verdicts"] = header["verdicts"]
    fingerprint = header.get("base_fingerprint") or _fingerprint(parts)
    return KGIndex(labels=labels, relations=relations, adjacency_offsets=offsets, edge_relations=edge_rel,
                   edge_objects=edge_obj, unwritable_triples=header["unwritable_triples"], span_syntax=syntax,
                   sitelinks=sitelinks, date_entities=None if dates is None else dates[0],
                   date_keys=None if dates is None else dates[1], verdicts=header.get("verdicts"),
                   expressions=bool(header.get("expressions", False)), base_fingerprint=fingerprint)


def main(argv: list[str] | None = None) -> None:
    """Build and save the KG index of a KG directory (the reference's
    `python -m xgraph.wikidata index`, src/xgraph/wikidata.py:1040-1139, for the
    policies this engine serves); --device builds the edge arrays on that GPU."""
    import argparse

    from .syntax import preset
    from .tokenizer import ServedTokenizer

    parser = argparse.ArgumentParser(prog="python -m xgraph_b200.index", description=main.__doc__)
    parser.add_argument("--kg", type=Path, required=True, help="KG directory (entity/relation label rows, triples)")
    parser.add_argument("--tokenizer", type=Path, required=True, help="served tokenizer.json")
    parser.add_argument("--out", type=Path, required=True, help="KG index directory to write")
    parser.add_argument("--syntax", default="brackets", help="span syntax preset the index is built for")
    parser.add_argument("--unique-aliases", action="store_true",
                        help="drop relation aliases that several properties share")
    parser.add_argument("--device", default=None, help="a CUDA device for the edge build (default: the host)")
    args = parser.parse_args(argv)
    index = build_kg_directory_index(args.kg, ServedTokenizer.from_file(args.tokenizer), preset(args.syntax),
                                     unique_aliases=args.unique_aliases, device=args.device)
    save_kg_index(index, args.out)
    print(f"{args.out}: {len(index.labels.owner_ids):,} entities, {index.labels.num_rows:,} label rows, "
          f"{len(index.relations.owner_ids):,} relations, {len(index.edge_objects):,} edges, "
          f"{index.unwritable_triples:,} unwritable triples")


if __name__ == "__main__":
    main()
