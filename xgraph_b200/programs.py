"""Offline execution of written paths on the GPU: the reference's MatchedExecutor
(src/xgraph/programs.py:328-1130), path mode with committed paths run after decoding.

A path written without the engine, `start · r1 · ... · rk` (parsed from a model's output),
executes as path mode would have executed it: labels read as the label index's rows, a
relation label or alias following every relation it names, starts in best-connected order
capped at 64, each frontier capped at 64 by start rank and first label row, the path
resolving to the entities of the least start rank present, and the answer the best
connected of the entities the answer span after the path may name (the first 64 label rows
of those entities).

Here the engine itself executes them: each path becomes the token stream of its span
(`⟦ start · r1 · ... · rk⟧`, each piece encoded on its own as the reference's `_rows`
reads a label: the label prefix and the text), one slot per path reading the path's KG
version, and a whole batch runs as one sync launch up to the last relation label and one
more for the closer.  The slot's memory then holds, from set_flags' separator test, the
capped next frontier with its start ranks (the path's last frontier), and after the closer
the reached label rows.  Only the final ordering (best-connected order: most sitelinks
with the sitelink rank, then most adjacency entries in the path's version, then first
label row) and the id lookups run on the host.  A path the engine would not have let be
written (a start naming nothing with triples, a relation the frontier lacks, a label cut
short) leaves its slot in the error phase and executes to nothing, as the reference's
executor returns for it.

Anchored paths start from the anchor's entities their start label names (each anchored
slot admitted with the anchor's label rows); a start naming none of them starts from every
anchor entity, as the reference's does, written with a label that names them all (refused
where no one label does).  With repair, an unknown relation is replaced, hop by hop, by the
frontier's most similar relation written with a label of its own (refused where it has
none).  With strip_quotes, a start naming nothing to start from is read without the
quotation marks wrapping it where that names something (MatchedPath.stripped).  Not
served (refused by name): the observation / menu / audit settings.
"""

from __future__ import annotations

from collections.abc import Iterable, Sequence
from dataclasses import dataclass, replace

import numpy as np

MAX_PATH_RELATIONS = 8  # src/xgraph/oracle.py:177
MAX_REACHED = 64        # src/xgraph/oracle.py:172-175

# slot memory (int32 words per slot; xgraph_b200/csrc/core.cuh, MemoryField)
_MEM_REACHED, _MEM_FRONTIER = 1, 2
_MEM_PENDING_LO, _MEM_PENDING_HI, _MEM_PENDING_COUNT = 4, 5, 6
_MEM_REACHED_ROWS = 8 + 3 * MAX_REACHED
_MEM_FRONTIER_ENT = _MEM_REACHED_ROWS + MAX_REACHED
_MEM_FRONTIER_RANK = _MEM_FRONTIER_ENT + MAX_REACHED
_MEM_PENDING_RANK = _MEM_FRONTIER_RANK + MAX_REACHED
_MEM_PENDING_FIRST = _MEM_PENDING_RANK + MAX_REACHED

_PHASE_ERROR = 3
_ENTITY_SPAN, _PATH_SPAN = 2, 4

_NOT_SERVED = {"observe_required": False, "observe_no_loop": False, "observe_defer": 0,
               "menu_close_next": False}

# (opening, closing) quotation marks strip_quotes removes around a written start
# (src/xgraph/programs.py:238-248)
QUOTE_PAIRS = (('"', '"'), ("'", "'"), ("\u201c", "\u201d"), ("\u2018", "\u2019"), ("\u201e", "\u201c"),
               ("\u00ab", "\u00bb"))


def strip_quotes(text: str) -> str:
    """The text without the paired quotation marks that wrap all of it, repeatedly, and the
    spaces inside them; unchanged where nothing would be left."""
    while len(text) > 2 and (text[0], text[-1]) in QUOTE_PAIRS and text[1:-1].strip():
        text = text[1:-1].strip()
    return text


@dataclass(frozen=True)
class MatchedPath:
    """A written path as path mode's committed paths resolve it (the reference's
    MatchedPath, src/xgraph/programs.py:328-366): the entities reached, best-connected
    first (empty where the engine would not have let the path be written), the answer
    delivered, and the plan (the start and relation labels path mode would write), None
    where the path reaches nothing or names no relation."""

    reached: tuple[str, ...]
    answer: str | None
    plan: tuple[str, ...] | None = None
    stripped: bool = False

    @property
    def recorded_plan(self) -> dict | None:
        if self.plan is None:
            return None
        return {"start": self.plan[0], "relations": list(self.plan[1:])}


class MatchedExecutor:
    """Parse-then-execute matched to path mode with committed paths (the reference's
    MatchedExecutor, src/xgraph/programs.py:368-440: same constructor keywords, `execute`
    signature and results), executed on the GPU by the engine; `execute_many` runs a whole
    batch of paths in two kernel launches.  `max_paths` is the batch the engine is sized
    for (larger batches run in pieces)."""

    def __init__(self, index, tokenizer, *, versions=None, start_rank: str = "degree",
                 unquoted_starts: bool = False, committed_paths: bool = True, max_paths: int = 256,
                 strip_quotes: bool = False, _runner=None, **others) -> None:
        from .engine import Engine
        from .index import IndexMismatch

        if index.tokenizer_fingerprint != tokenizer.fingerprint:
            raise IndexMismatch("the KG index was built for another tokenizer")
        for name, value in others.items():
            if name not in _NOT_SERVED:
                raise TypeError(f"MatchedExecutor() got an unexpected keyword argument {name!r}")
            if value != _NOT_SERVED[name]:
                raise ValueError(f"the {name} setting is not served by this executor")
        if max_paths < 1:
            raise ValueError(f"max_paths must be at least 1, got {max_paths}")
        self._index, self._tokenizer, self._versions = index, tokenizer, versions
        self._syntax = index.span_syntax
        # the engine-shaped runner that executes the batches (tests drive the host seam of the
        # same row logic through it); by default the CUDA engine
        self._runner = _runner if _runner is not None else _EngineRunner(Engine(
            index, tokenizer, self._syntax, max_paths, paths=True, committed_paths=committed_paths,
            versions=versions, start_rank=start_rank, unquoted_starts=unquoted_starts))
        self._sitelinks = index.sitelinks if start_rank == "sitelinks" else None
        self._unquoted, self._committed, self._strip = unquoted_starts, committed_paths, strip_quotes
        self._pieces: dict[str, list[int]] = {}
        self._first: np.ndarray | None = None

    # -- host pieces ---------------------------------------------------------------------

    def _encode(self, text: str) -> list[int]:
        tokens = self._pieces.get(text)
        if tokens is None:
            tokens = self._pieces[text] = list(self._tokenizer.encode(text))
        return tokens

    def _label(self, text: str) -> list[int] | None:
        """The tokens of a label as written (the label prefix, then the text), None for a
        blank label (one the reference's executor reads as naming nothing)."""
        if not text.strip():
            return None
        return self._encode(self._syntax.label_prefix + text) or None

    def _stream(self, start: str, relations: Sequence[str], label=None) -> tuple[list[int], int] | None:
        """The span's tokens and how many come before the closer, or None where a label
        is blank (`label`: the start's tokens, in place of the start text's)."""
        tokens = list(self._encode(self._syntax.opener))
        label = self._label(start) if label is None else label
        if label is None:
            return None
        tokens += label
        for written in relations:
            label = self._label(written)
            if label is None:
                return None
            tokens += self._encode(self._syntax.separator) + label
        return tokens + self._encode(self._syntax.closer), len(tokens)

    def _order(self, view, pairs: Iterable[tuple[int, int]], sitelinks=False) -> list[int]:
        """The entities of these (entity, label row) pairs in best-connected order (by the
        executor's start rank, or by the given sitelink counts; None: by degree)."""
        if sitelinks is False:
            sitelinks = self._sitelinks

        def key(pair: tuple[int, int]) -> tuple[int, int, int]:
            entity, row = pair
            linked = int(sitelinks[entity]) if sitelinks is not None else 0
            return (-linked, -len(view.edges_at(entity)[0]), row)

        return list(dict.fromkeys(entity for entity, _ in sorted(pairs, key=key)))

    def _first_rows(self) -> np.ndarray:
        """Each entity's first label row."""
        if self._first is None:
            owners = np.asarray(self._index.labels.owners, dtype=np.int64)
            first = np.full(len(self._index.labels.owner_ids), np.iinfo(np.int64).max, dtype=np.int64)
            np.minimum.at(first, owners, np.arange(len(owners), dtype=np.int64))
            self._first = first
        return self._first

    def _last_hop(self, view, memory: np.ndarray, lo: int, hi: int) -> list[tuple[int, int]]:
        """(entity, start rank) of the path's last frontier computed from the frontier before
        it and the last relation's label rows [lo, hi) -- only for a path of the full eight
        relations, where the engine's separator test (and so its cached next frontier) does
        not run: the objects under every relation the label names, each with the least rank
        it is reached from, kept to 64 by (rank, first label row)."""
        index = self._index
        follow = sorted({int(index.relations.owners[r]) for r in range(lo, hi)})
        owners, first = index.labels.owners, self._first_rows()
        reached: dict[int, int] = {}
        count = int(memory[_MEM_FRONTIER])
        for k in range(min(count, MAX_REACHED)):
            entity, rank = int(memory[_MEM_FRONTIER_ENT + k]), int(memory[_MEM_FRONTIER_RANK + k])
            relation_of, object_of = view.edges_at(entity)
            for row in np.asarray(object_of)[np.isin(relation_of, follow)].tolist():
                item = int(owners[row])
                reached[item] = min(reached.get(item, rank), rank)
        kept = sorted(reached, key=lambda e: (reached[e], int(first[e])))[:MAX_REACHED]
        return [(e, reached[e]) for e in kept]

    # -- execution -----------------------------------------------------------------------

    def _written_rows(self, start: str, labels=None) -> list[int]:
        """The label rows (of the entity labels, or of `labels`) written exactly as `start`
        (the reference's `_rows`)."""
        tokens = self._label(start)
        if tokens is None:
            return []
        labels = self._index.labels if labels is None else labels
        lo, hi = labels.prefix_range(tokens)
        offsets = np.asarray(labels.offsets)
        return [r for r in range(lo, hi) if int(offsets[r + 1] - offsets[r]) == len(tokens)]

    def _bound_rows(self, anchor: Sequence[str]) -> list[int]:
        """The first 64 label rows (row order) of the anchor's entities."""
        owners = np.asarray(self._index.labels.owners)
        at = {e: n for n, e in enumerate(self._index.labels.owner_ids)}
        entities = [at[e] for e in anchor if e in at]
        rows = np.flatnonzero(np.isin(owners, entities))[:MAX_REACHED].tolist()
        if not rows:
            raise ValueError(f"anchor has no writable label rows: {list(anchor)!r}")
        return rows

    def execute(self, start: str, relations: list[str], anchor: list[str] | None = None,
                version: str | None = None, repair: bool = False) -> MatchedPath:
        """The path from the start label along the relation labels (see the class).  With
        repair, a relation label that names no relation of its hop's frontier is replaced
        by the label or alias of the frontier's relation most like it (see _repair)."""
        return self.execute_many([(start, relations, version, anchor)], repair=repair)[0]

    def execute_many(self, paths: Iterable[tuple], *, repair: bool = False) -> list[MatchedPath]:
        """Each (start, relations, version) or (start, relations, version, anchor) path
        executed, in order.  An anchored path starts from the anchor's entities its start
        label names; one whose label names none of them (the reference then starts from every
        anchor entity, which no written span can express) raises ValueError."""
        originals = list(paths)
        paths = [(self._read(p[0], p[3] if len(p) > 3 else None, p[2]), *p[1:]) for p in originals]
        stripped = [p[0] != q[0] for p, q in zip(paths, originals, strict=True)]
        if repair:
            paths = [(p[0], self._repaired(p[0], list(p[1])[:MAX_PATH_RELATIONS], p[2], p[3] if len(p) > 3 else None),
                      *p[2:]) for p in paths]
        jobs = self._jobs(paths)
        out: list[MatchedPath] = []
        size = self._runner.max_sequences
        for at in range(0, len(jobs), size):
            out += self._batch(jobs[at: at + size])
        return [replace(path, stripped=True) if flag else path for path, flag in zip(out, stripped, strict=True)]

    def _read(self, start: str, anchor, version) -> str:
        """The start as read (src/xgraph/programs.py:887-895): with strip_quotes, a start
        that names nothing to start from is read without the quotation marks wrapping it,
        where that names something."""
        if not self._strip:
            return start
        view = self._runner.view(version)
        if self._names_start(view, start, anchor):
            return start
        unquoted = strip_quotes(start)
        return unquoted if unquoted != start and self._names_start(view, unquoted, anchor) else start

    def _names_start(self, view, start: str, anchor) -> bool:
        """Whether the start label names an entity with triples the path may start from
        (the anchor's among its rows, anchored; none for a quoted start under unquoted
        starts)."""
        owners = np.asarray(self._index.labels.owners)
        written = self._written_rows(start)
        if anchor is not None:
            bound = set(self._bound_rows(anchor))
            written = [r for r in written if r in bound]
        elif self._unquoted and self._syntax.quoted((self._syntax.label_prefix + start).encode("utf-8")):
            written = []
        return any(len(view.edges_at(int(owners[r]))[0]) for r in written)

    def _repaired(self, start: str, relations: list[str], version, anchor) -> list[str]:
        """The relation labels with each hop's unknown relation repaired (src/xgraph/
        programs.py:1094-1128): where a label names no relation of its hop's frontier (the
        engine's, one slot per prefix), the frontier's relation whose label or alias is
        most like it (similarity at least 0.6) is followed instead, written as its most
        similar label or alias that names no other relation of the frontier.  A relation
        with no such label cannot be written as a span: that repair raises ValueError."""
        index = self._index
        view = self._runner.view(version)
        labels = list(relations)
        for hop in range(len(labels)):
            frontier = self.frontiers([(start, labels[:hop], version, anchor)])[0]
            if not frontier:
                break
            have: set[int] = set()
            for entity, _ in frontier:
                have.update(int(r) for r in np.asarray(view.edges_at(entity)[0]).tolist())
            follow = {int(index.relations.owners[r]) for r in self._written_rows(labels[hop], index.relations)}
            if follow & have:
                continue
            best, label = self._repair(have, labels[hop])
            if best is None:
                break  # the hop leads nowhere: the path reaches nothing, repaired or not
            if label is None:
                raise ValueError(f"the repaired relation of {labels[hop]!r} has no label of its own on its "
                                 "frontier; such a path cannot be written as a span")
            labels[hop] = label
        return labels

    def _repair(self, have: set[int], written: str) -> tuple[int | None, str | None]:
        """The frontier relation (of `have`) with the label or alias most like the written
        one, at least 0.6 alike (the larger of difflib's ratio and the word sets' Jaccard
        overlap, on NFC-normalized casefolded text), the last of equal scores in relation
        order; and its most similar label or alias that names no other relation of `have`."""
        from difflib import SequenceMatcher
        from unicodedata import normalize

        def norm(text: str) -> str:
            return normalize("NFC", text).casefold().strip()

        def similarity(a: str, b: str) -> float:
            words_a, words_b = set(a.split()), set(b.split())
            overlap = len(words_a & words_b) / len(words_a | words_b) if words_a | words_b else 0.0
            return max(SequenceMatcher(None, a, b).ratio(), overlap)

        names = self._relation_names()
        best, score = None, 0.6
        for relation in sorted(have):
            for name in names.get(relation, ()):
                ratio = similarity(norm(name), norm(written))
                if ratio >= score:
                    best, score = relation, ratio
        if best is None:
            return None, None
        index = self._index
        for name in sorted(names[best], key=lambda n: -similarity(norm(n), norm(written))):
            owners = {int(index.relations.owners[r]) for r in self._written_rows(name, index.relations)}
            if owners & have == {best}:
                return best, name
        return best, None

    def _relation_names(self) -> dict[int, list[str]]:
        """Each relation's labels and aliases as its index rows write them, in row order."""
        if getattr(self, "_names", None) is None:
            index, prefix = self._index.relations, self._syntax.label_prefix
            self._names: dict[int, list[str]] = {}
            for row in range(index.num_rows):
                text = b"".join(self._tokenizer.token_bytes(t) for t in index.row_tokens(row))
                self._names.setdefault(int(index.owners[row]), []).append(
                    text.decode("utf-8", errors="replace").removeprefix(prefix))
        return self._names

    def _jobs(self, paths) -> list[tuple]:
        """(start, relations capped at 8, version, anchor, start tokens, fallback) of each
        path, checked before any launch: an unknown version or an anchor without label rows
        raises.  An anchored start naming none of the anchor's entities falls back, as the
        reference's executor does, to every anchor entity (src/xgraph/programs.py:832-836):
        its span is written with a label that names exactly the anchor's entities among its
        bound rows (the start tokens; the written start then plans nothing); where no label
        does (anchor entities without a shared label), that fallback raises."""
        jobs = []
        for path in paths:
            start, relations, version = path[0], list(path[1])[:MAX_PATH_RELATIONS], path[2]
            anchor = path[3] if len(path) > 3 else None
            self._runner.view(version)
            tokens, fallback = None, False
            if anchor is not None:
                bound = self._bound_rows(anchor)
                if not set(self._written_rows(start)) & set(bound):
                    tokens, fallback = self._covering_label(bound), True
                    if tokens is None:
                        raise ValueError(f"the anchored start {start!r} names none of the anchor's entities "
                                         f"{list(anchor)!r}, and no one label names them all; that fallback "
                                         "is not served")
                anchor = list(anchor)
            jobs.append((start, relations, version, anchor, tokens, fallback))
        return jobs

    def _covering_label(self, bound: list[int]) -> list[int] | None:
        """The tokens of a label whose rows among the bound rows name every entity they name,
        or None."""
        labels = self._index.labels
        owners = np.asarray(labels.owners)
        every = {int(owners[r]) for r in bound}
        named: dict[tuple[int, ...], set[int]] = {}
        for row in bound:
            named.setdefault(tuple(labels.row_tokens(row)), set()).add(int(owners[row]))
        for tokens, entities in named.items():  # (bound rows are in row order: the first such label)
            if entities == every:
                return list(tokens)
        return None

    # -- the live frontier (src/xgraph/programs.py:598-812) ------------------------------

    def named(self, label: str) -> set[str]:
        """The entities a label written exactly as this text names."""
        ids, owners = self._index.labels.owner_ids, self._index.labels.owners
        return {ids[int(owners[row])] for row in self._written_rows(label)}

    def starts(self, start: str, anchor: list[str] | None = None, version: str | None = None) -> tuple[str, ...]:
        """The entities a path from this start starts from, best-connected first: those the
        label names (the anchor's, anchored) that have triples, the first 64 (the start as
        written: no quotation marks are stripped here)."""
        ids = self._index.labels.owner_ids
        return tuple(ids[e] for e, _ in self.frontiers([(start, [], version, anchor)])[0])

    def frontier(self, start: str, relations: list[str], anchor: list[str] | None = None,
                 version: str | None = None) -> tuple[str, ...]:
        """The capped live frontier after the relations (every start sense that survives,
        by start rank and first label row), or the starts for no relation."""
        ids = self._index.labels.owner_ids
        start = self._read(start, anchor, version)
        return tuple(ids[e] for e, _ in self.frontiers([(start, relations, version, anchor)])[0])

    def frontier_relations(self, start: str, relations: list[str], anchor: list[str] | None = None,
                           version: str | None = None) -> list[tuple[str, int]]:
        """The relations path mode offers after the path so far: every relation of its whole
        frontier, as (relation id, the frontier's edges with it), most edges first, then
        index order; empty where the path has as many relations as a path may name."""
        if len(relations) >= MAX_PATH_RELATIONS:
            if anchor is not None:
                self._bound_rows(anchor)
            return []
        view = self._runner.view(version)
        start = self._read(start, anchor, version)
        counts: dict[int, int] = {}
        for entity, _ in self.frontiers([(start, relations, version, anchor)])[0]:
            found, times = np.unique(np.asarray(view.edges_at(entity)[0]), return_counts=True)
            for relation, n in zip(found.tolist(), times.tolist(), strict=True):
                counts[relation] = counts.get(relation, 0) + n
        ids = self._index.relations.owner_ids
        return [(ids[r], counts[r]) for r in sorted(counts, key=lambda r: (-counts[r], r))]

    def frontier_labels(self, start: str, relations: list[str], anchor: list[str] | None = None,
                        version: str | None = None) -> list[str]:
        """The writable relation labels and aliases of the whole frontier, sorted."""
        have = {relation for relation, _ in self.frontier_relations(start, relations, anchor, version)}
        return self.relation_labels(have) if have else []

    def relation_labels(self, relations: set[str] | None = None) -> list[str]:
        """The writable relation vocabulary (the index's relation rows as written), or the
        named relations' labels only, sorted."""
        index, prefix = self._index.relations, self._syntax.label_prefix
        ids = index.owner_ids
        names = set()
        for row in range(index.num_rows):
            if relations is None or ids[int(index.owners[row])] in relations:
                text = b"".join(self._tokenizer.token_bytes(t) for t in index.row_tokens(row))
                names.add(text.decode("utf-8", errors="replace").removeprefix(prefix))
        return sorted(names)

    def derivations(self, start: str, relations: list[str], anchor: list[str] | None = None,
                    version: str | None = None, rank: str | None = None) -> tuple[tuple[str, int], ...]:
        """The entities the path resolves to (MatchedPath.reached), each with its number of
        derivations: the distinct relation paths from the start it resolves from, one
        relation and one entity of each hop's live frontier per hop (src/xgraph/programs.py:
        606-662), best-connected first under `rank` (by default the executor's start rank).
        The engine gives every hop's frontier (one slot per prefix of the path, one launch);
        the paths are counted on the host.  Empty where the path is empty or names no
        relation."""
        from .index import check_start_rank

        relations = list(relations)[:MAX_PATH_RELATIONS]
        if not relations:
            if anchor is not None:
                self._bound_rows(anchor)
            return ()
        start = self._read(start, anchor, version)
        jobs = [(start, relations[:k], version, anchor) for k in range(len(relations) + 1)]
        starts, *hops = self.frontiers(jobs)
        if not hops[-1]:
            return ()
        index, view = self._index, self._runner.view(version)
        owners = np.asarray(index.labels.owners)
        best = min(r for _, r in hops[-1])
        counts = {starts[best][0]: 1}
        for written, kept in zip(relations, hops, strict=True):
            follow = sorted({int(index.relations.owners[r]) for r in self._written_rows(written, index.relations)})
            members = {e for e, _ in kept}
            reached: dict[int, int] = {}
            for entity, n in counts.items():
                relation_of, object_of = view.edges_at(entity)
                chosen = np.isin(relation_of, follow)
                steps = {(int(r), int(owners[row])) for r, row in zip(np.asarray(relation_of)[chosen],
                                                                       np.asarray(object_of)[chosen], strict=True)}
                for _, item in steps:
                    if item in members:
                        reached[item] = reached.get(item, 0) + n
            counts = reached
        sitelinks = False
        if rank is not None:
            sitelinks = index.sitelinks if check_start_rank(rank, index) == "sitelinks" else None
        first = self._first_rows()
        final = [e for e, r in hops[-1] if r == best]
        ordered = self._order(view, [(e, int(first[e])) for e in final], sitelinks)
        ids = index.labels.owner_ids
        return tuple((ids[e], counts.get(e, 0)) for e in ordered)

    def execute_set(self, start: str, relations: list[str], anchor: list[str] | None = None,
                    version: str | None = None, *, witnesses: bool = False) -> dict:
        """Complete answer support after commitment, with each cap the path met
        (src/xgraph/programs.py:486-560): `reached`, the entities the capped walk's answer
        binds (the best start's final entities' label rows, the first 64, best-connected);
        `uncapped_reached`, the same walk with no start, frontier or label-row cap (a
        sensitivity of the fixed plan, computed on the host as the reference does); and
        `cap_events`, each cap met (path relations, anchor label rows, starts, a hop's
        frontier, answer label rows) with the count before it; with witnesses (an index
        with sitelink counts), `witnesses`: for each reached entity one start-to-endpoint
        entity chain through the capped walk, chains ranked step by step by most sitelinks,
        then numeric entity id.  The capped walk's frontiers come from the engine (one slot
        per prefix of the path); the counts before each cap and the chains are taken on the
        host."""
        if witnesses and self._index.sitelinks is None:
            raise ValueError("endpoint witnesses require an index with sitelink counts")
        view = self._runner.view(version)
        start = self._read(start, anchor, version)
        index = self._index
        owners = np.asarray(index.labels.owners)
        ids = index.labels.owner_ids
        events: list[dict] = []
        if len(relations) > MAX_PATH_RELATIONS:
            events.append({"stage": "path_relations", "before": len(relations), "kept": MAX_PATH_RELATIONS})
        relations = list(relations)[:MAX_PATH_RELATIONS]
        if anchor is not None:
            at = {e: n for n, e in enumerate(ids)}
            count = int(np.count_nonzero(np.isin(owners, sorted({at[e] for e in anchor if e in at}))))
            if not count:
                raise ValueError(f"anchor has no writable label rows: {anchor!r}")
            if count > MAX_REACHED:
                events.append({"stage": "anchor_label_rows", "before": count, "kept": MAX_REACHED})
        result = {"reached": [], "uncapped_reached": [], "cap_events": events}
        if witnesses:
            result["witnesses"] = {}
        if not relations:
            return result
        # the capped walk: the engine's starts and hop frontiers; the host counts what each cap cut
        starts, *hops = self.frontiers([(start, relations[:k], version, anchor) for k in range(len(relations) + 1)])
        written = self._start_rows(start, anchor, uncapped=False)
        with_triples = {int(owners[r]) for r in written if len(view.edges_at(int(owners[r]))[0])}
        if len(with_triples) > MAX_REACHED:
            events.append({"stage": "starts", "before": len(with_triples), "kept": MAX_REACHED})
        previous = starts
        for hop, (label, kept) in enumerate(zip(relations, hops, strict=True), start=1):
            if not previous:
                break
            reached = self._step(view, {e for e, _ in previous}, label)
            if len(reached) > MAX_REACHED:
                events.append({"stage": "frontier", "hop": hop, "before": len(reached), "kept": MAX_REACHED})
            previous = kept
        if hops[-1]:
            rows = self._final_rows(hops[-1])
            if len(rows) > MAX_REACHED:
                events.append({"stage": "answer_label_rows", "before": len(rows), "kept": MAX_REACHED})
            ordered = self._order(view, [(int(owners[r]), r) for r in rows[:MAX_REACHED]])
            result["reached"] = [ids[e] for e in ordered]
            if witnesses:
                chains = self._witnesses(view, starts, relations, hops)
                result["witnesses"] = {ids[e]: [ids[p] for p in chains[e]] for e in ordered}
        # the uncapped walk (host): every start, every entity each hop reaches
        ranks = self._uncapped_starts(view, start, anchor)
        for label in relations:
            if not ranks:
                break
            reached: dict[int, int] = {}
            for entity, rank in ranks.items():
                for item in self._step(view, {entity}, label):
                    reached[item] = min(reached.get(item, rank), rank)
            ranks = reached
        if ranks:
            rows = self._final_rows(list(ranks.items()))
            result["uncapped_reached"] = [ids[e] for e in self._order(view, [(int(owners[r]), r) for r in rows])]
        return result

    def _witnesses(self, view, starts, relations, hops) -> dict[int, tuple[int, ...]]:
        """One chain per entity of the capped walk's last frontier with the best rank,
        restricted to the walk's own frontiers (src/xgraph/programs.py:562-595): from the
        starts of the best rank (every start, union paths), each hop extends the chains in
        order of (most sitelinks, numeric id) per step, and an entity keeps the first chain
        that reaches it."""
        index = self._index
        ids, owners, sitelinks = index.labels.owner_ids, np.asarray(index.labels.owners), index.sitelinks
        best = min(r for _, r in hops[-1])
        paths = {e: (e,) for e, rank in starts if not self._committed or rank == best}

        def key(entity):
            return tuple((-int(sitelinks[e]), int(ids[e][1:])) for e in paths[entity])

        for label, kept in zip(relations, hops, strict=True):
            follow = sorted({int(index.relations.owners[r]) for r in self._written_rows(label, index.relations)})
            ranks = dict(kept)
            reached: dict[int, tuple[int, ...]] = {}
            for entity in sorted(paths, key=key):
                relation_of, object_of = view.edges_at(entity)
                for row in np.asarray(object_of)[np.isin(relation_of, follow)].tolist():
                    item = int(owners[row])
                    if ranks.get(item) == best:
                        reached.setdefault(item, (*paths[entity], item))
            paths = reached
        return paths

    def _start_rows(self, start: str, anchor, *, uncapped: bool) -> list[int]:
        """The label rows a path's start may name (src/xgraph/programs.py:832-860): the
        anchor's (its first 64 rows, or all of them uncapped) among those written as the
        start, or all of them when the start names none; unanchored, those written as the
        start (none for a quoted start under unquoted starts)."""
        written = self._written_rows(start)
        if anchor is None:
            if self._unquoted and self._syntax.quoted((self._syntax.label_prefix + start).encode("utf-8")):
                return []
            return written
        at = {e: n for n, e in enumerate(self._index.labels.owner_ids)}
        bound = np.flatnonzero(np.isin(np.asarray(self._index.labels.owners),
                                       sorted({at[e] for e in anchor if e in at}))).tolist()
        if not uncapped:
            bound = bound[:MAX_REACHED]
        named = [r for r in bound if r in set(written)]
        return named or bound

    def _uncapped_starts(self, view, start: str, anchor) -> dict[int, int]:
        """Every start with triples and its rank (0 for union paths), uncapped."""
        owners = np.asarray(self._index.labels.owners)
        rows = self._start_rows(start, anchor, uncapped=True)
        pairs = [(int(owners[r]), r) for r in rows if len(view.edges_at(int(owners[r]))[0])]
        ordered = self._order(view, pairs)
        if not self._committed:
            first = self._first_rows()
            ordered.sort(key=lambda e: int(first[e]))
        return {e: (rank if self._committed else 0) for rank, e in enumerate(ordered)}

    def _step(self, view, entities: set[int], label: str) -> set[int]:
        """The entities reached from these under every relation the label names."""
        index = self._index
        owners = np.asarray(index.labels.owners)
        follow = sorted({int(index.relations.owners[r]) for r in self._written_rows(label, index.relations)})
        out: set[int] = set()
        for entity in entities:
            relation_of, object_of = view.edges_at(entity)
            out.update(int(owners[row]) for row in np.asarray(object_of)[np.isin(relation_of, follow)].tolist())
        return out

    def _final_rows(self, frontier) -> list[int]:
        """The label rows, sorted, of the frontier's entities of the least start rank."""
        best = min(rank for _, rank in frontier)
        rows = np.asarray(self._index.labels.owners)
        final = sorted({e for e, rank in frontier if rank == best})
        return np.flatnonzero(np.isin(rows, final)).tolist()

    def frontiers(self, paths: Iterable[tuple]) -> list[list[tuple[int, int]]]:
        """Each (start, relations, version[, anchor]) path's live frontier as (entity
        position, start rank) pairs in order, from one engine slot each, a batch in one
        launch: the ranked starts after `⟦ start ·` for no relation, else the frontier the
        last relation reaches (read before the closer); empty where the engine would not
        have let the path be written."""
        jobs = self._jobs(paths)
        out: list[list[tuple[int, int]]] = []
        size = self._runner.max_sequences
        for at in range(0, len(jobs), size):
            out += self._frontier_batch(jobs[at: at + size])
        return out

    def _frontier_batch(self, paths) -> list[list[tuple[int, int]]]:
        size = self._runner.max_sequences
        streams = []
        for start, relations, _, _, start_tokens, _ in paths:
            if relations:
                stream = self._stream(start, relations, start_tokens)
                streams.append(None if stream is None else (stream[0][: stream[1]], stream[1]))
            else:  # the starts: the span up to the separator after its start
                label = self._label(start) if start_tokens is None else start_tokens
                tokens = None if label is None else (self._encode(self._syntax.opener) + label
                                                     + self._encode(self._syntax.separator))
                streams.append(None if tokens is None else (tokens, len(tokens)))
        width = max([len(s[0]) for s in streams if s is not None] + [1])
        history = np.zeros((size, width), dtype=np.int32)
        upto = np.zeros(size, dtype=np.int32)
        for k, stream in enumerate(streams):
            if stream is not None:
                history[k, : len(stream[0])] = stream[0]
                upto[k] = stream[1]
        admissions = [(k, job[2], job[3]) for k, job in enumerate(paths)]
        states, memory, _, _ = self._runner.run(history, upto, upto, admissions)
        owners, first = self._index.labels.owners, self._first_rows()
        out = []
        for k, (_, relations, version, _, _, _) in enumerate(paths):
            if streams[k] is None or int(states["phase"][k]) == _PHASE_ERROR:
                out.append([])
                continue
            row = memory[k]
            if not relations:  # the ranked starts, as next_segment stored them
                count = int(row[_MEM_FRONTIER])
                out.append([(int(row[_MEM_FRONTIER_ENT + i]), int(row[_MEM_FRONTIER_RANK + i])) for i in range(count)])
                continue
            lo, hi = int(states["lo"][k]), int(states["ex_hi"][k])
            if int(row[_MEM_PENDING_LO]) == lo and int(row[_MEM_PENDING_HI]) == hi:
                pairs = [(int(owners[int(row[_MEM_PENDING_FIRST + i])]), int(row[_MEM_PENDING_RANK + i]))
                         for i in range(int(row[_MEM_PENDING_COUNT]))]
            else:  # the eighth relation: no separator test ran
                pairs = self._last_hop(self._runner.view(version), row, lo, hi)
            least: dict[int, int] = {}
            for entity, rank in pairs:  # an entity may be listed once per rank it is reached with
                least[entity] = min(least.get(entity, rank), rank)
            out.append(sorted(least.items(), key=lambda p: (p[1], int(first[p[0]]))))
        return out

    def _batch(self, paths) -> list[MatchedPath]:
        index = self._index
        n, size = len(paths), self._runner.max_sequences
        streams = [self._stream(start, relations, tokens) for start, relations, _, _, tokens, _ in paths]
        width = max([len(s[0]) for s in streams if s is not None] + [1])
        history = np.zeros((size, width), dtype=np.int32)
        before = np.zeros(size, dtype=np.int32)
        total = np.zeros(size, dtype=np.int32)
        for k, stream in enumerate(streams):
            if stream is not None:
                history[k, : len(stream[0])] = stream[0]
                before[k], total[k] = stream[1], len(stream[0])
        admissions = [(k, job[2], job[3]) for k, job in enumerate(paths)]
        states_a, memory_a, states_b, memory_b = self._runner.run(history, before, total, admissions)
        owners, ids = index.labels.owners, index.labels.owner_ids

        results = []
        for k, (start, relations, version, anchor, _, fallback) in enumerate(paths):
            empty = MatchedPath((), None, None)
            if streams[k] is None or int(states_b["phase"][k]) == _PHASE_ERROR:
                results.append(empty)
                continue
            view = self._runner.view(version)
            kind = int(states_b["last_kind"][k])
            if not relations:  # an entity span: every entity its label names (the anchor's, anchored)
                if kind != _ENTITY_SPAN:
                    results.append(empty)
                    continue
                lo, hi = int(states_b["last_lo"][k]), int(states_b["last_hi"][k])
                rows = (range(lo, hi) if anchor is None else self._bound_rows(anchor) if fallback
                        else sorted(set(self._written_rows(start)) & set(self._bound_rows(anchor))))
                starts = self._order(view, [(int(owners[r]), r) for r in rows])
                results.append(MatchedPath(tuple(ids[e] for e in starts), ids[starts[0]] if starts else None, None))
                continue
            if kind != _PATH_SPAN:
                results.append(empty)
                continue
            memory = memory_a[k]
            lo, hi = int(states_a["lo"][k]), int(states_a["ex_hi"][k])
            if int(memory[_MEM_PENDING_LO]) == lo and int(memory[_MEM_PENDING_HI]) == hi:
                count = int(memory[_MEM_PENDING_COUNT])
                frontier = [(int(owners[int(memory[_MEM_PENDING_FIRST + i])]), int(memory[_MEM_PENDING_RANK + i]))
                            for i in range(count)]
            else:  # the eighth relation: no separator test ran
                frontier = self._last_hop(view, memory, lo, hi)
            if not frontier:
                results.append(empty)
                continue
            best = min(rank for _, rank in frontier)
            final = list(dict.fromkeys(e for e, rank in frontier if rank == best))
            first = self._first_rows()
            entities = self._order(view, [(e, int(first[e])) for e in final])
            rows = memory_b[k][_MEM_REACHED_ROWS: _MEM_REACHED_ROWS + int(memory_b[k][_MEM_REACHED])].tolist()
            answer = self._order(view, [(int(owners[r]), r) for r in rows])
            # a fallback start plans nothing: the written start names no entity it starts from
            results.append(MatchedPath(tuple(ids[e] for e in entities), ids[answer[0]] if answer else None,
                                       None if fallback else (start, *relations)))
        return results


class _EngineRunner:
    """The CUDA engine as the executor drives it: a batch of paths, one slot each (admitted
    with its KG version and anchors in one launch), synced once up to each path's last
    relation label and once through its closer; the slots' states and memory read back
    after each."""

    def __init__(self, engine) -> None:
        self._engine = engine

    @property
    def max_sequences(self) -> int:
        return self._engine.max_sequences

    def view(self, version):
        return self._engine.view(version)

    def run(self, history: np.ndarray, before: np.ndarray, total: np.ndarray, admissions):
        import torch

        from .engine import Admission

        engine = self._engine
        n, size = len(admissions), engine.max_sequences
        device = torch.device("cuda", torch.cuda.current_device())
        engine.reset()
        engine.admit([Admission(k, True, anchors=tuple(anchor or ()), version=version)
                      for k, version, anchor in admissions])
        slots = torch.arange(n, dtype=torch.int32, device=device)
        history_d = torch.from_numpy(history).to(device)
        prompt = torch.zeros(size, dtype=torch.int32, device=device)
        engine.sync(slots, history_d, prompt, torch.from_numpy(before).to(device))
        states_a, memory_a = engine.states_host(n), engine.memory_host(n)
        engine.sync(slots, history_d, prompt, torch.from_numpy(total).to(device))
        return states_a, memory_a, engine.states_host(n), engine.memory_host(n)
