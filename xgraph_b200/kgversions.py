"""KG versions: named edit sets over one KG index, chosen per request slot.

Semantics follow the reference (src/xgraph/kgversions.py:203-303): an edit
``(subject, relation, object)`` replaces every object of its (subject, relation)
pair; ``None`` as the object deletes the pair.  An edit whose subject has no label row
or whose relation has no relation row changes nothing; an edit whose object has no
label row still removes the pair's old objects.  Each edited subject gets its whole
versioned edge list in the base adjacency's layout (sorted by relation, then object
row), so a device reader swaps one subject's CSR slice for another and nothing else:
version k (1-based; 0 is the base) owns ``subjects[offsets[k-1]:offsets[k]]``
(sorted) and subject i's edges are ``edge_*[adjacency[i]:adjacency[i+1]]``.
"""

from __future__ import annotations

import json
from collections.abc import Iterable, Mapping
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .index import IndexMismatch, KGIndex

Edit = tuple[str, str, "str | None"]


@dataclass(frozen=True)
class VersionStats:
    name: str
    edits: int
    pairs: int
    unwritable_edits: int
    subjects: int
    edges: int


@dataclass(frozen=True)
class KGVersions:
    names: tuple[str, ...]
    stats: tuple[VersionStats, ...]
    offsets: np.ndarray  # int64 [versions + 1]
    subjects: np.ndarray  # int32
    adjacency: np.ndarray  # int64 [len(subjects) + 1]
    edge_relations: np.ndarray  # int32
    edge_objects: np.ndarray  # int32
    base_fingerprint: str

    def number(self, name: str | None) -> int:
        if name is None:
            return 0
        if name not in self.names:
            raise ValueError(f"no KG version {name!r}; the registered ones are {list(self.names)}")
        return self.names.index(name) + 1

    def matches(self, index: KGIndex) -> bool:
        return self.base_fingerprint == index.base_fingerprint

    def check_base(self, index: KGIndex) -> None:
        if not self.matches(index):
            raise IndexMismatch(
                "the KG versions were built for another KG index: base fingerprint "
                f"{self.base_fingerprint} does not match {index.base_fingerprint}"
            )

    def view(self, index: KGIndex, name: str | None):
        number = self.number(name)
        self.check_base(index)
        return index if number == 0 else VersionView(index, self, number)


class VersionView:
    """The index as a slot reading one version sees it: `relations_of`, `object_rows`
    and `edges_at` read the version's edge list for edited subjects."""

    def __init__(self, index: KGIndex, versions: KGVersions, number: int) -> None:
        versions.check_base(index)
        self.labels, self.relations = index.labels, index.relations
        self._index, self._versions = index, versions
        self._first = int(versions.offsets[number - 1])
        self._subjects = versions.subjects[self._first: int(versions.offsets[number])]

    def edges_at(self, entity: int) -> tuple[np.ndarray, np.ndarray]:
        at = int(np.searchsorted(self._subjects, entity))
        if at < len(self._subjects) and int(self._subjects[at]) == entity:
            v = self._versions
            a, b = int(v.adjacency[self._first + at]), int(v.adjacency[self._first + at + 1])
            return v.edge_relations[a:b], v.edge_objects[a:b]
        return self._index.edges_at(entity)

    def relations_of(self, subject: str) -> list[str]:
        relations, _ = self.edges_at(self._index._position("_entity_at", subject, "entity"))
        return [self.relations.owner_ids[r] for r in np.unique(relations)]

    def object_rows(self, subject: str, relation: str, lo: int = 0, hi: int | None = None) -> list[int]:
        relations, objects = self.edges_at(self._index._position("_entity_at", subject, "entity"))
        r = self._index._position("_relation_at", relation, "relation")
        a, b = np.searchsorted(relations, r, "left"), np.searchsorted(relations, r, "right")
        objects = objects[a:b]
        hi = self.labels.num_rows if hi is None else hi
        x, y = np.searchsorted(objects, lo, "left"), np.searchsorted(objects, hi, "left")
        return [int(o) for o in objects[x:y]]


class VersionBuilder:
    """Builds versions of one KG index, one at a time (the lookups from ids to positions and
    label rows are made once): each is the base with every edited (subject, relation) pair's
    objects replaced, written as its edited subjects' whole edge lists."""

    def __init__(self, index: KGIndex) -> None:
        self.index = index
        self.entity_at = {e: n for n, e in enumerate(index.labels.owner_ids)}
        self.relation_at = {r: n for n, r in enumerate(index.relations.owner_ids)}
        owners = np.asarray(index.labels.owners, dtype=np.int64)
        self.row_count = np.bincount(owners, minlength=len(index.labels.owner_ids))
        self.order = np.argsort(owners, kind="stable")
        self.row_start = np.zeros(len(self.row_count) + 1, dtype=np.int64)
        np.cumsum(self.row_count, out=self.row_start[1:])
        self.writable = set(np.unique(np.asarray(index.relations.owners)).tolist())

    def rows_of(self, entity: int | None) -> list[int]:
        if entity is None:
            return []
        return self.order[self.row_start[entity]: self.row_start[entity + 1]].tolist()

    def overlay(self, name: str, edits: Iterable[Edit]):
        """(subjects int32, adjacency int64 [subjects + 1] from 0, edge_relations int32,
        edge_objects int32, VersionStats) of one version."""
        edits = [(str(s), str(r), None if o is None else str(o)) for s, r, o in edits]
        replaced: dict[int, dict[int, set[int]]] = {}
        unwritable = 0
        for s, r, o in edits:
            subject, relation = self.entity_at.get(s), self.relation_at.get(r)
            if subject is None or self.row_count[subject] == 0 or relation not in self.writable:
                unwritable += 1
                continue
            rows = self.rows_of(self.entity_at.get(o)) if o is not None else []
            if o is not None and not rows:
                unwritable += 1
            replaced.setdefault(subject, {}).setdefault(relation, set()).update(rows)
        subjects, adjacency, rel_parts, obj_parts = [], [0], [], []
        for subject in sorted(replaced):
            rels, objs = self.index.edges_at(subject)
            rels = np.asarray(rels, dtype=np.int64)
            objs = np.asarray(objs, dtype=np.int64)
            keep = ~np.isin(rels, list(replaced[subject]))
            added = np.array(
                [(r, row) for r, rows in replaced[subject].items() for row in rows], dtype=np.int64
            ).reshape(-1, 2)
            pairs = np.unique(np.concatenate([np.stack([rels[keep], objs[keep]], axis=1), added]), axis=0)
            rel_parts.append(pairs[:, 0].astype(np.int32))
            obj_parts.append(pairs[:, 1].astype(np.int32))
            subjects.append(subject)
            adjacency.append(adjacency[-1] + len(pairs))
        stats = VersionStats(name=name, edits=len(edits), pairs=sum(len(v) for v in replaced.values()),
                             unwritable_edits=unwritable, subjects=len(replaced), edges=adjacency[-1])
        return (np.array(subjects, dtype=np.int32), np.array(adjacency, dtype=np.int64), _join(rel_parts),
                _join(obj_parts), stats)


def _join(parts: list[np.ndarray]) -> np.ndarray:
    return np.concatenate(parts) if parts else np.zeros(0, dtype=np.int32)


def build_kg_versions(index: KGIndex, versions: Mapping[str, Iterable[Edit]],
                      builder: VersionBuilder | None = None) -> KGVersions:
    for name in versions:
        if not isinstance(name, str) or not name:
            raise ValueError(f"a KG version needs a non-empty name, got {name!r}")
    builder = builder or VersionBuilder(index)
    offsets, subjects, adjacency = [0], [], [np.zeros(1, dtype=np.int64)]
    rel_parts: list[np.ndarray] = []
    obj_parts: list[np.ndarray] = []
    stats = []
    edges = 0
    for name, edits in versions.items():
        subj, adj, rel, obj, stat = builder.overlay(name, edits)
        subjects.append(subj)
        adjacency.append(adj[1:] + edges)
        rel_parts.append(rel)
        obj_parts.append(obj)
        edges += int(adj[-1])
        offsets.append(offsets[-1] + len(subj))
        stats.append(stat)
    return KGVersions(
        names=tuple(versions),
        stats=tuple(stats),
        offsets=np.array(offsets, dtype=np.int64),
        subjects=_join(subjects).astype(np.int32),
        adjacency=np.concatenate(adjacency).astype(np.int64),
        edge_relations=_join(rel_parts),
        edge_objects=_join(obj_parts),
        base_fingerprint=index.base_fingerprint,
    )


VERSIONS_FILE = "kg-versions.json"
VERSIONS_FORMAT = "xgraph-b200-versions-1"


def write_kg_versions(directory, versions: Mapping[str, Iterable[Edit]], index: KGIndex) -> None:
    """Write named edit sets as a version file of this library's format: kg-versions.json in
    `directory`, each version's (subject, relation, object-or-None) id triples in order,
    bound to the index's base fingerprint (the reference's files are out of its scope)."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    listed = [{"name": name, "edits": [[s, r, o] for s, r, o in edits]} for name, edits in versions.items()]
    header = {"format": VERSIONS_FORMAT, "base_fingerprint": index.base_fingerprint, "versions": listed}
    (directory / VERSIONS_FILE).write_text(json.dumps(header) + "\n", encoding="utf-8")


def _version_header(directory) -> dict:
    path = Path(directory) / VERSIONS_FILE
    if not path.is_file():
        raise ValueError(f"{directory} holds no {VERSIONS_FILE}")
    header = json.loads(path.read_text(encoding="utf-8"))
    if header.get("format") != VERSIONS_FORMAT:
        raise ValueError(f"{path} is of format {header.get('format')!r}; this library reads {VERSIONS_FORMAT!r}")
    return header


def version_names(directory) -> list[str]:
    """The names a version file registers, in order (its header alone is read)."""
    return [entry["name"] for entry in _version_header(directory)["versions"]]


def load_kg_versions(directory, index: KGIndex) -> KGVersions:
    """Read a version file written by write_kg_versions and build its versions for `index`
    (which must be the index the file was written for)."""
    header = _version_header(directory)
    if header.get("base_fingerprint") != index.base_fingerprint:
        raise IndexMismatch(f"the KG versions in {directory} were written for another KG index")
    edits = {entry["name"]: [tuple(e) for e in entry["edits"]] for entry in header["versions"]}
    return build_kg_versions(index, edits)
