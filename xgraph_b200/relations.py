"""Relation supports of path mode's relation segments (the reference's src/xgraph/relations.py).

"frontier" executes paths over the entity frontier (the default); "vocabulary" admits every
relation in every relation segment; "successor" admits every relation first, then only the
successors of the preceding label's relations: the relations some object of one of its
edges is the subject of, in the slot's KG version.  The weaker two execute nothing and bind
no answer (src/xgraph/oracle.py:67-79).  Successor support reads per-KG tables built here
once per engine, for the base KG and each version built into the engine.
"""

from __future__ import annotations

import numpy as np

RELATIONS = ("frontier", "vocabulary", "successor")
"""Mode names, in the order of their codes (XgOptions.relations)."""

_CHUNK = 1 << 20  # edges joined per round, whatever the KG size


def check_relations(mode: str, *, paths: bool, stop: str | None, expressions: bool = False) -> None:
    """The reference's checks (src/xgraph/relations.py:24-28), in its words."""
    if mode not in RELATIONS:
        raise ValueError(f"unknown relations mode {mode!r}; expected one of {RELATIONS}")
    if mode != "frontier" and (not paths or expressions or stop):
        raise ValueError("weaker relations need path mode without expressions or STOP")


def _edges(index, versions, name):
    """(subject entity, relation, object label row) of every edge of the KG `name` reads:
    the base adjacency, each edited subject's list replaced by the version's."""
    offsets = np.asarray(index.adjacency_offsets, dtype=np.int64)
    subjects = np.repeat(np.arange(len(offsets) - 1, dtype=np.int64), np.diff(offsets))
    relations = np.asarray(index.edge_relations, dtype=np.int64)
    objects = np.asarray(index.edge_objects, dtype=np.int64)
    if name is None:
        return subjects, relations, objects
    number = versions.number(name)
    first, last = int(versions.offsets[number - 1]), int(versions.offsets[number])
    edited = np.asarray(versions.subjects[first:last], dtype=np.int64)
    adjacency = np.asarray(versions.adjacency[first: last + 1], dtype=np.int64)
    keep = ~np.isin(subjects, edited)
    a, b = int(adjacency[0]), int(adjacency[-1])
    return (np.concatenate([subjects[keep], np.repeat(edited, np.diff(adjacency))]),
            np.concatenate([relations[keep], np.asarray(versions.edge_relations[a:b], dtype=np.int64)]),
            np.concatenate([objects[keep], np.asarray(versions.edge_objects[a:b], dtype=np.int64)]))


def relation_successors(index, versions=None) -> np.ndarray:
    """uint32 [1 + versions, R, ceil(R / 32)]: bit r2 of row r1 of table v is set when some
    object of an r1 edge is the subject of an r2 edge in KG v (0 the base, then the versions
    in order).  Aliases add no witness (an object's label rows name one entity)."""
    relation_count = len(index.relations.owner_ids)
    words = (relation_count + 31) // 32
    names = list(versions.names) if versions is not None else []
    out = np.zeros((1 + len(names), relation_count, max(words, 1)), dtype=np.uint32)[:, :, :words]
    if relation_count == 0:
        return out
    owners = np.asarray(index.labels.owners, dtype=np.int64)
    entities = len(index.labels.owner_ids)
    for v, name in enumerate([None, *names]):
        subjects, relations, objects = _edges(index, versions, name)
        outgoing = np.zeros((entities, words), dtype=np.uint32)  # each entity's relations
        np.bitwise_or.at(outgoing, (subjects, relations >> 5), (np.uint32(1) << (relations & 31).astype(np.uint32)))
        table = out[v]
        for at in range(0, len(relations), _CHUNK):
            rel = relations[at: at + _CHUNK]
            np.bitwise_or.at(table, rel, outgoing[owners[objects[at: at + _CHUNK]]])
    return out
