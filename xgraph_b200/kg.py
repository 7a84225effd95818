"""Source knowledge graph: entities and relations with labels, and ID triples.

Same data model as the reference (src/xgraph/kg.py:12-56): `Entity(id, labels)`,
`Relation(id, labels)`, `KnowledgeGraph(entities, relations, triples)`, with the
canonical label first and aliases after it.  `validate` checks an in-memory graph the
way the reference does for that case (src/xgraph/kg.py:100-139): unique nonempty ids,
string labels, and triples naming declared ids.
"""

from __future__ import annotations

from dataclasses import dataclass


class KGFormatError(ValueError):
    """A knowledge graph is inconsistent, such as a triple naming an unknown entity."""


@dataclass(frozen=True)
class Entity:
    id: str
    labels: tuple[str, ...]


@dataclass(frozen=True)
class Relation:
    id: str
    labels: tuple[str, ...]


@dataclass(frozen=True)
class KnowledgeGraph:
    entities: tuple[Entity, ...]
    relations: tuple[Relation, ...] = ()
    triples: tuple[tuple[str, str, str], ...] = ()


def validate(graph: KnowledgeGraph) -> None:
    if not isinstance(graph, KnowledgeGraph):
        raise KGFormatError("expected a KnowledgeGraph")
    for kind in ("entities", "relations", "triples"):
        if not isinstance(getattr(graph, kind), (tuple, list)):
            raise KGFormatError(f"{kind}: expected a sequence of source records")
    declared: dict[str, dict[str, int]] = {}
    for kind, cls in (("entities", Entity), ("relations", Relation)):
        seen: dict[str, int] = {}
        for row, item in enumerate(getattr(graph, kind), 1):
            if not isinstance(item, cls):
                raise KGFormatError(f"{kind} row {row}: expected {cls.__name__}, got {item!r}")
            where = f"{kind} row {row}, ID {item.id!r}"
            if not isinstance(item.id, str) or not item.id:
                raise KGFormatError(f"{where}: ID must be a nonempty string")
            if item.id in seen:
                raise KGFormatError(f"{where}: duplicate ID (first row {seen[item.id]})")
            seen[item.id] = row
            if not isinstance(item.labels, (tuple, list)):
                raise KGFormatError(f"{where}: labels must be a sequence of strings")
            for at, label in enumerate(item.labels, 1):
                if not isinstance(label, str):
                    raise KGFormatError(f"{where}, label {at}: expected a string, got {label!r}")
        declared[kind] = seen
    for row, triple in enumerate(graph.triples, 1):
        if not isinstance(triple, (tuple, list)) or len(triple) != 3:
            raise KGFormatError(f"triples row {row}: expected three IDs, got {triple!r}")
        for name, kind in zip(triple, ("entities", "relations", "entities"), strict=True):
            if not isinstance(name, str):
                raise KGFormatError(f"triples row {row}, ID {name!r}: ID must be a string")
            if name not in declared[kind]:
                raise KGFormatError(
                    f"triples row {row}, ID {name!r}: triple names unknown {name} in {kind}"
                )
