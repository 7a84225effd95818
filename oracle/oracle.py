"""CPU restatement of the reference Oracle: the specification the engine is checked against.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (xgraph_b200/) imports this module;
only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline arm use it, and only
as the checker or as the timed CPU baseline.

Parity is pinned: tests/test_oracle_golden.py replays the golden walks in tests/golden/
(made by tests/golden/make_golden.py from the reference's own Oracle,
src/xgraph/oracle.py) through this oracle and requires every allowed set, public
state projection and closed span to be equal.

Scope: the span language of src/xgraph/oracle.py with the policies the engine serves:
ordinary entity/fact spans, escapes, repeats, derivation, paths (union and committed),
bound_escapes, unquoted_starts, start_rank "degree"/"sitelinks", KG versions,
end_after_answer, opened states, residual-goal STOP (src/xgraph/oracle.py:1608-1635,
with the question's relation table of xgraph_b200.stopping), the weaker relation
supports relations="vocabulary" / "successor" (src/xgraph/oracle.py:67-79) and
expressions, the date and value comparisons (src/xgraph/oracle.py:104-133).  The
reference's observation, menu and audit policies are not restated; asking for them
raises.

Like the reference it reads a KG index's arrays as plain data (edge tuples, token
tuples) and recomputes everything per token from them.  One restructuring, for speed
only: `allowed` computes the token-independent part of a span step (the complete
candidates and which delimiters may start) once per state instead of once per token;
each token then takes the same branch logic as `advance`.
"""

from __future__ import annotations

from bisect import bisect_left, bisect_right
from collections.abc import Iterable, Mapping
from dataclasses import dataclass, replace
from enum import Enum

MAX_FACTS = 64  # src/xgraph/oracle.py:172
MAX_REACHED = 64  # src/xgraph/oracle.py:175
MAX_PATH_RELATIONS = 8  # src/xgraph/oracle.py:177
COMPARISONS = ("earlier", "later", "same")  # src/xgraph/oracle.py:196, by operator position


class Phase(Enum):
    FREE = "free text"
    SPAN = "span"
    ESCAPED = "escaped"


class Segment(Enum):
    SUBJECT = "subject"
    RELATION = "relation"
    OBJECT = "object"


class TokenNotAllowed(ValueError):
    pass


class IndexMismatch(ValueError):
    pass


@dataclass(frozen=True)
class ClosedSpan:
    """src/xgraph/oracle.py:202-240."""

    labels: tuple[tuple[int, ...], ...]
    entity_ids: tuple[str, ...]
    triples: tuple[tuple[str, str, str], ...]
    resolved: bool
    operator: str = ""
    operands: tuple[str, ...] = ()
    path: bool = False


UNRESOLVED = ClosedSpan((), (), (), resolved=False)


@dataclass(frozen=True)
class OracleState:
    """The in-scope fields of src/xgraph/oracle.py:249-341."""

    phase: Phase
    tail: bytes = b""
    segment: Segment = Segment.SUBJECT
    subjects: frozenset[str] = frozenset()
    relations: frozenset[str] = frozenset()
    written: tuple[tuple[int, ...], ...] = ()
    typed: tuple[int, ...] | None = ()
    closing: bytes | None = None
    closing_label: tuple[int, ...] = ()
    separating: bytes | None = None
    separating_label: tuple[int, ...] = ()
    escaping: bytes | None = None
    last_span: ClosedSpan | None = None
    facts: tuple[tuple[tuple[int, ...], ...], ...] = ()
    reached: frozenset[int] | None = None
    ranks: tuple[tuple[str, int], ...] = ()
    version: str | None = None
    answer_complete: bool = False
    stop: object = None  # the request's STOP table (xgraph_b200.stopping.StopRelations), kept across spans
    operating: bytes | None = None  # expressions: operator bytes typed so far (after the label prefix)
    operator: int = 0  # expressions: the span's operator, its position + 1 (0: none)
    starts: tuple[tuple[str, ...], ...] = ()  # expressions: each written operand's ranked starts
    ranks_b: tuple[tuple[str, int], ...] = ()  # expressions: operand B's frontier with its ranks


RELATIONS = ("frontier", "vocabulary", "successor")  # src/xgraph/relations.py:18


class _Graph:
    """One KG version's plain edges (src/xgraph/oracle.py:344-364), by subject.  A version
    holds only the subjects its edits touch and reads every other subject from the base
    graph: the same edge set as the reference's full copy, without copying it."""

    def __init__(self, outgoing: dict[str, list[tuple[str, str, int]]], base: _Graph | None = None) -> None:
        self._outgoing = outgoing
        self._base = base

    def edges_of(self, subject: str):
        if self._base is not None and subject not in self._outgoing:
            return self._base.edges_of(subject)
        return self._outgoing.get(subject, ())

    def degree(self, subject: str) -> int:
        return len(self.edges_of(subject))

    def has_triples(self, subject: str) -> bool:
        return self.degree(subject) > 0

    def from_subjects(self, subjects):
        for s in subjects:
            yield from self.edges_of(s)


@dataclass
class _SpanContext:
    """Token-independent facts of one span state (which delimiter branches may start)."""

    complete: list[tuple[str, int]]
    closes: bool
    separates: bool
    escapes: bool
    forced: bool = False  # residual-goal STOP: only the closer (or the label) goes on
    separator: bytes = b""  # the delimiter the separator branch matches (operand A: the operand separator)
    operates: bool = False  # expressions: an operator may start with this token


_UNSUPPORTED = {
    "observe": 0,
    "observe_width": 0, "observe_defer": 0, "menu_close_next": False, "observe_select": False,
    "observe_answer": False, "observe_required": False, "observe_no_loop": False,
    "audit": False, "menu": 0, "observe_terminal": 0,
}


def check_expressions(index) -> None:
    """src/xgraph/index.py:686-704: the index a comparison can run on."""
    if not index.span_syntax.writes_expressions:
        raise ValueError("expressions need a KG index built for a span syntax with operators and an "
                         f"operand separator, not {index.span_syntax}")
    if not index.expressions:
        raise ValueError("the KG index was saved before labels holding expression syntax were excluded")
    if index.date_entities is None:
        raise ValueError("expressions need a KG index with the date table")


class Oracle:
    """src/xgraph/oracle.py:367-1923, restricted to the policies listed in the module doc."""

    def __init__(
        self,
        index,
        tokenizer,
        syntax,
        *,
        escapes: bool = True,
        repeats: bool = True,
        derivation: bool = False,
        paths: bool = False,
        bound_escapes: bool = True,
        committed_paths: bool = False,
        versions: Mapping[str, Iterable[tuple[str, str, str | None]]] | None = None,
        start_rank: str = "degree",
        unquoted_starts: bool = False,
        end_after_answer: bool = False,
        eos_token_ids: Iterable[int] = (),
        stop: str | None = None,
        relations: str = "frontier",
        expressions: bool = False,
        **others,
    ) -> None:
        # Constructor checks in the reference's order (src/xgraph/oracle.py:439-455).
        if index.tokenizer_fingerprint != tokenizer.fingerprint:
            raise IndexMismatch("the KG index was built for another tokenizer")
        if index.span_syntax != syntax:
            raise IndexMismatch("the KG index was built for another span syntax")
        if not (escapes or repeats):
            raise ValueError("repeats can only be switched off with escapes, the way out")
        if committed_paths and not paths:
            raise ValueError("committed_paths needs path mode (paths=True)")
        if end_after_answer and not paths:
            raise ValueError("end_after_answer needs path mode (paths=True)")
        for name, value in others.items():
            if name not in _UNSUPPORTED:
                raise TypeError(f"unexpected keyword argument {name!r}")
            if value != _UNSUPPORTED[name]:
                raise ValueError(f"the {name} policy is not restated by this oracle")
        # src/xgraph/oracle.py:540-545
        if expressions and not committed_paths:
            raise ValueError("expressions need committed paths (committed_paths=True)")
        if expressions and not escapes:
            raise ValueError("expressions need escapes, the way out of an operand or relation")
        if expressions and len(syntax.operators) > len(COMPARISONS):
            raise ValueError(f"expressions know the operators of {COMPARISONS}, by position")
        if stop not in (None, "residual-goal"):
            raise ValueError(f"unknown STOP rule {stop!r}; expected residual-goal")
        if stop and not committed_paths:
            raise ValueError("residual-goal STOP needs committed paths (committed_paths=True)")
        # src/xgraph/relations.py:24-28 (check_relations)
        if relations not in RELATIONS:
            raise ValueError(f"unknown relations mode {relations!r}; expected one of {RELATIONS}")
        if relations != "frontier" and (not paths or expressions or stop):
            raise ValueError("weaker relations need path mode without expressions or STOP")
        self._relations = relations
        self._stop_terms = None
        if stop:
            from xgraph_b200.stopping import RelationTerms

            self._stop_terms = RelationTerms.from_index(index, tokenizer)
        self._eos = tokenizer.check_eos_token_ids(eos_token_ids) if end_after_answer else frozenset()
        self._end_after_answer = end_after_answer
        if start_rank not in ("degree", "sitelinks"):
            raise ValueError(f"start_rank must be one of ('degree', 'sitelinks'), got {start_rank!r}")
        labels, relations = index.labels, index.relations
        # expressions (src/xgraph/oracle.py:557-569): each date entity's date; the operators
        # offered (the value comparison only with the verdict entities), with the label prefix
        self._expressions = expressions
        self._dates = {}
        if expressions:
            from xgraph_b200.dates import unpack_date

            check_expressions(index)
            self._dates = {labels.owner_ids[int(e)]: unpack_date(int(k))
                           for e, k in zip(index.date_entities, index.date_keys, strict=True)}
        offered = syntax.operators if index.verdicts else syntax.operators[:2]
        self._operators = [(syntax.label_prefix + op).encode("utf-8") for op in offered]
        self._verdicts = dict(index.verdicts or {})
        self._operand_separator = syntax.operand_separator.encode("utf-8")
        self._sitelinks: dict[str, int] = {}
        if start_rank == "sitelinks":
            if index.sitelinks is None:
                raise ValueError("the sitelink rank needs a KG index with sitelink counts")
            self._sitelinks = {e: int(n) for e, n in zip(labels.owner_ids, index.sitelinks, strict=True)}
        self._entity_rows = [(labels.row_tokens(r), labels.owner_id(r)) for r in range(labels.num_rows)]
        self._relation_rows = [
            (relations.row_tokens(r), relations.owner_id(r)) for r in range(relations.num_rows)
        ]
        self._relation_number = {owner: n for n, owner in enumerate(relations.owner_ids)}
        self._label_prefix = syntax.label_prefix
        self._first_row: dict[str, int] = {}
        self._rows_of: dict[str, list[int]] = {}
        for row, (_, owner) in enumerate(self._entity_rows):
            self._first_row.setdefault(owner, row)
            self._rows_of.setdefault(owner, []).append(row)
        # Plain base edges (src/xgraph/oracle.py:581-587).
        edges: set[tuple[str, str, int]] = set()
        for entity, subject in enumerate(labels.owner_ids):
            a, b = int(index.adjacency_offsets[entity]), int(index.adjacency_offsets[entity + 1])
            for e in range(a, b):
                edges.add((subject, relations.owner_ids[int(index.edge_relations[e])],
                           int(index.edge_objects[e])))
        outgoing: dict[str, list[tuple[str, str, int]]] = {}
        for edge in edges:
            outgoing.setdefault(edge[0], []).append(edge)
        base = _Graph(outgoing)
        self._graphs: dict[str | None, _Graph] = {None: base}
        # A version replaces every edge of an edited pair (src/xgraph/oracle.py:588-624).
        writable = {owner for _, owner in self._relation_rows}
        for name, edits in (versions or {}).items():
            if not isinstance(name, str) or not name:
                raise ValueError(f"a KG version needs a non-empty name, got {name!r}")
            edits = list(edits)
            pairs = {(s, r) for s, r, _ in edits}
            added = {
                (s, r, row)
                for s, r, o in edits
                if s in self._rows_of and r in writable
                for row in self._rows_of.get(o, ())
            }
            touched: dict[str, set[tuple[str, str, int]]] = {s: set() for s, _ in pairs}
            for s in touched:  # the subject's edges outside the edited pairs
                touched[s].update(e for e in base.edges_of(s) if (s, e[1]) not in pairs)
            for edge in added:
                touched[edge[0]].add(edge)
            self._graphs[name] = _Graph({s: list(v) for s, v in touched.items()}, base)
        # successor support (src/xgraph/oracle.py:625-636): per KG version, relation r1 ->
        # the relations some object of an r1 edge is the subject of
        self._successors: dict[str | None, dict[str, set[str]]] = {}
        if self._relations == "successor":
            for name, graph in self._graphs.items():
                all_edges = [e for subject in labels.owner_ids for e in graph.edges_of(subject)]
                outgoing_of: dict[str, set[str]] = {}
                for subject, relation, _ in all_edges:
                    outgoing_of.setdefault(subject, set()).add(relation)
                pairs: dict[str, set[str]] = {}
                for _, relation, obj in all_edges:
                    pairs.setdefault(relation, set()).update(outgoing_of.get(self._entity_rows[obj][1], ()))
                self._successors[name] = pairs
        self._derivation = derivation or paths
        self._paths = paths
        self._bound_escapes = bound_escapes
        self._committed = committed_paths
        self._escapes = escapes
        self._repeats = repeats
        self._bytes = [tokenizer.token_bytes(t) for t in range(tokenizer.vocab_size)]
        self._special = tokenizer.special_ids
        self._opener = syntax.opener.encode("utf-8")
        self._closer = syntax.closer.encode("utf-8")
        self._separator = syntax.separator.encode("utf-8")
        self._escape = syntax.escape.encode("utf-8")
        self._entity_ids = labels.owner_ids
        # rows no unbound subject names: quoted ones with unquoted starts, and always the
        # verdict entities' (src/xgraph/oracle.py:650-659)
        verdict_ids = set(self._verdicts.values())
        self._quoted_rows = frozenset(
            row
            for row, (tokens, owner) in enumerate(self._entity_rows)
            if owner in verdict_ids
            or (unquoted_starts and syntax.quoted(b"".join(self._bytes[t] for t in tokens)))
        )

    # -- states (src/xgraph/oracle.py:660-724) ------------------------------------

    def initial_state(self, version: str | None = None, *, question: str | None = None) -> OracleState:
        stop = self._stop_terms.for_question(question) if self._stop_terms is not None else None
        return OracleState(Phase.FREE, version=self._version(version), stop=stop)

    def anchored_state(self, entities: list[str], version: str | None = None, *,
                       question: str | None = None) -> OracleState:
        rows = self._rows_for(entities)
        if not rows:
            raise ValueError(f"anchor has no writable label rows: {entities!r}")
        stop = self.initial_state(question=question).stop
        return OracleState(Phase.FREE, reached=frozenset(rows[:MAX_REACHED]), version=self._version(version),
                           stop=stop)

    def opened_state(self, state: OracleState) -> OracleState:
        if state.answer_complete:
            raise ValueError("the answer is complete; only EOS may follow")
        if state.phase is not Phase.FREE:
            raise ValueError(f"a span opens from free text, not from {state.phase.value}")
        return OracleState(Phase.SPAN, last_span=state.last_span, facts=state.facts,
                           reached=state.reached, version=state.version, stop=state.stop)

    def _version(self, version: str | None) -> str | None:
        if version not in self._graphs:
            names = sorted(n for n in self._graphs if n is not None)
            raise ValueError(f"the oracle has no KG version {version!r}; it has {names}")
        return version

    def _graph(self, state: OracleState) -> _Graph:
        return self._graphs[state.version]

    def _rows_for(self, entities) -> list[int]:
        return sorted(r for e in set(entities) for r in self._rows_of.get(e, ()))

    # -- stepping (src/xgraph/oracle.py:736-828) ----------------------------------

    def allowed(self, state: OracleState) -> frozenset[int]:
        ctx = self._context(state) if state.phase is Phase.SPAN and not state.answer_complete else None
        return frozenset(t for t in range(len(self._bytes)) if self._step(state, t, ctx) is not None)

    def advance(self, state: OracleState, token: int) -> OracleState:
        following = self._step(state, token, None)
        if following is None:
            raise TokenNotAllowed(f"token {token} is not allowed in {state.phase.value}")
        return following

    def _step(self, state: OracleState, token: int, ctx: _SpanContext | None) -> OracleState | None:
        if not 0 <= token < len(self._bytes):
            return None
        if state.answer_complete:
            return state if token in self._eos else None
        data = self._bytes[token]
        if state.phase is Phase.FREE and token in self._special:
            return replace(state, tail=b"")
        if data is None:
            return None
        if state.phase is Phase.FREE:
            return self._free_step(state, data)
        if state.phase is Phase.SPAN:
            return self._span_step(state, token, data, ctx or self._context(state))
        return self._escaped_step(state, data)

    def _free_step(self, state: OracleState, data: bytes) -> OracleState | None:
        text = state.tail + data
        at = text.find(self._opener)
        if at < 0:
            keep = len(self._opener) - 1
            return replace(state, tail=text[len(text) - keep:] if keep > 0 else b"")
        if at + len(self._opener) != len(text):
            return None
        return self.opened_state(state)

    def _escaped_step(self, state: OracleState, data: bytes) -> OracleState | None:
        text = state.tail + data
        at = text.find(self._closer)
        if at < 0:
            keep = len(self._closer) - 1
            return replace(state, tail=text[len(text) - keep:] if keep > 0 else b"")
        if at + len(self._closer) != len(text):
            return None
        return OracleState(Phase.FREE, last_span=UNRESOLVED, facts=state.facts,
                           reached=state.reached, version=state.version, stop=state.stop)

    # -- candidates (src/xgraph/oracle.py:830-894) --------------------------------

    def _unbound(self, state: OracleState) -> bool:
        return state.segment is Segment.SUBJECT and (not self._derivation or state.reached is None)

    def _candidates(self, state: OracleState, prefix, *, exact: bool = False):
        """(tokens, item, row) of the segment's candidate rows that start with (or, exact,
        equal) prefix, in row order."""
        if prefix is None:
            return []
        if self._unbound(state):
            n = len(prefix)
            key = (lambda item: item[0]) if exact else (lambda item: item[0][:n])
            lo = bisect_left(self._entity_rows, prefix, key=key)
            hi = bisect_right(self._entity_rows, prefix, key=key)
            return [(*self._entity_rows[r], r) for r in range(lo, hi) if r not in self._quoted_rows]
        n = len(prefix)
        return [
            c for c in self._segment_candidates(state)
            if (c[0] == prefix if exact else c[0][:n] == prefix)
        ]

    def _segment_candidates(self, state: OracleState):
        if state.segment is Segment.SUBJECT:
            return [(*self._entity_rows[r], r) for r in sorted(state.reached)]
        graph = self._graph(state)
        if state.segment is Segment.RELATION:
            if self._relations != "frontier":  # src/xgraph/oracle.py:865-878
                if self._relations == "vocabulary" or not state.relations:
                    have = {r for _, r in self._relation_rows}
                else:
                    have = set().union(*(self._successors[state.version].get(r, set()) for r in state.relations))
            else:
                have = {r for _, r, _ in graph.from_subjects(state.subjects)}
                if state.operator:  # a comparison: the relations both frontiers have
                    have &= {r for _, r, _ in graph.from_subjects(dict(state.ranks_b))}
            return [(tokens, r, row) for row, (tokens, r) in enumerate(self._relation_rows) if r in have]
        objects = {
            o for s, r, o in graph.from_subjects(state.subjects)
            if s in state.subjects and r in state.relations
        }
        return [(*self._entity_rows[r], r) for r in sorted(objects)]

    # -- span step (src/xgraph/oracle.py:896-1263, in-scope branches) -------------

    def _context(self, state: OracleState) -> _SpanContext:
        complete: list[tuple[str, int]] = []
        if state.typed is not None:
            complete = [(item, row) for _, item, row in self._candidates(state, state.typed, exact=True)]
        closes = bool(complete) and (state.segment is not Segment.RELATION or self._paths)
        if closes and state.segment is Segment.OBJECT and not self._repeats:
            closes = (*state.written, state.typed) not in state.facts
        if closes and state.operator:  # a comparison closes after a relation, where it has a result
            closes = state.segment is Segment.RELATION and self._result(state, state.typed) is not None
        graph = self._graph(state)
        operands = 2 if state.operator else 1  # the subject labels a path or comparison writes
        separates = False
        if state.segment is Segment.SUBJECT:
            separates = not self._answers_path(state) and any(graph.has_triples(e) for e, _ in complete)
        elif state.segment is Segment.RELATION and complete:
            separates = not self._paths or (  # src/xgraph/oracle.py:1060-1078
                len(state.written) - operands < MAX_PATH_RELATIONS - 1
                and (self._relations != "frontier"
                     or all(any(graph.has_triples(e) for e in self._frontier(state, state.typed, k))
                            for k in range(operands)))
                and (self._relations != "successor" or bool(self._successors_after(state, state.typed)))
            )
        # residual-goal STOP (src/xgraph/oracle.py:1081-1111): the separator and the escape
        # marker neither start nor go on; the closer and the label do
        forced = bool(complete) and self._residual_goal_stop(state)
        if forced:
            separates = False
        escapes = self._escapes and state.typed is not None and self._may_escape(state) and not forced
        # operand A of a comparison is followed by the operand separator instead
        operand_a = state.operator and state.segment is Segment.SUBJECT and not state.written
        operates = (self._expressions and state.segment is Segment.SUBJECT and not state.operator
                    and state.typed == () and not state.reached)  # src/xgraph/oracle.py:1669-1678
        return _SpanContext(complete, closes, separates, escapes, forced,
                            self._operand_separator if operand_a else self._separator, operates)

    @staticmethod
    def _branch(typed, label, data, delimiter, may_start, current):
        """src/xgraph/oracle.py:1637-1653."""
        if typed is not None:
            typed += data
        elif may_start:
            typed, label = data, current or ()
        if typed is None or not delimiter.startswith(typed):
            return None, ()
        return typed, label

    def _span_step(self, state: OracleState, token: int, data: bytes, ctx: _SpanContext):
        label = None
        if state.typed is not None and self._candidates(state, (*state.typed, token)):
            label = (*state.typed, token)
        closing, closing_label = self._branch(
            state.closing, state.closing_label, data, self._closer, ctx.closes, state.typed)
        separating, separating_label = self._branch(
            None if ctx.forced else state.separating, state.separating_label, data, ctx.separator, ctx.separates,
            state.typed)
        operating = state.operating + data if state.operating is not None else data if ctx.operates else None
        if operating is not None and not any(op.startswith(operating) for op in self._operators):
            operating = None
        escaping, _ = self._branch(None if ctx.forced else state.escaping, (), data, self._escape, ctx.escapes,
                                   state.typed)

        if closing == self._closer and state.operator:  # a comparison ends (src/xgraph/oracle.py:1115-1130)
            committed, result = self._result(state, closing_label)
            rows = self._rows_for(result)
            return OracleState(
                Phase.FREE,
                last_span=ClosedSpan((*state.written, closing_label), tuple(sorted(result)), (), True,
                                     COMPARISONS[state.operator - 1], committed),
                facts=state.facts,
                reached=frozenset(rows[:MAX_REACHED]),
                version=state.version, stop=state.stop,
            )
        if closing == self._closer and state.segment is Segment.RELATION:  # a path ends
            if self._relations != "frontier":  # an unexecuted plan (src/xgraph/oracle.py:1138-1147)
                return OracleState(
                    Phase.FREE,
                    last_span=ClosedSpan((*state.written, closing_label), (), (), False),
                    facts=state.facts,
                    version=state.version, stop=state.stop,
                )
            frontier = self._frontier(state, closing_label)
            if self._committed:
                best = min(frontier.values())
                frontier = {e: rank for e, rank in frontier.items() if rank == best}
            rows = self._rows_for(frontier)
            return OracleState(
                Phase.FREE,
                last_span=ClosedSpan((*state.written, closing_label), tuple(sorted(frontier)), (), True),
                facts=state.facts,
                reached=frozenset(rows[:MAX_REACHED]),
                version=state.version, stop=state.stop,
            )
        if closing == self._closer:
            facts, reached = state.facts, state.reached
            if state.segment is Segment.OBJECT:
                if len(facts) < MAX_FACTS:
                    facts = (*facts, (*state.written, closing_label))
                if self._derivation:
                    reached = self._reached(state, closing_label)
            return OracleState(
                Phase.FREE,
                last_span=self._resolve(state, closing_label),
                answer_complete=self._end_after_answer and self._answers_path(state),
                facts=facts,
                reached=reached,
                version=state.version, stop=state.stop,
            )
        if separating == ctx.separator:
            return self._next_segment(state, separating_label)
        if escaping == self._escape:
            return OracleState(Phase.ESCAPED, last_span=state.last_span, facts=state.facts,
                               reached=state.reached, version=state.version, stop=state.stop)
        if operating in self._operators:  # operand A follows
            return OracleState(Phase.SPAN, last_span=state.last_span, facts=state.facts, reached=state.reached,
                               version=state.version, stop=state.stop,
                               operator=self._operators.index(operating) + 1)
        if label is None and closing is None and separating is None and escaping is None and operating is None:
            return None
        return replace(
            state,
            typed=label,
            closing=closing,
            closing_label=closing_label,
            separating=separating,
            separating_label=separating_label,
            escaping=escaping,
            operating=operating,
        )

    # -- resolution and frontiers (src/xgraph/oracle.py:1655-1922) ---------------

    def _resolve(self, state: OracleState, label) -> ClosedSpan:
        rows = [(item, row) for _, item, row in self._candidates(state, label, exact=True)]
        if state.segment is Segment.SUBJECT and self._derivation and state.reached is not None:
            return ClosedSpan((label,), (self._best_connected(state, rows)[0],), (), True)
        if state.segment is Segment.SUBJECT:
            return ClosedSpan((label,), tuple(sorted(e for e, _ in rows)), (), True)
        objects = {row: entity for entity, row in rows}
        triples = {
            (s, r, objects[o]) for s, r, o in self._graph(state).from_subjects(state.subjects)
            if r in state.relations and o in objects
        }
        return ClosedSpan((*state.written, label), (), tuple(sorted(triples)), True)

    def _residual_goal_stop(self, state: OracleState) -> bool:
        """src/xgraph/oracle.py:1608-1635: inside a path, the typed relation label is
        complete, one of the relations it names is one the question's answer head names,
        and no relation of the new, whole frontier covers a question word that neither the
        written start nor the relations written so far (this one included) cover."""
        goal = state.stop
        if goal is None or not goal.head or state.operator or state.segment is not Segment.RELATION:
            return False
        followed = {self._relation_number[r] for tokens, r in self._relation_rows if tokens == state.typed}
        if not followed & goal.head:
            return False
        start = b"".join(self._bytes[t] for t in state.written[0]).decode("utf-8", "replace")
        used = goal.used_by_start(start.removeprefix(self._label_prefix))
        for label in (*state.written[1:], state.typed):
            used |= goal.used_by_relations(
                self._relation_number[r] for tokens, r in self._relation_rows if tokens == label)
        frontier = self._frontier(state, state.typed)
        return not any(goal.coverage.get(self._relation_number[r], 0) & ~used
                       for _, r, _ in self._graph(state).from_subjects(frontier))

    def _may_escape(self, state: OracleState) -> bool:
        bound = state.segment is Segment.SUBJECT and self._derivation and bool(state.reached)
        return self._bound_escapes or not bound

    def _best_connected(self, state: OracleState, rows) -> list[str]:
        graph, sitelinks = self._graph(state), self._sitelinks
        ordered = sorted(rows, key=lambda p: (-sitelinks.get(p[0], 0), -graph.degree(p[0]), p[1]))
        return list(dict.fromkeys(e for e, _ in ordered))

    def _kept(self, ranks: dict[str, int]) -> dict[str, int]:
        if self._committed:
            order = sorted(ranks, key=lambda e: (ranks[e], self._first_row[e]))
        else:
            order = sorted(ranks, key=self._first_row.get)
        return {e: ranks[e] for e in order[:MAX_REACHED]}

    def _frontier(self, state: OracleState, label, operand: int = 0) -> dict[str, int]:
        """The objects of operand `operand`'s frontier (a comparison's B: ranks_b) under
        every relation the label names, each with its least start rank, kept."""
        relations = {r for tokens, r in self._relation_rows if tokens == label}
        start = dict(state.ranks_b if operand else state.ranks)
        subjects = frozenset(start) if operand else state.subjects
        ranks: dict[str, int] = {}
        for s, r, o in self._graph(state).from_subjects(subjects):
            if s in subjects and r in relations:
                entity = self._entity_rows[o][1]
                ranks[entity] = min(ranks.get(entity, start[s]), start[s])
        return self._kept(ranks)

    def _result(self, state: OracleState, label):
        """A comparison closed after this relation label: the start entity each operand
        commits to and the result, or None where it cannot close (src/xgraph/oracle.py:
        1680-1737)."""
        if COMPARISONS[state.operator - 1] == "same":
            return self._same(state, label)
        fronts = [self._frontier(state, label, k) for k in (0, 1)]
        if not all(any(e in self._dates for e in front) for front in fronts):
            return None
        picked = []
        for k, front in enumerate(fronts):  # each operand's best start that reaches a date
            dated = {e: rank for e, rank in front.items() if e in self._dates}
            best = min(dated.values())
            earliest = min((self._dates[e] for e, rank in dated.items() if rank == best), key=lambda d: (d.lo, d.hi))
            picked.append((state.starts[k][best], earliest))
        (a, date_a), (b, date_b) = picked
        if date_a.before(date_b):
            earlier, later = {a}, {b}
        elif date_b.before(date_a):
            earlier, later = {b}, {a}
        else:  # equal or overlapping: undetermined, both
            earlier = later = {a, b}
        return (a, b), frozenset(earlier if COMPARISONS[state.operator - 1] == "earlier" else later)

    def _same(self, state: OracleState, label):
        """A value comparison: each operand's best start with any value, and the verdict
        entity (yes: a shared entity or an equal stored date)."""
        reached = []
        for k in (0, 1):
            front = self._frontier(state, label, k)
            if not front:
                return None
            best = min(front.values())
            reached.append((state.starts[k][best], {e for e, rank in front.items() if rank == best}))
        (a, values_a), (b, values_b) = reached
        entities_a = {e for e in values_a if e not in self._dates}
        entities_b = {e for e in values_b if e not in self._dates}
        if bool(entities_a) != bool(entities_b):  # values of two kinds
            return None
        dates_a = {self._dates[e] for e in values_a if e in self._dates}
        dates_b = {self._dates[e] for e in values_b if e in self._dates}
        verdict = "yes" if entities_a & entities_b or dates_a & dates_b else "no"
        return (a, b), frozenset({self._verdicts[verdict]})

    def _answers_path(self, state: OracleState) -> bool:
        last = state.last_span
        return self._paths and last is not None and (len(last.labels) > 1 or last.path)

    def _reached(self, state: OracleState, label) -> frozenset[int]:
        rows = {row for _, _, row in self._candidates(state, label, exact=True)}
        entities = {
            self._entity_rows[o][1] for s, r, o in self._graph(state).from_subjects(state.subjects)
            if r in state.relations and o in rows
        }
        reached = [row for row, (_, e) in enumerate(self._entity_rows) if e in entities]
        return frozenset(reached[:MAX_REACHED])

    def _successors_after(self, state: OracleState, label) -> set[str]:
        """src/xgraph/oracle.py:1599-1605."""
        return set().union(*(
            self._successors[state.version].get(r, set())
            for tokens, r, _ in self._candidates(state, label, exact=True) if tokens == label
        ))

    def _next_segment(self, state: OracleState, label) -> OracleState:
        candidates = [(item, row) for _, item, row in self._candidates(state, label, exact=True)]
        items = [item for item, _ in candidates]
        written = (*state.written, label)
        graph = self._graph(state)
        if self._relations != "frontier":  # no frontier (src/xgraph/oracle.py:1809-1822)
            return OracleState(
                Phase.SPAN, segment=Segment.RELATION,
                relations=frozenset(items) if state.segment is Segment.RELATION else frozenset(),
                written=written, last_span=state.last_span, facts=state.facts, reached=state.reached,
                version=state.version, stop=state.stop,
            )
        if state.segment is Segment.SUBJECT:
            subjects = frozenset(e for e in items if graph.has_triples(e))
            ranks: dict[str, int] = {}
            if self._paths:
                starts = self._best_connected(state, [(e, r) for e, r in candidates if e in subjects])
                ranks = self._kept({e: rank for rank, e in enumerate(starts)})
                subjects = frozenset(ranks)
            if state.operator:  # a comparison: rank this operand's starts (src/xgraph/oracle.py:1834-1870)
                ranked = tuple(sorted(ranks, key=ranks.get))
                if not state.written:  # operand A: operand B follows
                    return OracleState(
                        Phase.SPAN, written=written, last_span=state.last_span, facts=state.facts,
                        reached=state.reached, version=state.version, stop=state.stop,
                        operator=state.operator, starts=(ranked,), ranks=tuple(sorted(ranks.items())),
                    )
                return OracleState(  # operand B: both frontiers go on in lock step
                    Phase.SPAN, segment=Segment.RELATION, subjects=frozenset(dict(state.ranks)), written=written,
                    last_span=state.last_span, facts=state.facts, reached=state.reached,
                    version=state.version, stop=state.stop, ranks=state.ranks, operator=state.operator,
                    starts=(*state.starts, ranked), ranks_b=tuple(sorted(ranks.items())),
                )
            if not self._paths and self._derivation and subjects:
                best = self._best_connected(state, [(e, r) for e, r in candidates if e in subjects])
                subjects = frozenset(best[:1])
            return OracleState(
                Phase.SPAN, segment=Segment.RELATION, subjects=subjects, written=written,
                last_span=state.last_span, facts=state.facts, reached=state.reached,
                version=state.version, stop=state.stop, ranks=tuple(sorted(ranks.items())),
            )
        if self._paths:
            frontier = self._frontier(state, label)
            other = self._frontier(state, label, 1) if state.operator else {}
            return OracleState(
                Phase.SPAN, segment=Segment.RELATION, subjects=frozenset(frontier), written=written,
                last_span=state.last_span, facts=state.facts, reached=state.reached,
                version=state.version, stop=state.stop, ranks=tuple(sorted(frontier.items())),
                operator=state.operator, starts=state.starts, ranks_b=tuple(sorted(other.items())),
            )
        return OracleState(
            Phase.SPAN, segment=Segment.OBJECT, subjects=state.subjects, relations=frozenset(items),
            written=written, last_span=state.last_span, facts=state.facts, reached=state.reached,
            version=state.version, stop=state.stop,
        )
