"""The fused step's early writes, pinned to the reference's own walks (CPU).

The fused step writes -inf early, before a row's state machine runs, outside rel_any (every
relation label token and every delimiter token) for a row whose one new token (a) is
allowed, continues no delimiter and leaves the row in a relation segment, or (b) completes
the separator (and not the closer) after a subject or a path relation.  The rule rests on
two facts about the span language, checked here on every state of the golden walks (the
reference Oracle's, tests/golden/make_golden.py) through the oracle that reproduces them:

- every allowed set of a state in a relation segment lies inside rel_any;
- wherever the rule's premises hold (computed from the state and the token the way the
  kernel computes them: the delimiter branches that may start or go on, the token's bytes),
  the next state is in a relation segment, so its allowed set lies inside rel_any.
"""

from __future__ import annotations

from functools import cache

import numpy as np

from tests.conftest import case_index, golden_walks, make_oracle, start_state, world, world_index


@cache
def rel_any(world_name: str, escapes: bool, with_sitelinks: bool) -> frozenset[int]:
    """rel_any as derive_kernel builds it: the relation rows' tokens and the packed
    delimiter lists' tokens (the escape list empty without escapes)."""
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.tables import delimiter_lists

    _, served, _ = world(world_name)
    index = world_index(world_name, with_sitelinks)
    syntax = SpanSyntax()
    token_bytes = [served.token_bytes(t) for t in range(served.vocab_size)]
    tokens = set(np.asarray(index.relations.tokens).tolist())
    for name in ("closer", "separator", "escape"):
        if name == "escape" and not escapes:
            continue
        _, listed, _ = delimiter_lists(getattr(syntax, name).encode("utf-8"), token_bytes)
        tokens |= set(listed.tolist())
    return frozenset(tokens)


def delimiter_tokens(world_name: str, escapes: bool) -> frozenset[int]:
    """Tokens that continue some delimiter from some byte position (the packed word of
    delimiter steps is non-zero for them)."""
    from xgraph_b200.syntax import SpanSyntax
    from xgraph_b200.tables import delimiter_lists

    _, served, _ = world(world_name)
    syntax = SpanSyntax()
    token_bytes = [served.token_bytes(t) for t in range(served.vocab_size)]
    out: set[int] = set()
    for name in ("closer", "separator", "escape"):
        if name == "escape" and not escapes:
            continue
        _, listed, _ = delimiter_lists(getattr(syntax, name).encode("utf-8"), token_bytes)
        out |= set(listed.tolist())
    return frozenset(out)


def test_relation_segment_masks_lie_inside_rel_any_and_the_early_rule_holds():
    from xgraph_b200.syntax import SpanSyntax

    syntax = SpanSyntax()
    closer, separator = syntax.closer.encode("utf-8"), syntax.separator.encode("utf-8")
    relation_states = fired_a = fired_b = 0
    for case in golden_walks():
        options = case["options"]
        escapes = options.get("escapes", True)
        paths = options.get("paths", False)
        superset = rel_any(case["world"], escapes, case_index(case).sitelinks is not None)
        delims = delimiter_tokens(case["world"], escapes)
        _, served, _ = world(case["world"])
        oracle = make_oracle(case)
        for k, sequence in enumerate(case["sequences"]):
            state = start_state(oracle, sequence)
            for step, token in enumerate(sequence["tokens"]):
                where = (case["name"], k, step)
                allowed = oracle.allowed(state)
                in_span = state.phase.value == "span" and not state.answer_complete
                if in_span and state.segment.value == "relation":
                    relation_states += 1
                    assert allowed <= superset, where
                rule_a = rule_b = False
                if in_span and token in allowed:
                    data = served.token_bytes(token)
                    ctx = oracle._context(state)
                    if state.segment.value == "relation" and token not in delims:
                        rule_a = True
                    elif state.segment.value == "subject" or (state.segment.value == "relation" and paths):
                        close = (state.closing + data if state.closing is not None
                                 else data if ctx.closes else None)
                        going = state.separating is not None and not ctx.forced
                        sep = state.separating + data if going else data if ctx.separates else None
                        rule_b = close != closer and sep == separator
                nxt = oracle.advance(state, token)
                if rule_a or rule_b:
                    fired_a += rule_a
                    fired_b += rule_b
                    assert nxt.phase.value == "span" and nxt.segment.value == "relation", where
                    assert oracle.allowed(nxt) <= superset, where
                state = nxt
    assert relation_states > 500 and fired_a > 100 and fired_b > 50, (relation_states, fired_a, fired_b)


def test_early_rule_holds_on_the_expression_walks():
    """The same two facts on every state of the reference's expression walks (date and value
    comparisons, tests/golden/make_expression_cases.py): a comparison's relation segment
    allows only relation label and delimiter tokens, and the rule -- whose separator case
    leaves out a comparison's operands, whose separator (the operand separator after operand
    A) the packed delimiter steps do not describe -- leads only into relation segments."""
    from tests.test_expressions import edits_of, expression_cases, make_oracle
    from xgraph_b200.syntax import SpanSyntax

    syntax = SpanSyntax()
    closer, separator = syntax.closer.encode("utf-8"), syntax.separator.encode("utf-8")
    relation_states = fired = 0
    for case in expression_cases():
        superset = rel_any(case["world"], True, False)
        delims = delimiter_tokens(case["world"], True)
        _, served, _ = world(case["world"])
        oracle = make_oracle(case)
        assert edits_of(case) is None or oracle is not None
        for n, w in enumerate(case["walks"]):
            state = oracle.initial_state(w["version"])
            for step, token in enumerate(w["tokens"]):
                where = (case["world"], n, step)
                allowed = oracle.allowed(state)
                in_span = state.phase.value == "span" and not state.answer_complete
                if in_span and state.segment.value == "relation":
                    relation_states += 1
                    assert allowed <= superset, where
                rule = False
                if in_span and token in allowed:
                    data = served.token_bytes(token)
                    ctx = oracle._context(state)
                    if state.segment.value == "relation" and token not in delims:
                        rule = True
                    elif (state.segment.value == "subject" and not state.operator) or state.segment.value == "relation":
                        close = (state.closing + data if state.closing is not None
                                 else data if ctx.closes else None)
                        going = state.separating is not None and not ctx.forced
                        sep = state.separating + data if going else data if ctx.separates else None
                        rule = close != closer and sep == separator
                nxt = oracle.advance(state, token)
                if rule:
                    fired += 1
                    assert nxt.phase.value == "span" and nxt.segment.value == "relation", where
                    assert oracle.allowed(nxt) <= superset, where
                state = nxt
    assert relation_states > 100 and fired > 50, (relation_states, fired)
