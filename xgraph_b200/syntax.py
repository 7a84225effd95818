"""Span syntax: the byte strings that open, separate, escape and close a KG span.

Mirrors the reference's `SpanSyntax` (src/xgraph/syntax.py:9-96): the same field
names, defaults, validation order and presets, so an index header written by
either side names the same syntax.  Only the parts the constraint engine reads are
used on the device: the opener, label prefix, separator, closer and escape marker.
Operators and the operand separator are kept so that `excludes` removes the same
labels as the reference index builder does.
"""

from __future__ import annotations

from dataclasses import dataclass

QUOTATION_MARKS = ('"', "“", "”", "„", "‟", "«", "»")
"""Double quotation marks and guillemets; a label starting with one is a quoted label
(src/xgraph/syntax.py:99-103).  Single quotes are not in the list on purpose: they
also write apostrophes at the start of names."""


@dataclass(frozen=True)
class SpanSyntax:
    """Delimiters of a span, e.g. ``⟦ Marie Curie · spouse · Pierre Curie⟧``.

    Inside a span the closer, separator, escape marker and operand separator are
    matched side by side, so none of them may be a prefix of another; the same
    holds among the escape marker and the operators written after the label prefix.
    """

    opener: str = "⟦"
    label_prefix: str = " "
    separator: str = " ·"
    closer: str = "⟧"
    escape: str = " ⁇"
    operand_separator: str = " |"
    operators: tuple[str, ...] = ("earlier:", "later:", "same:")

    def __post_init__(self) -> None:
        object.__setattr__(self, "operators", tuple(self.operators))
        for name in ("opener", "separator", "closer", "escape"):
            if not getattr(self, name):
                raise ValueError(f"the span {name} must not be empty")
        if self.operators and not self.operand_separator:
            raise ValueError("operators need an operand separator between their operands")
        if any(not op for op in self.operators):
            raise ValueError("an operator must not be empty")
        side_by_side = {
            "span closer": self.closer,
            "separator": self.separator,
            "escape marker": self.escape,
        }
        if self.operand_separator:
            side_by_side["operand separator"] = self.operand_separator
        at_start = {"escape marker": self.escape}
        for k, op in enumerate(self.operators):
            at_start[f"operator {k} ({op!r})"] = self.label_prefix + op
        for group in (side_by_side, at_start):
            encoded = {name: text.encode("utf-8") for name, text in group.items()}
            for name, text in encoded.items():
                for other, other_text in encoded.items():
                    if name != other and other_text.startswith(text):
                        raise ValueError(
                            f"the {name} {group[name]!r} must not be a prefix of the {other} "
                            f"{group[other]!r}"
                        )

    @property
    def delimiters(self) -> tuple[str, ...]:
        return (self.opener, self.separator, self.closer, self.escape)

    @property
    def writes_expressions(self) -> bool:
        return bool(self.operators)

    def excludes(self, label: str) -> bool:
        """A label whose written form (prefix + label) holds a delimiter or the operand
        separator anywhere, or starts with an operator, cannot be indexed."""
        written = self.label_prefix + label
        inner = list(self.delimiters)
        if self.operand_separator:
            inner.append(self.operand_separator)
        if any(d in written for d in inner):
            return True
        return any(written.startswith(self.label_prefix + op) for op in self.operators)

    def quoted(self, written: bytes) -> bool:
        """Whether an index row's bytes (label prefix + label) start with a quotation mark
        after the label prefix."""
        prefix = self.label_prefix.encode("utf-8")
        label = written[len(prefix):] if written.startswith(prefix) else written
        return any(label.startswith(mark.encode("utf-8")) for mark in QUOTATION_MARKS)


PRESETS: dict[str, SpanSyntax] = {
    "brackets": SpanSyntax(),
    "wiki": SpanSyntax(opener="[[", label_prefix="", separator="|", closer="]]"),
    "tags": SpanSyntax(opener="<kg>", label_prefix="", separator="|", closer="</kg>"),
    "cjk": SpanSyntax(opener="【", label_prefix="", separator="|", closer="】"),
    "json": SpanSyntax(opener='["', label_prefix="", separator='", "', closer='"]'),
}


def preset(name: str) -> SpanSyntax:
    if name not in PRESETS:
        raise ValueError(f"unknown span syntax {name!r}; expected one of {sorted(PRESETS)}")
    return PRESETS[name]
