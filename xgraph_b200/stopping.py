"""Residual-goal STOP: the per-request relation table the engine's STOP rule reads.

The rule (src/xgraph/stopping.py:1-10, src/xgraph/oracle.py:1608-1635): inside a path, a
complete relation label whose relations include one named by the question's answer head
closes the path there -- only the closer may follow -- unless some relation of the new,
whole frontier still covers a question word that neither the written start nor the
relations consumed so far cover.  The host side is the reference's
(src/xgraph/stopping.py:48-133 StopRelations and RelationTerms, over the word helpers of
src/xgraph/repair.py:192-284): the question's answer head, its content stems, and for
each relation the question words its label words cover, one bit per word (at most
MAX_STOP_WORDS words).  `StopRelations.arrays` packs one request's table for the engine
(xg_set_stop).

The word lists, the stemming steps and the head pattern below are the reference's: STOP
must fire on exactly the questions and relations the reference's does.
"""

from __future__ import annotations

import os
import re
from dataclasses import dataclass, field

import numpy as np

MAX_STOP_WORDS = 64
MAX_STOP_BYTES = 4096
"""Bounds on a request's relevant raw question words and their UTF-8 bytes
(src/xgraph/stopping.py:45-47)."""

_WORD = re.compile(r"\w+")
_STOPWORDS = frozenset({
    "a", "an", "the", "of", "in", "on", "at", "to", "into", "from", "for", "by", "with",
    "as", "is", "was", "are", "were", "be", "been", "being", "does", "did", "do", "has",
    "have", "had", "which", "what", "who", "whom", "whose", "where", "when", "how", "that",
    "this", "these", "those", "it", "its", "their", "his", "her", "and", "or", "not", "any",
    "some", "one", "there", "located",
})
"""Function words (and `located`), neither question content nor relation words
(src/xgraph/repair.py:197-203)."""
_SYNONYMS = {"born": "birth", "died": "death", "die": "death", "dies": "death"}
_SUFFIXES = ("ship", "ation", "ing", "ion", "ed", "er", "es", "s")
_HEAD = re.compile(
    r"^\s*(?:(?:in|on|of|to|into|from|at|for|by|with|under|through)\s+)?"
    r"(which|what|who|whom|whose|where)\b\s*"
    r"(?:(?:is|was|are|were|does|did|do|has|had)\s+)?(?:(?:the|a|an)\s+)?(\w+)?",
    re.IGNORECASE,
)
WH_HEADS = ("who", "whom", "whose", "where")
"""Question words that are their own answer head (src/xgraph/repair.py:214)."""


def _lexical_text(text: str) -> str:
    """src/xgraph/repair.py:236-241: the optional freebase schema adaptation."""
    schema = os.environ.get("XGRAPH_LEXICAL_SCHEMA", "")
    if schema not in ("", "freebase"):
        raise ValueError(f"unknown XGRAPH_LEXICAL_SCHEMA: {schema!r}")
    return text.replace("_", " ").replace(".", " ") if schema else text


def stem(word: str) -> str:
    """src/xgraph/repair.py:255-264: a synonym, then one suffix stripped when three
    letters remain, then the first five letters."""
    word = _SYNONYMS.get(word, word)
    for suffix in _SUFFIXES:
        if word.endswith(suffix) and len(word) - len(suffix) >= 3:
            word = word[: -len(suffix)]
            break
    return word[:5]


def content_stems(text: str, drop: frozenset[str] | set[str] = frozenset()) -> set[str]:
    """src/xgraph/repair.py:267-270: stems of the case-folded words that are neither
    stopwords nor dropped."""
    return {stem(w) for w in _WORD.findall(_lexical_text(text).casefold()) if w not in _STOPWORDS and w not in drop}


def answer_head(question: str) -> str | None:
    """src/xgraph/repair.py:273-283: the word after a leading which / what, else who,
    whom, whose or where itself; None for a question that starts otherwise."""
    found = _HEAD.match(question)
    if not found:
        return None
    wh, word = found.group(1).casefold(), (found.group(2) or "").casefold()
    if wh in WH_HEADS:
        return wh
    return word if word and word not in _STOPWORDS else None


def label_words(text: str) -> set[str]:
    """src/xgraph/stopping.py:41-42: case-folded words with trailing s removed."""
    return {word.rstrip("s") for word in _WORD.findall(text.casefold())}


def start_words(text: str) -> list[str]:
    """The case-folded words of a written start label, as StopRelations.used_by_start reads
    them (src/xgraph/stopping.py:61-63)."""
    return _WORD.findall(text.casefold())


@dataclass(frozen=True)
class StopRelations:
    """One request's STOP table (src/xgraph/stopping.py:50-71): the relations its answer
    head names, one bit per relevant raw question word, each relation's covered words."""

    head: frozenset[int]
    residual: frozenset[int]
    words: tuple[str, ...]
    coverage: dict[int, int]

    def used_by_start(self, start: str) -> int:
        found = set(start_words(start))
        return sum(1 << i for i, word in enumerate(self.words) if word in found)

    def used_by_relations(self, relations) -> int:
        mask = 0
        for relation in relations:
            mask |= self.coverage.get(relation, 0)
        return mask

    def arrays(self, relations: int) -> tuple[np.ndarray, np.ndarray, bytes]:
        """The engine's layout of this table: (per relation number [head flag, coverage low
        32 bits, coverage high 32 bits] int32 [relations, 3]; word offsets int32
        [MAX_STOP_WORDS + 2]: the word count, then each word's byte offset and the end;
        the words' UTF-8 bytes)."""
        table = np.zeros((relations, 3), dtype=np.int32)
        for relation in self.head:
            table[relation, 0] = 1
        for relation, mask in self.coverage.items():
            table[relation, 1] = np.int64(mask & 0xFFFFFFFF).astype(np.int32)
            table[relation, 2] = np.int64((mask >> 32) & 0xFFFFFFFF).astype(np.int32)
        encoded = [w.encode("utf-8") for w in self.words]
        offsets = np.zeros(MAX_STOP_WORDS + 2, dtype=np.int32)
        offsets[0] = len(encoded)
        offsets[1: len(encoded) + 2] = np.concatenate([[0], np.cumsum([len(b) for b in encoded])]) if encoded else 0
        return table, offsets, b"".join(encoded)


@dataclass(frozen=True)
class RelationTerms:
    """Words and content stems of the indexed relation labels, by relation number
    (src/xgraph/stopping.py:74-133)."""

    words: dict[int, set[str]]
    stems: dict[int, set[str]]
    _by_word: dict[str, set[int]] = field(init=False, repr=False, compare=False)
    _by_stem: dict[str, set[int]] = field(init=False, repr=False, compare=False)

    def __post_init__(self) -> None:
        for source, name in ((self.words, "_by_word"), (self.stems, "_by_stem")):
            indexed: dict[str, set[int]] = {}
            for relation, terms in source.items():
                for term in terms:
                    indexed.setdefault(term, set()).add(relation)
            object.__setattr__(self, name, indexed)

    @classmethod
    def from_index(cls, index, tokenizer) -> RelationTerms:
        words: dict[int, set[str]] = {}
        stems: dict[int, set[str]] = {}
        prefix = index.span_syntax.label_prefix
        for row in range(index.relations.num_rows):
            raw = b"".join(tokenizer.token_bytes(t) or b"" for t in index.relations.row_tokens(row))
            name = raw.decode("utf-8", "replace").removeprefix(prefix)
            relation = int(index.relations.owners[row])
            words.setdefault(relation, set()).update(label_words(name))
            stems.setdefault(relation, set()).update(content_stems(name))
        return cls(words, stems)

    def for_question(self, question: str) -> StopRelations:
        if not isinstance(question, str) or not question.strip():
            raise ValueError("residual-goal STOP needs the question text")
        head = answer_head(question)
        heads = frozenset(self._by_word.get(head.rstrip("s"), ())) if head else frozenset()
        if head is None or head in WH_HEADS or not heads:
            return StopRelations(frozenset(), frozenset(), (), {})
        head_stem = stem(head)
        question_stems = {
            word: normalized
            for word in set(_WORD.findall(question.casefold()))
            for normalized in content_stems(word)
            if normalized in self._by_stem and normalized != head_stem
        }
        words = tuple(sorted(question_stems))
        if len(words) > MAX_STOP_WORDS or sum(len(w.encode("utf-8")) for w in words) > MAX_STOP_BYTES:
            raise ValueError(
                f"residual-goal STOP supports at most {MAX_STOP_WORDS} relevant question "
                f"words and {MAX_STOP_BYTES} UTF-8 bytes"
            )
        coverage: dict[int, int] = {}
        for i, word in enumerate(words):
            for relation in self._by_stem[question_stems[word]]:
                coverage[relation] = coverage.get(relation, 0) | (1 << i)
        return StopRelations(heads, frozenset(coverage), words, coverage)


def label_word_table(index, tokenizer) -> tuple[np.ndarray, np.ndarray]:
    """The engine's label words (xg_enable_stop): for every entity label row, the
    case-folded \\w+ words of its text after the label prefix, each followed by a 0 byte, as
    CSR (offsets int64 [rows + 1], bytes uint8); the reference's stop_label_offsets /
    stop_label_words (src/xgraph/engine.py:537-551)."""
    prefix = index.span_syntax.label_prefix
    offsets = np.zeros(index.labels.num_rows + 1, dtype=np.int64)
    written = bytearray()
    for row in range(index.labels.num_rows):
        raw = b"".join(tokenizer.token_bytes(t) or b"" for t in index.labels.row_tokens(row))
        name = raw.decode("utf-8", "replace").removeprefix(prefix)
        written.extend(b"\0".join(w.encode("utf-8") for w in start_words(name)) + b"\0")
        offsets[row + 1] = len(written)
    return offsets, np.frombuffer(written, dtype=np.uint8)
