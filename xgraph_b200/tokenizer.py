"""The served tokenizer: the vocabulary whose ids the engine masks, seen as bytes.

Same contract as the reference's `ServedTokenizer` (src/xgraph/tokenizer.py:19-86):
a dense id domain ``0 .. vocab_size - 1``, ``token_bytes(t)`` (None for special and
unused ids), ``special_ids``, ``encode`` without special tokens, and a SHA-256
``fingerprint`` of the serialized tokenizer that binds a KG index to it.
Two vocabulary families are read: byte-level BPE (GPT-2 style printable alphabet)
and SentencePiece-style BPE with ``<0xNN>`` byte fallback and ``▁`` for a space.
"""

from __future__ import annotations

import hashlib
import json
import re
from collections.abc import Iterable
from functools import cache
from pathlib import Path

from tokenizers import Tokenizer


class UnsupportedTokenizer(ValueError):
    """The tokenizer's vocabulary cannot be read as bytes, or its ids are not dense."""


SPACE = "▁"
_BYTE_PIECE = re.compile(r"<0x([0-9A-Fa-f]{2})>")


@cache
def byte_level_alphabet() -> dict[str, int]:
    """The GPT-2 byte-to-character map, inverted (character -> byte).

    Printable Latin-1 bytes stand for themselves; the other 68 bytes are shifted, in
    increasing byte order, to the code points 256, 257, ... (the published
    ``bytes_to_unicode`` construction of GPT-2's encoder)."""
    kept = set(range(0x21, 0x7F)) | set(range(0xA1, 0xAD)) | set(range(0xAE, 0x100))
    inverse: dict[str, int] = {}
    shifted = 0
    for byte in range(256):
        if byte in kept:
            inverse[chr(byte)] = byte
        else:
            inverse[chr(256 + shifted)] = byte
            shifted += 1
    return inverse


def _flatten_decoders(decoder: dict | None) -> list[dict]:
    if not decoder:
        return []
    if decoder.get("type") == "Sequence":
        out: list[dict] = []
        for inner in decoder.get("decoders", []):
            out.extend(_flatten_decoders(inner))
        return out
    return [decoder]


def _vocabulary(spec: dict) -> tuple[list[bytes | None], frozenset[int]]:
    steps = _flatten_decoders(spec.get("decoder"))
    byte_level = any(step.get("type") == "ByteLevel" for step in steps)
    space_step = {"type": "Replace", "pattern": {"String": SPACE}, "content": " "}
    sentencepiece = (
        spec["model"].get("byte_fallback") is True
        and space_step in steps
        and any(step.get("type") == "ByteFallback" for step in steps)
    )
    if spec["model"].get("type") != "BPE" or not (byte_level or sentencepiece):
        raise UnsupportedTokenizer(
            "only byte-level BPE or SentencePiece-style BPE with byte fallback is supported; "
            f"got model {spec['model'].get('type')!r} with decoder {spec.get('decoder')!r}"
        )
    vocab: dict[str, int] = spec["model"]["vocab"]
    added = spec.get("added_tokens", [])
    size = 1 + max([*vocab.values(), *(a["id"] for a in added)])
    table: list[bytes | None] = [None] * size
    unknown = spec["model"].get("unk_token")
    alphabet = byte_level_alphabet()
    for piece, token in vocab.items():
        if piece == unknown and not byte_level:
            continue
        if byte_level:
            try:
                table[token] = bytes(alphabet[ch] for ch in piece)
            except KeyError as error:
                raise UnsupportedTokenizer(
                    f"token {token} ({piece!r}) has a character outside the byte-level alphabet"
                ) from error
        else:
            one = _BYTE_PIECE.fullmatch(piece)
            table[token] = (
                bytes([int(one[1], 16)]) if one else piece.replace(SPACE, " ").encode("utf-8")
            )
    special: set[int] = set()
    for entry in added:
        if entry["special"]:
            table[entry["id"]] = None
            special.add(entry["id"])
        else:
            table[entry["id"]] = entry["content"].encode("utf-8")
    return table, frozenset(special)


class ServedTokenizer:
    """A snapshot of a ``tokenizers.Tokenizer`` with a byte view of every id."""

    def __init__(self, tokenizer: Tokenizer) -> None:
        serialized = tokenizer.to_str()
        self._tokenizer = Tokenizer.from_str(serialized)
        ids = set(self._tokenizer.get_vocab(with_added_tokens=True).values())
        size = self._tokenizer.get_vocab_size(with_added_tokens=True)
        if not ids or ids != set(range(size)):
            raise UnsupportedTokenizer(
                "a nonempty dense token ID domain 0 .. vocab_size - 1 is required"
            )
        self.fingerprint = hashlib.sha256(serialized.encode("utf-8")).hexdigest()
        self._token_bytes, self._special_ids = _vocabulary(json.loads(serialized))

    @classmethod
    def from_file(cls, path: str | Path) -> ServedTokenizer:
        return cls(Tokenizer.from_file(str(path)))

    @property
    def vocab_size(self) -> int:
        return self._tokenizer.get_vocab_size(with_added_tokens=True)

    def encode(self, text: str) -> list[int]:
        return self._tokenizer.encode(text, add_special_tokens=False).ids

    def encode_batch(self, texts: list[str]) -> list[list[int]]:
        return [e.ids for e in self._tokenizer.encode_batch(texts, add_special_tokens=False)]

    @property
    def special_ids(self) -> frozenset[int]:
        return self._special_ids

    def token_bytes(self, token: int) -> bytes | None:
        return self._token_bytes[token] if 0 <= token < len(self._token_bytes) else None

    def byte_table(self):
        """Every id of the byte view as CSR: (offsets int64 [n + 1], bytes uint8, kind int8
        [n]: 0 known bytes, 1 special, 2 unknown bytes), n = the ids the view covers."""
        import numpy as np

        cached = getattr(self, "_byte_table", None)
        if cached is None:
            table = self._token_bytes
            kind = np.array([1 if t in self._special_ids else 2 if b is None else 0 for t, b in enumerate(table)],
                            dtype=np.int8)
            lengths = np.fromiter((0 if b is None else len(b) for b in table), dtype=np.int64, count=len(table))
            offsets = np.zeros(len(table) + 1, dtype=np.int64)
            np.cumsum(lengths, out=offsets[1:])
            data = np.frombuffer(bytearray(b"".join(b for b in table if b is not None)), dtype=np.uint8)
            cached = self._byte_table = (offsets, data, kind)
        return cached

    def all_token_bytes(self) -> list[bytes | None]:
        """Every id's bytes, in id order (a copy)."""
        return list(self._token_bytes[: self.vocab_size]) + [None] * max(
            0, self.vocab_size - len(self._token_bytes)
        )

    def check_eos_token_ids(self, tokens: Iterable[int]) -> frozenset[int]:
        ids = tuple(tokens)
        if not ids or any(type(t) is not int or not 0 <= t < self.vocab_size for t in ids):
            raise ValueError(
                "end_after_answer needs nonempty EOS token ids in the served vocabulary"
            )
        return frozenset(ids)
