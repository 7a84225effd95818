"""Pack a KG index into the engine's device blob (one allocation, 16-byte aligned tables).

Counterpart of the reference's `native_tables` (src/xgraph/engine.py:311-556), in this
engine's own layout (include/xgraph_b200.h, XgLayout):

- label rows and relation rows (tokens, int32 offsets, owners), each entity's first row
  and its rows (CSR), the subject adjacency (int32 CSR of relation / object row);
- the opener automaton for free text and the closer automaton for escaped spans: per
  matched-byte state and token, the next state, REJECT (-1) or COMPLETE (-2), plus each
  state's allowed-token mask (src/xgraph/engine.py:110-143 states the rule: a delimiter
  must end exactly at a token's end; special tokens reset the opener and are refused
  inside escapes; ids without bytes are refused);
- inside spans, per byte position of the closer, separator and escape marker, the
  sorted token ids that continue it and where they end (engine.py:146-162);
- the root mask (first tokens of the rows an unbound subject may name) and "wide"
  masks: the next-token mask of every unbound prefix range of >= WIDE_ROWS rows at
  depth 1..8, so the mask builder never scans thousands of rows per step;
- prefix counts of the rows an unbound subject may name (unquoted starts);
- KG-version overlays and sitelink counts.
All mask rows are padded to a multiple of four words so the device copies them with
16-byte vector loads.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

WIDE_ROWS = 1024
MAX_WIDE_DEPTH = 8
REJECT = -1
COMPLETE = -2
ALIGN = 64


class XgLayout(ctypes.Structure):
    _fields_ = (
        [("blob_bytes", ctypes.c_int64)]
        + [(n, ctypes.c_int32) for n in (
            "vocab", "words", "words_padded", "entity_rows", "relation_rows", "entities",
            "relations", "relation_words", "opener_len", "closer_len", "separator_len",
            "escape_len", "versions", "wide_count", "ent_cols", "rel_cols", "pad0", "pad1")]
        + [(n, ctypes.c_int64) for n in (
            "ent_tok", "ent_off", "ent_owner", "rel_tok", "rel_off", "rel_owner",
            "ent_col", "rel_col", "ent_first", "rel_first",
            "ent_first_row", "ent_rows_off", "ent_rows", "adj_off", "edge_rel", "edge_obj",
            "sitelinks", "kept_prefix", "root_mask", "wide_keys", "wide_masks",
            "free_next", "free_mask", "esc_next", "esc_mask", "eos_mask",
            "closer_off", "closer_tok", "closer_next", "separator_off", "separator_tok",
            "separator_next", "escape_off", "escape_tok", "escape_next",
            "ver_off", "ver_subj", "ver_adj", "ver_edge_rel", "ver_edge_obj", "dstep", "row_degree",
            "row_first", "run_off", "runs", "run_rel", "edge_first",
            "row_sitelinks")]
    )


class XgOptions(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "escapes", "repeats", "derivation", "paths", "bound_escapes", "committed_paths",
        "sitelinks_rank", "end_after_answer", "release_top")] + [
        ("release_log_mass", ctypes.c_float), ("escape_bias", ctypes.c_float), ("relations", ctypes.c_int32),
        ("expressions", ctypes.c_int32)]


def mask_words(vocab_size: int) -> int:
    return (vocab_size + 31) // 32


def padded_words(vocab_size: int) -> int:
    return (mask_words(vocab_size) + 3) // 4 * 4


def pack_mask(allowed: np.ndarray, words: int) -> np.ndarray:
    """A boolean array over token ids as uint32 words, bit i of word w for token 32w + i."""
    bits = np.zeros(words * 32, dtype=bool)
    bits[: len(allowed)] = allowed
    return np.packbits(bits, bitorder="little").view("<u4").astype(np.uint32)


def _kmp_failure(pattern: bytes) -> list[int]:
    fail = [0] * len(pattern)
    k = 0
    for i in range(1, len(pattern)):
        while k and pattern[i] != pattern[k]:
            k = fail[k - 1]
        if pattern[i] == pattern[k]:
            k += 1
        fail[i] = k
    return fail


def delimiter_automaton(delimiter: bytes, token_bytes, special: frozenset[int], specials_pass: bool):
    """Next-state codes int8 [len(delimiter), vocab] and boolean allowed [len, vocab]."""
    n = len(delimiter)
    fail = _kmp_failure(delimiter)
    # byte transition table of the partial-match automaton (states 0..n-1)
    step = np.zeros((n, 256), dtype=np.int16)
    for q in range(n):
        for byte in range(256):
            k = q
            while k and delimiter[k] != byte:
                k = fail[k - 1]
            step[q, byte] = k + 1 if delimiter[k] == byte else 0
    vocab = len(token_bytes)
    codes = np.full((n, vocab), REJECT, dtype=np.int8)
    for token, data in enumerate(token_bytes):
        if data is None:
            if token in special and specials_pass:
                codes[:, token] = 0
            continue
        for start in range(n):
            q = start
            code = None
            for at, byte in enumerate(data):
                q = int(step[q, byte])
                if q == n:
                    code = COMPLETE if at == len(data) - 1 else REJECT
                    break
            codes[start, token] = q if code is None else code
    return codes, codes != REJECT


def delimiter_lists(delimiter: bytes, token_bytes) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Per byte position p: sorted tokens whose bytes continue the delimiter from p, and
    the position after them (CSR offsets [len + 1], tokens, next)."""
    per: list[list[tuple[int, int]]] = [[] for _ in delimiter]
    for token, data in enumerate(token_bytes):
        if not data or len(data) > len(delimiter):
            continue
        for p in range(len(delimiter) - len(data) + 1):
            if delimiter.startswith(data, p):
                per[p].append((token, p + len(data)))
    off = np.zeros(len(delimiter) + 1, dtype=np.int32)
    np.cumsum([len(x) for x in per], out=off[1:])
    flat = [e for x in per for e in x]
    return off, np.array([t for t, _ in flat], dtype=np.int32), np.array([q for _, q in flat], dtype=np.int32)


def _row_columns(tokens: np.ndarray, offsets: np.ndarray, depth: int) -> np.ndarray:
    lengths = np.diff(offsets)
    col = np.full(len(lengths), -1, dtype=np.int64)
    has = lengths > depth
    col[has] = tokens[offsets[:-1][has] + depth]
    return col


def wide_masks(tokens, offsets, kept: np.ndarray | None, words_padded: int, wide: int = WIDE_ROWS):
    """Keys (range start * 16 + depth) and next-token masks of every prefix range of
    >= `wide` rows at depth 1..MAX_WIDE_DEPTH, counting only kept rows' next tokens."""
    rows = len(offsets) - 1
    keys: list[int] = []
    masks: list[np.ndarray] = []
    if rows < wide:
        return np.zeros(0, dtype=np.int64), np.zeros((0, words_padded), dtype=np.uint32)
    same = np.ones(rows, dtype=bool)  # row shares the first d tokens with the row before it
    same[0] = False
    for depth in range(1, MAX_WIDE_DEPTH + 1):
        col = _row_columns(tokens, offsets, depth - 1)
        present = col >= 0
        same[1:] &= (col[1:] == col[:-1]) & present[1:]
        same[0] = False
        starts = np.flatnonzero(~same & present)
        if not len(starts):
            break
        ends = np.empty_like(starts)
        # a run continues while `same` holds
        breaks = np.flatnonzero(~same)
        nxt = np.searchsorted(breaks, starts, side="right")
        ends[:] = np.where(nxt < len(breaks), breaks[np.minimum(nxt, len(breaks) - 1)], rows)
        following = _row_columns(tokens, offsets, depth)
        for lo, hi in zip(starts.tolist(), ends.tolist(), strict=True):
            if hi - lo < wide:
                continue
            nexts = following[lo:hi]
            if kept is not None:
                nexts = nexts[kept[lo:hi]]
            nexts = np.unique(nexts[nexts >= 0])
            mask = np.zeros(words_padded, dtype=np.uint32)
            np.bitwise_or.at(mask, nexts >> 5, (np.uint32(1) << (nexts & 31).astype(np.uint32)))
            keys.append(lo * 16 + depth)
            masks.append(mask)
        if not np.any(np.diff(np.append(starts, rows)) >= wide):
            break
    if not keys:
        return np.zeros(0, dtype=np.int64), np.zeros((0, words_padded), dtype=np.uint32)
    order = np.argsort(np.array(keys, dtype=np.int64))
    return np.array(keys, dtype=np.int64)[order], np.stack(masks)[order]


def quoted_rows(labels, token_bytes, syntax) -> np.ndarray:
    """Rows whose label starts with a quotation mark after the label prefix."""
    out = np.zeros(labels.num_rows, dtype=bool)
    tokens = np.asarray(labels.tokens)
    offsets = np.asarray(labels.offsets)
    need = len(syntax.label_prefix.encode("utf-8")) + 3
    for row in range(labels.num_rows):
        a, b = int(offsets[row]), int(offsets[row + 1])
        written = b""
        for t in tokens[a:b]:
            written += token_bytes[int(t)] or b""
            if len(written) >= need:
                break
        out[row] = syntax.quoted(written)
    return out


MAX_COLUMNS = 8


def column_table(tokens: np.ndarray, offsets: np.ndarray) -> np.ndarray:
    """int32 [cols, rows]: each row's token at depth d (-1 past its end), for the first
    MAX_COLUMNS depths, so a search step over a row range reads one word."""
    offsets = np.asarray(offsets, dtype=np.int64)
    rows = len(offsets) - 1
    longest = int(np.diff(offsets).max()) if rows else 1
    cols = max(1, min(MAX_COLUMNS, longest))
    out = np.full((cols, max(rows, 0)), -1, dtype=np.int32)
    for d in range(cols):
        out[d] = _row_columns(np.asarray(tokens), offsets, d)
    return out


def first_token_starts(tokens: np.ndarray, offsets: np.ndarray, vocab: int) -> np.ndarray:
    """int32 [vocab + 1]: the first row whose first token is >= t (rows sorted, nonempty)."""
    offsets = np.asarray(offsets, dtype=np.int64)
    firsts = np.asarray(tokens)[offsets[:-1]] if len(offsets) > 1 else np.zeros(0, dtype=np.int64)
    return np.searchsorted(firsts, np.arange(vocab + 1), side="left").astype(np.int32)


def packed_delimiter_steps(delimiters: list[bytes | None], token_bytes) -> np.ndarray | None:
    """uint64 [vocab]: for every token, 4 bits per (delimiter, byte position) pair holding
    the position after the token when its bytes continue the delimiter there (0 if not);
    pairs are numbered delimiter by delimiter.  None when the pairs exceed 16 nibbles.
    A delimiter given as None (escapes off) is left out: the engine never asks for it."""
    total = sum(len(d) for d in delimiters if d is not None)
    if total > 16 or any(d is not None and len(d) > 15 for d in delimiters):
        return None
    out = np.zeros(len(token_bytes), dtype=np.uint64)
    for token, data in enumerate(token_bytes):
        if not data:
            continue
        word, offset = 0, 0
        for d in delimiters:
            if d is None:
                continue
            for pos in range(len(d)):
                if len(data) <= len(d) - pos and d.startswith(data, pos):
                    word |= (pos + len(data)) << (4 * (offset + pos))
            offset += len(d)
        out[token] = word
    return out


def _int32(name: str, array) -> np.ndarray:
    a = np.asarray(array)
    if a.size and (a.min() < -(2**31) or a.max() >= 2**31):
        raise ValueError(f"the {name} table does not fit int32")
    return np.ascontiguousarray(a, dtype=np.int32)


@dataclass
class PackedTables:
    blob: np.ndarray  # uint8
    layout: XgLayout
    words: int
    words_padded: int


def _relation_runs(index, entities: int, first_row: np.ndarray, ent_owner: np.ndarray) -> dict:
    """Per entity, its adjacency cut into runs of one relation (the edges are sorted by
    relation within an entity): `run_off` [entities + 1] CSR offsets, `runs` the (relation,
    first edge) pairs closed by (INT32_MAX, edges), `run_rel` their relations alone; and
    `edge_first`, the first label row of each edge's object with bit 31 set when the object
    entity has no triples.  A lookup of one relation's objects then scans an entity's runs,
    not its edges, and the next path frontier reads its keys without an owner hop."""
    offsets = np.asarray(index.adjacency_offsets, dtype=np.int64)
    rel = np.asarray(index.edge_relations, dtype=np.int32)
    obj = np.asarray(index.edge_objects, dtype=np.int64)
    edges = len(rel)
    degree = np.diff(offsets)
    subject = np.repeat(np.arange(len(degree), dtype=np.int64), degree)
    starts = np.ones(edges, dtype=bool)
    if edges:
        starts[1:] = (rel[1:] != rel[:-1]) | (subject[1:] != subject[:-1])
    run_start = np.flatnonzero(starts)
    run_off = np.zeros(len(degree) + 1, dtype=np.int64)
    np.cumsum(np.bincount(subject[run_start], minlength=len(degree)), out=run_off[1:])
    runs = np.empty((len(run_start) + 1, 2), dtype=np.int32)
    runs[:-1, 0] = rel[run_start]
    runs[:-1, 1] = _int32("run starts", run_start)
    runs[-1] = (np.iinfo(np.int32).max, _int32("edges", np.array([edges]))[0])
    if edges:
        owner = ent_owner.astype(np.int64)[obj]
        first = first_row[owner].astype(np.int64)
        if (first < 0).any():
            raise ValueError("an edge object has no label row")
        edge_first = (first | (np.where(degree[owner] == 0, 1, 0) << 31)).astype(np.uint32).view(np.int32)
    else:
        edge_first = np.zeros(0, np.int32)
    return {"run_off": _int32("run offsets", run_off), "runs": runs,
            "run_rel": np.ascontiguousarray(runs[:-1, 0]), "edge_first": edge_first}


def pack_tables(index, tokenizer, syntax, *, escapes: bool, versions=None,
                unquoted_starts: bool = False, eos_token_ids=()) -> PackedTables:
    vocab = tokenizer.vocab_size
    words = mask_words(vocab)
    wp = padded_words(vocab)
    token_bytes = [tokenizer.token_bytes(t) for t in range(vocab)]
    if any(b is not None and len(b) == 0 for b in token_bytes):
        raise ValueError("the served vocabulary holds a token with no bytes; the engine cannot mask it")
    special = tokenizer.special_ids
    labels, relations = index.labels, index.relations
    opener, closer = syntax.opener.encode("utf-8"), syntax.closer.encode("utf-8")
    separator, escape = syntax.separator.encode("utf-8"), syntax.escape.encode("utf-8")

    def padded(masks_bool: np.ndarray) -> np.ndarray:
        out = np.zeros((masks_bool.shape[0], wp), dtype=np.uint32)
        for i in range(masks_bool.shape[0]):
            out[i, :words] = pack_mask(masks_bool[i], words)
        return out

    free_next, free_ok = delimiter_automaton(opener, token_bytes, special, True)
    esc_next, esc_ok = delimiter_automaton(closer, token_bytes, special, False)
    ent_tok = _int32("label token", labels.tokens)
    ent_off = _int32("label offset", labels.offsets)
    ent_owner = _int32("label owner", labels.owners)
    entities = len(labels.owner_ids)
    owners64 = ent_owner.astype(np.int64)
    ent_rows = np.argsort(owners64, kind="stable").astype(np.int32)
    ent_rows_off = np.zeros(entities + 1, dtype=np.int64)
    np.cumsum(np.bincount(owners64, minlength=entities), out=ent_rows_off[1:])
    first_row = np.full(entities, -1, dtype=np.int32)
    has_rows = np.diff(ent_rows_off) > 0
    first_row[has_rows] = ent_rows[ent_rows_off[:-1][has_rows]]
    # rows no unbound subject names: quoted ones with unquoted starts, and always the
    # verdict entities' (src/xgraph/oracle.py:650-659)
    kept = None
    excluded = np.zeros(labels.num_rows, dtype=bool)
    if unquoted_starts:
        excluded |= quoted_rows(labels, token_bytes, syntax)
    if index.verdicts:
        verdict_positions = [labels.owner_ids.index(v) for v in index.verdicts.values()]
        excluded |= np.isin(np.asarray(labels.owners, dtype=np.int64), verdict_positions)
    if excluded.any():
        kept = ~excluded
    kept_prefix = None
    if kept is not None:
        kept_prefix = np.zeros(labels.num_rows + 1, dtype=np.int32)
        np.cumsum(kept, out=kept_prefix[1:])
    first_tokens = ent_tok[ent_off[:-1][np.diff(ent_off) > 0]] if labels.num_rows else np.zeros(0, np.int32)
    root = np.zeros(wp, dtype=np.uint32)
    if labels.num_rows:
        use = first_tokens if kept is None else first_tokens[kept]
        root[:words] = pack_mask(np.isin(np.arange(vocab), use), words)
    wide_keys, wide = wide_masks(ent_tok, ent_off.astype(np.int64), kept, wp)
    eos = np.zeros(wp, dtype=np.uint32)
    eos[:words] = pack_mask(np.isin(np.arange(vocab), list(eos_token_ids)), words)

    if versions is not None:
        ver_off = _int32("version offsets", versions.offsets)
        ver_subj = _int32("version subjects", versions.subjects)
        ver_adj = _int32("version adjacency", versions.adjacency)
        ver_rel = _int32("version relations", versions.edge_relations)
        ver_obj = _int32("version objects", versions.edge_objects)
        count = len(ver_off) - 1
    else:
        ver_off = np.zeros(1, np.int32)
        ver_subj = ver_rel = ver_obj = np.zeros(0, np.int32)
        ver_adj = np.zeros(1, np.int32)
        count = 0

    rel_tok = _int32("relation token", relations.tokens)
    rel_off = _int32("relation offset", relations.offsets)
    ent_col = column_table(ent_tok, ent_off)
    rel_col = column_table(rel_tok, rel_off)
    arrays: dict[str, np.ndarray] = {
        "ent_tok": ent_tok, "ent_off": ent_off, "ent_owner": ent_owner,
        "rel_tok": rel_tok, "rel_off": rel_off,
        "rel_owner": _int32("relation owner", relations.owners),
        "ent_col": ent_col, "rel_col": rel_col,
        "ent_first": first_token_starts(ent_tok, ent_off, vocab),
        "rel_first": first_token_starts(rel_tok, rel_off, vocab),
        "ent_first_row": first_row, "ent_rows_off": _int32("entity rows", ent_rows_off),
        "row_first": first_row[owners64] if labels.num_rows else np.zeros(0, np.int32),
        "row_degree": _int32("row degrees", np.diff(np.asarray(index.adjacency_offsets, dtype=np.int64))[owners64]
                             if labels.num_rows else np.zeros(0, np.int64)),
        "ent_rows": ent_rows,
        **_relation_runs(index, entities, first_row, ent_owner),
        "adj_off": _int32("adjacency offsets", index.adjacency_offsets),
        "edge_rel": _int32("edge relations", index.edge_relations),
        "edge_obj": _int32("edge objects", index.edge_objects),
        "root_mask": root,
        "free_next": np.ascontiguousarray(free_next), "free_mask": padded(free_ok),
        "esc_next": np.ascontiguousarray(esc_next), "esc_mask": padded(esc_ok),
        "eos_mask": eos,
        "ver_off": ver_off, "ver_subj": ver_subj, "ver_adj": ver_adj,
        "ver_edge_rel": ver_rel, "ver_edge_obj": ver_obj,
    }
    for name, delim in (("closer", closer), ("separator", separator), ("escape", escape)):
        off, tok, nxt = delimiter_lists(delim, token_bytes)
        if name == "escape" and not escapes:
            off, tok, nxt = np.zeros(len(delim) + 1, np.int32), np.zeros(0, np.int32), np.zeros(0, np.int32)
        arrays[f"{name}_off"], arrays[f"{name}_tok"], arrays[f"{name}_next"] = off, tok, nxt
    optional = {}
    dstep = packed_delimiter_steps([closer, separator, escape if escapes else None], token_bytes)
    if dstep is not None:
        optional["dstep"] = dstep
    if index.sitelinks is not None:
        optional["sitelinks"] = _int32("sitelinks", index.sitelinks)
        optional["row_sitelinks"] = optional["sitelinks"][owners64] if labels.num_rows else np.zeros(0, np.int32)
    if kept_prefix is not None:
        optional["kept_prefix"] = kept_prefix
    if len(wide_keys):
        optional["wide_keys"] = np.ascontiguousarray(wide_keys, dtype=np.int64)
        optional["wide_masks"] = np.ascontiguousarray(wide, dtype=np.uint32)

    layout = XgLayout()
    pieces: list[bytes] = []
    cursor = 0
    for name, array in list(arrays.items()) + list(optional.items()):
        data = np.ascontiguousarray(array).tobytes()
        setattr(layout, name, cursor)
        pieces.append(data)
        pad = (-len(data)) % ALIGN
        pieces.append(b"\0" * pad)
        cursor += len(data) + pad
    for name in ("sitelinks", "row_sitelinks", "kept_prefix", "wide_keys", "wide_masks", "dstep"):
        if name not in optional:
            setattr(layout, name, -1)
    blob = np.frombuffer(b"".join(pieces) or b"\0" * ALIGN, dtype=np.uint8).copy()
    layout.blob_bytes = len(blob)
    layout.vocab, layout.words, layout.words_padded = vocab, words, wp
    layout.entity_rows, layout.relation_rows = labels.num_rows, relations.num_rows
    layout.entities, layout.relations = entities, len(relations.owner_ids)
    layout.relation_words = (layout.relations + 31) // 32
    layout.opener_len, layout.closer_len = len(opener), len(closer)
    layout.separator_len, layout.escape_len = len(separator), len(escape)
    layout.versions = count
    layout.wide_count = len(wide_keys)
    layout.ent_cols, layout.rel_cols = ent_col.shape[0], rel_col.shape[0]
    return PackedTables(blob=blob, layout=layout, words=words, words_padded=wp)


def expression_tables(index, tokenizer, syntax):
    """The tables of expressions, as xg_set_expressions takes them: the packed delimiter
    lists (the operand separator's, then each offered operator's, written after the label
    prefix; per list its length, CSR offsets, tokens and next positions), the number of
    operators offered (the value comparison only with the verdict entities), their leading
    shared bytes [operators * operators], the date table (entity positions, keys) and the
    verdict entities' positions (yes, no) or None (src/xgraph/engine.py:345-360, 500-530)."""
    token_bytes = [tokenizer.token_bytes(t) for t in range(tokenizer.vocab_size)]
    offered = syntax.operators if index.verdicts else syntax.operators[:2]
    if not offered or not syntax.operand_separator:
        raise ValueError(f"expressions need a span syntax with operators and an operand separator, not {syntax}")
    if len(offered) > 4:
        raise ValueError("the engine holds at most 4 operators")
    written = [(syntax.label_prefix + op).encode("utf-8") for op in offered]
    parts = []
    for delimiter in [syntax.operand_separator.encode("utf-8"), *written]:
        if len(delimiter) > 64:
            raise ValueError(f"an expression delimiter of {len(delimiter)} bytes is longer than 64")
        off, tok, nxt = delimiter_lists(delimiter, token_bytes)
        parts += [np.array([len(delimiter)], dtype=np.int32), off, tok, nxt]
    delimiters = np.ascontiguousarray(np.concatenate(parts), dtype=np.int32)
    lcp = np.zeros((len(written), len(written)), dtype=np.int32)
    for k, a in enumerate(written):
        for j, b in enumerate(written):
            n = 0
            while n < min(len(a), len(b)) and a[n] == b[n]:
                n += 1
            lcp[k, j] = n
    entities = np.ascontiguousarray(index.date_entities, dtype=np.int32)
    keys = np.ascontiguousarray(index.date_keys, dtype=np.int32)
    verdicts = None
    if index.verdicts:
        ids = index.labels.owner_ids
        verdicts = np.array([ids.index(index.verdicts["yes"]), ids.index(index.verdicts["no"])], dtype=np.int32)
    return delimiters, len(written), np.ascontiguousarray(lcp.reshape(-1)), entities, keys, verdicts
