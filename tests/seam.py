"""The host test seam: the engine's per-row logic (xgraph_b200/csrc/core.cuh) built with
g++ as a sequential library (seam.cpp), driven through ctypes.  Test infrastructure: it
checks the kernels' logic against the oracle on the CPU; the product never loads it."""

from __future__ import annotations

import ctypes
import subprocess
from functools import cache
from pathlib import Path

import numpy as np

from xgraph_b200.engine import STATE_FIELDS, STATE_INTS
from xgraph_b200.relations import RELATIONS, relation_successors
from xgraph_b200.tables import XgLayout, XgOptions, pack_tables

ROOT = Path(__file__).resolve().parents[1]
SOURCE = ROOT / "xgraph_b200" / "csrc" / "seam.cpp"
BUILT = ROOT / "tests" / "_seam" / "libxgseam.so"


@cache
def library():
    BUILT.parent.mkdir(exist_ok=True)
    sources = [SOURCE, SOURCE.with_name("core.cuh"), ROOT / "include" / "xgraph_b200.h"]
    if not BUILT.exists() or BUILT.stat().st_mtime < max(p.stat().st_mtime for p in sources):
        subprocess.run(["g++", "-std=c++17", "-O2", "-g", "-fPIC", "-shared", "-o", str(BUILT), str(SOURCE)], check=True)
    lib = ctypes.CDLL(str(BUILT))
    p, i32 = ctypes.c_void_p, ctypes.c_int32
    lib.xgs_create.argtypes = [p, ctypes.POINTER(XgLayout), ctypes.POINTER(XgOptions), i32]
    lib.xgs_create.restype = p
    for name, args in {
        "xgs_destroy": [p], "xgs_begin": [p, i32, i32], "xgs_set_version": [p, i32, i32],
        "xgs_set_reached": [p, i32, p, i32], "xgs_open_span": [p, i32], "xgs_advance": [p, p, i32],
        "xgs_masks": [p, i32, p], "xgs_states": [p, i32, p], "xgs_memory": [p, i32, p],
        "xgs_set_successors": [p, p, i32], "xgs_advance_slot": [p, i32, i32],
    }.items():
        getattr(lib, name).argtypes = args
        getattr(lib, name).restype = None
    lib.xgs_memory_ints.argtypes = [p]
    lib.xgs_memory_ints.restype = i32
    lib.xgs_relation_slice.argtypes = [p, i32, i32, i32, p]
    lib.xgs_relation_slice.restype = None
    lib.xgs_escape_policy.argtypes = [p, i32, p, p, p, p, i32]
    lib.xgs_escape_policy.restype = i32
    lib.xgs_enable_stop.argtypes = [p, p, p, ctypes.c_int64]
    lib.xgs_enable_stop.restype = None
    lib.xgs_set_stop.argtypes = [p, i32, p, p, i32, p, i32]
    lib.xgs_set_stop.restype = None
    lib.xgs_set_expressions.argtypes = [p, p, ctypes.c_int64, i32, p, p, p, i32, p]
    lib.xgs_set_expressions.restype = i32
    return lib


class SeamEngine:
    """Engine-shaped driver of the seam (slots 0..n-1)."""

    def __init__(self, index, tokenizer, syntax, slots, *, versions=None, escapes=True, repeats=True,
                 derivation=False, paths=False, bound_escapes=True, committed_paths=False,
                 start_rank="degree", unquoted_starts=False, end_after_answer=False, eos_token_ids=(),
                 relations="frontier", expressions=False):
        self.lib = library()
        self.index, self.versions = index, versions
        self.tables = pack_tables(index, tokenizer, syntax, escapes=escapes, versions=versions,
                                  unquoted_starts=unquoted_starts,
                                  eos_token_ids=sorted(eos_token_ids) if end_after_answer else ())
        self.options = XgOptions(escapes=int(escapes), repeats=int(repeats), derivation=int(derivation or paths),
                                 paths=int(paths), bound_escapes=int(bound_escapes),
                                 committed_paths=int(committed_paths),
                                 sitelinks_rank=int(start_rank == "sitelinks"),
                                 end_after_answer=int(end_after_answer), release_log_mass=-np.inf,
                                 relations=RELATIONS.index(relations), expressions=int(expressions))
        self.slots = slots
        self.handle = self.lib.xgs_create(self.tables.blob.ctypes.data_as(ctypes.c_void_p),
                                          ctypes.byref(self.tables.layout), ctypes.byref(self.options), slots)
        if expressions:
            from xgraph_b200.tables import expression_tables

            self._expr = expression_tables(index, tokenizer, syntax)
            delims, operators, lcp, entities, keys, verdicts = self._expr
            ptr = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
            assert self.lib.xgs_set_expressions(self.handle, ptr(delims), len(delims), operators, ptr(lcp),
                                                ptr(entities), ptr(keys), len(entities), ptr(verdicts)) == 0
        if relations == "successor":
            self._successors = np.ascontiguousarray(relation_successors(index, versions), dtype=np.uint32)
            self.lib.xgs_set_successors(self.handle, self._successors.ctypes.data_as(ctypes.c_void_p),
                                        self._successors.shape[0])

    def __del__(self):
        if getattr(self, "handle", None):
            self.lib.xgs_destroy(self.handle)

    def escape_policy(self, slot, cap=4096):
        """(escape position or -1, tokens that commit the slot to the escape marker, the
        escape marker's next tokens from that position) as the kernels compute them."""
        commits, released = np.zeros(cap, dtype=np.int32), np.zeros(cap, dtype=np.int32)
        counts = np.zeros(2, dtype=np.int32)
        pos = self.lib.xgs_escape_policy(
            self.handle, slot, commits.ctypes.data_as(ctypes.c_void_p), counts[0:].ctypes.data_as(ctypes.c_void_p),
            released.ctypes.data_as(ctypes.c_void_p), counts[1:].ctypes.data_as(ctypes.c_void_p), cap)
        assert counts.max() <= cap
        return int(pos), set(commits[: counts[0]].tolist()), set(released[: counts[1]].tolist())

    def enable_stop(self, tokenizer):
        """Residual-goal STOP with the index's label words (as Engine(stop=...) does)."""
        from xgraph_b200.stopping import RelationTerms, label_word_table

        self._stop_offsets, self._stop_words = label_word_table(self.index, tokenizer)
        self.lib.xgs_enable_stop(self.handle, self._stop_offsets.ctypes.data_as(ctypes.c_void_p),
                                 self._stop_words.ctypes.data_as(ctypes.c_void_p), len(self._stop_words))
        self._stop_terms = RelationTerms.from_index(self.index, tokenizer)

    def set_stop(self, slot, question):
        goal = self._stop_terms.for_question(question)
        relations, offsets, words = goal.arrays(len(self.index.relations.owner_ids))
        count = int(offsets[0])
        word_offsets = np.ascontiguousarray(offsets[1: count + 2], dtype=np.int32)
        buffer = np.frombuffer(words, dtype=np.uint8) if words else np.zeros(1, dtype=np.uint8)
        self.lib.xgs_set_stop(self.handle, slot, relations.ctypes.data_as(ctypes.c_void_p),
                              buffer.ctypes.data_as(ctypes.c_void_p), len(words),
                              word_offsets.ctypes.data_as(ctypes.c_void_p), len(word_offsets))

    def relation_slice(self, entity, relation, version=0):
        out = np.zeros(3, dtype=np.int32)
        self.lib.xgs_relation_slice(self.handle, version, entity, relation, out.ctypes.data_as(ctypes.c_void_p))
        return int(out[0]), int(out[1]), int(out[2])

    def begin(self, slot):
        self.lib.xgs_begin(self.handle, slot, 1)

    def set_version(self, slot, name):
        self.lib.xgs_set_version(self.handle, slot, 0 if name is None else self.versions.number(name))

    def anchor(self, slot, entities):
        labels = self.index.labels
        rows = sorted(r for r in range(labels.num_rows) if labels.owner_id(r) in set(entities))
        arr = np.ascontiguousarray(rows[:64], dtype=np.int32)
        self.lib.xgs_set_reached(self.handle, slot, arr.ctypes.data_as(ctypes.c_void_p), len(arr))

    def open_span(self, slot):
        self.lib.xgs_open_span(self.handle, slot)

    def advance(self, tokens):
        arr = np.ascontiguousarray(tokens, dtype=np.int32)
        self.lib.xgs_advance(self.handle, arr.ctypes.data_as(ctypes.c_void_p), len(arr))

    def advance_slot(self, slot, token):
        self.lib.xgs_advance_slot(self.handle, int(slot), int(token))

    def memory(self):
        out = np.zeros((self.slots, self.lib.xgs_memory_ints(self.handle)), dtype=np.int32)
        self.lib.xgs_memory(self.handle, self.slots, out.ctypes.data_as(ctypes.c_void_p))
        return out

    def masks(self):
        out = np.zeros((self.slots, self.tables.words), dtype=np.uint32)
        self.lib.xgs_masks(self.handle, self.slots, out.ctypes.data_as(ctypes.c_void_p))
        return out

    def states(self):
        raw = np.zeros((self.slots, STATE_INTS), dtype=np.int32)
        self.lib.xgs_states(self.handle, self.slots, raw.ctypes.data_as(ctypes.c_void_p))
        return {name: raw[:, i].copy() for i, name in enumerate(STATE_FIELDS)}

    def view(self, version):
        return self.index if version is None else self.versions.view(self.index, version)

    # Engine-shaped surface used by xgraph_b200.synthetic.sample_streams (device="cpu").
    @property
    def words(self):
        return self.tables.words

    def reset(self):
        for slot in range(self.slots):
            self.lib.xgs_begin(self.handle, slot, 0)

    def fill_mask(self, n=None):
        import torch

        self._mask[:] = torch.from_numpy(self.masks().view(np.int32))
        raw = np.zeros((self.slots, 64), dtype=np.int32)
        self.lib.xgs_states(self.handle, self.slots, raw.ctypes.data_as(ctypes.c_void_p))
        self._states[:] = torch.from_numpy(raw)

    def mask_view(self):
        import torch

        if not hasattr(self, "_mask"):
            self._mask = torch.zeros((self.slots, self.tables.words), dtype=torch.int32)
            self._states = torch.zeros((self.slots, 64), dtype=torch.int32)
        return self._mask

    def states_view(self):
        self.mask_view()
        return self._states

    def begin_all(self, slots):
        for slot in slots.tolist():
            self.begin(int(slot))

    def errors(self, n=None):
        return int((self.states()["phase"][: n or self.slots] == 3).sum())
