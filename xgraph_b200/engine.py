"""The GPU engine: per-slot constraint states, advanced and masked on the device.

Same API and error behaviour as the reference's `xgraph.engine.Engine`
(src/xgraph/engine.py:559-1069) for the policies it serves: `reset`, `begin`, `end`,
`anchor`, `set_version`, `open_span`, `advance`, `sync`, `fill_mask`, `mask`,
`mask_host`, `apply_mask`, `states_host`, `errors`, `view`, `max_sequences`; every
method takes `stream` (a raw cudaStream_t as int, 0 = default stream).  Underneath, each
call is one C-ABI function of libxgraph_b200.so (include/xgraph_b200.h) — hand-written
sm_100a kernels.  There is no fallback: without the built library the constructor
raises EngineUnavailable.

Tensor arguments are torch tensors (device memory, or pinned host memory where the
reference accepts it); host token arrays may also be numpy.
"""

from __future__ import annotations

import ctypes
import math
from collections.abc import Iterable
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .index import IndexMismatch, check_expressions, check_start_rank
from .tables import XgLayout, XgOptions, mask_words, pack_mask, pack_tables  # noqa: F401

PHASES = ("free text", "span", "escaped", "error")
PHASE_ERROR = PHASES.index("error")
SEGMENTS = ("subject", "relation", "object")
CLOSED = ("none", "unresolved", "entity span", "fact span", "path span", "comparison", "relation plan")
COMPARISONS = ("earlier", "later", "same")  # the comparison each operator writes, by position
MAX_FACTS = 64
MAX_REACHED = 64
MAX_DELIMITER_BYTES = 127
STATE_FIELDS = (
    "phase", "pos", "segment", "depth", "lo", "hi", "close_pos", "close_lo", "close_hi",
    "sep_pos", "sep_lo", "sep_hi", "esc_pos", "subj_lo", "subj_hi", "rel_lo", "rel_hi",
    "subj_key", "hops", "op_pos", "op_kind", "op", "operand", "answer_complete",
    "last_kind", "last_lo", "last_hi", "last_subj_lo", "last_subj_hi", "last_rel_lo",
    "last_rel_hi", "ex_hi", "flags", "stop_used_lo", "stop_used_hi",
)
"""Names of the leading int32 words of a slot state (XgState in include/xgraph_b200.h)."""
STATE_INTS = 64
LIBRARY = Path(__file__).resolve().parent / "libxgraph_b200.so"

XG_OK, XG_EINVAL, XG_ECUDA, XG_ENOMEM = 0, 1, 2, 3
ABI_VERSION = 4
"""XG_ABI_VERSION of include/xgraph_b200.h that these bindings follow."""
ADMISSION_INTS = 5 + MAX_REACHED
"""int32 words of one admission record (XgAdmission: slot, on, version, open_span,
anchor_count, 64 anchor rows)."""
DTYPES = {"float32": 0, "bfloat16": 1, "float16": 2}

# Reference constructor options this engine does not serve, with their neutral values.
_NOT_SERVED = {
    "observe": 0, "observe_width": 0,
    "observe_defer": 0, "menu_close_next": False, "observe_select": False,
    "observe_answer": False, "observe_required": False, "observe_no_loop": False,
    "audit": False, "audit_entities": 20, "audit_relations": 8, "menu": 0,
    "relation_labels": None, "observe_terminal": 0, "terminal_order": "identity",
    "terminal_seed": 17, "request_path_options": False,
}


class EngineUnavailable(RuntimeError):
    """The CUDA library of the engine was not built (run __graft_entry__.build())."""


class _Info(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("max_sequences", "vocab", "words", "words_padded", "memory_ints", "device")]


_lib = None


def load_library(path: Path = LIBRARY):
    """The engine's C ABI, loaded once; EngineUnavailable if it was never built."""
    global _lib
    if _lib is not None:
        return _lib
    if not path.is_file():
        raise EngineUnavailable(f"{path} is missing: build the CUDA engine first (__graft_entry__.build())")
    lib = ctypes.CDLL(str(path))
    p, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    sigs = {
        "xg_last_error": ([], ctypes.c_char_p),
        "xg_abi_version": ([], i32),
        "xg_create": ([p, ctypes.POINTER(XgLayout), ctypes.POINTER(XgOptions), i32, ctypes.POINTER(p)], ctypes.c_int),
        "xg_create_from_device": ([p, ctypes.POINTER(XgLayout), ctypes.POINTER(XgOptions), i32, ctypes.POINTER(p)], ctypes.c_int),
        "xg_destroy": ([p], ctypes.c_int),
        "xg_info": ([p, ctypes.POINTER(_Info)], ctypes.c_int),
        "xg_reset": ([p, p], ctypes.c_int),
        "xg_begin": ([p, p, i32, i32, p], ctypes.c_int),
        "xg_set_reached": ([p, i32, p, i32, p], ctypes.c_int),
        "xg_set_version": ([p, i32, i32, p], ctypes.c_int),
        "xg_open_span": ([p, i32, p], ctypes.c_int),
        "xg_advance": ([p, p, i32, i32, p], ctypes.c_int),
        "xg_sync": ([p, p, i32, p, i64, i64, p, p, i64, p], ctypes.c_int),
        "xg_fill_mask": ([p, i32, p], ctypes.c_int),
        "xg_mask_device": ([p, ctypes.POINTER(p)], ctypes.c_int),
        "xg_states_device": ([p, ctypes.POINTER(p)], ctypes.c_int),
        "xg_mask_host": ([p, i32, p], ctypes.c_int),
        "xg_states_host": ([p, i32, p], ctypes.c_int),
        "xg_memory_host": ([p, i32, p], ctypes.c_int),
        "xg_apply_mask": ([p, p, i32, i32, i32, i64, p, p, p, p], ctypes.c_int),
        "xg_sync_apply": ([p, p, i32, p, i64, i64, p, p, i64, p, i32, i32, i64, p], ctypes.c_int),
        "xg_sync_apply_admit": ([p, p, i32, p, i64, i64, p, p, i64, p, i32, i32, i64, p, i32, i32, p], ctypes.c_int),
        "xg_admit": ([p, p, i32, i32, p], ctypes.c_int),
        "xg_faults": ([p, ctypes.POINTER(i32)], ctypes.c_int),
        "xg_add_version": ([p, p, i32, p, p, p, p, ctypes.POINTER(i32)], ctypes.c_int),
        "xg_drop_version": ([p, i32, p], ctypes.c_int),
        "xg_build_adjacency": ([p, p, p, i64, p, p, i32, i32, p, i32, i64, p, p, p, p, p, p], ctypes.c_int),
        "xg_enable_stop": ([p, p, p, i64], ctypes.c_int),
        "xg_set_stop": ([p, i32, p, i32, p, i32, p, i32, p], ctypes.c_int),
        "xg_set_relation_successors": ([p, p, i32], ctypes.c_int),
        "xg_set_expressions": ([p, p, i64, i32, p, p, p, i32, p], ctypes.c_int),
        "xg_build_label_rows": ([i32, p, p, i64, p, p, i64, p, i32, i32, p, p, i64, p, p, p, p, p, p, p, p],
                                ctypes.c_int),
    }
    for name, (args, res) in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes, fn.restype = args, res
    if lib.xg_abi_version() != ABI_VERSION:
        raise EngineUnavailable(f"{path} has ABI {lib.xg_abi_version()}, expected {ABI_VERSION} (rebuild it)")
    _lib = lib
    return lib


def _check(rc: int) -> None:
    if rc == XG_OK:
        return
    message = _lib.xg_last_error().decode("utf-8", "replace")
    if rc == XG_EINVAL:
        raise ValueError(message)
    if rc == XG_ENOMEM:
        raise MemoryError(message)
    raise RuntimeError(message)


def _stream(stream) -> ctypes.c_void_p:
    return ctypes.c_void_p(int(stream) if stream else 0)


def _device_ptr(tensor, name: str, *, ndim: int | None = None, dtype=None):
    import torch

    if not isinstance(tensor, torch.Tensor):
        raise ValueError(f"{name} must be a torch tensor on the GPU")
    if ndim is not None and tensor.dim() != ndim:
        raise ValueError(f"{name} must have {ndim} dimensions")
    if dtype is not None and tensor.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}")
    if not tensor.is_cuda and not tensor.is_pinned():
        raise ValueError(f"{name} must be on the GPU or in pinned host memory")
    return ctypes.c_void_p(tensor.data_ptr())


class _CudaArray:
    """__cuda_array_interface__ holder so torch can view engine-owned device memory."""

    def __init__(self, ptr: int, shape, strides, owner) -> None:
        self.owner = owner  # keeps the engine (and its memory) alive while viewed
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "strides": tuple(strides), "typestr": "<i4",
            "data": (int(ptr), False), "version": 3,
        }


def _device_view(ptr: int, shape, strides, device: int, owner):
    import torch

    return torch.as_tensor(_CudaArray(ptr, shape, strides, owner), device=f"cuda:{device}")


class Engine:
    """Shared KG tables and independent constraint slots resident on the GPU.

    Construction validates the options in the reference's order
    (src/xgraph/engine.py:817-901), packs the index (tables.pack_tables) and copies it
    to the current CUDA device with `max_sequences` slots, all inactive.

    The logit policies act in apply_mask (and sync_apply, which includes it) inside spans,
    as the reference's (src/xgraph/engine.py:626-640): with release_mass > 0 a row whose
    logits put less than that share of their softmax (over the served vocabulary, at the
    logits' own temperature) on the allowed set, and with release_top a row whose own top
    token is disallowed, may write only the escape marker's next tokens; release is per
    call and leaves the slot's recorded mask alone.  escape_bias is added to the logits of
    the tokens that commit to the escape marker (16-bit logits hold the sum rounded to
    nearest).

    With expressions=True (committed paths, escapes, frontier support and an index with the
    date table, src/xgraph/engine.py:655-664) a span may be a date comparison
    `⟦ earlier: A | B · r⟧` (or `later:`), or with the index's verdict entities a value
    comparison `⟦ same: A | B · r⟧`; its result binds the answer span after it, and
    closed_span reads it back as a "comparison" record."""

    def __init__(
        self,
        index,
        tokenizer,
        syntax,
        max_sequences: int,
        *,
        escapes: bool = True,
        repeats: bool = True,
        release_mass: float = 0.0,
        release_top: bool = False,
        derivation: bool = False,
        escape_bias: float = 0.0,
        paths: bool = False,
        bound_escapes: bool = True,
        committed_paths: bool = False,
        versions=None,
        start_rank: str = "degree",
        unquoted_starts: bool = False,
        end_after_answer: bool = False,
        eos_token_ids: Iterable[int] = (),
        stop: str | None = None,
        relations: str = "frontier",
        expressions: bool = False,
        device_blob=None,
        **others,
    ) -> None:
        self._lib = load_library()
        if index.tokenizer_fingerprint != tokenizer.fingerprint:
            raise IndexMismatch(
                f"the KG index was built for tokenizer {index.tokenizer_fingerprint[:12]}, "
                f"not the served tokenizer {tokenizer.fingerprint[:12]}"
            )
        if index.span_syntax != syntax:
            raise IndexMismatch(f"the KG index was built for span syntax {index.span_syntax}, not {syntax}")
        if not (escapes or repeats):
            raise ValueError("repeats can only be switched off with escapes, the way out")
        if committed_paths and not paths:
            raise ValueError("committed_paths needs path mode (paths=True)")
        if end_after_answer and not paths:
            raise ValueError("end_after_answer needs path mode (paths=True)")
        eos = tokenizer.check_eos_token_ids(eos_token_ids) if end_after_answer else frozenset()
        for name, value in others.items():
            if name not in _NOT_SERVED:
                raise TypeError(f"Engine() got an unexpected keyword argument {name!r}")
            if value != _NOT_SERVED[name]:
                raise ValueError(f"the {name} policy is not served by this engine")
        if stop not in (None, "residual-goal"):
            raise ValueError(f"unknown STOP rule {stop!r}; expected residual-goal")
        if stop and not committed_paths:
            raise ValueError("residual-goal STOP needs committed paths (committed_paths=True)")
        # expressions (src/xgraph/engine.py:757-762)
        if expressions and not committed_paths:
            raise ValueError("expressions need committed paths (committed_paths=True)")
        if expressions and not escapes:
            raise ValueError("expressions need escapes, the way out of an operand or relation")
        if expressions:
            check_expressions(index)
        from .relations import RELATIONS, check_relations

        check_relations(relations, paths=paths, stop=stop, expressions=expressions)
        self._relations = relations
        sitelinks_rank = check_start_rank(start_rank, index) == "sitelinks"
        if not escapes and (release_mass > 0 or release_top):
            raise ValueError("release needs escapes: it releases to the escape marker")
        if not 0.0 <= release_mass < 1.0:
            raise ValueError(f"release_mass must be in [0, 1), got {release_mass}")
        if max_sequences < 1:
            raise ValueError(f"max_sequences must be at least 1, got {max_sequences}")
        for name in ("opener", "separator", "closer", "escape"):
            size = len(getattr(syntax, name).encode("utf-8"))
            if size > MAX_DELIMITER_BYTES:
                raise ValueError(
                    f"the span {name} is {size} bytes in UTF-8; the engine supports at most {MAX_DELIMITER_BYTES}"
                )
        if versions is not None:
            versions.check_base(index)
        self._index, self._versions = index, versions
        self._added: dict[str, tuple[int, object]] = {}  # versions registered while running: name -> (number, view data)
        self._builder = None
        self._entity_index: dict[str, int] | None = None
        self._tables = pack_tables(
            index, tokenizer, syntax, escapes=escapes, versions=versions,
            unquoted_starts=unquoted_starts, eos_token_ids=sorted(eos),
        ) if device_blob is None else device_blob[1]
        self._options = XgOptions(
            escapes=int(escapes), repeats=int(repeats), derivation=int(derivation or paths),
            paths=int(paths), bound_escapes=int(bound_escapes), committed_paths=int(committed_paths),
            sitelinks_rank=int(sitelinks_rank), end_after_answer=int(end_after_answer),
            release_top=int(bool(release_top)),
            release_log_mass=math.log(release_mass) if release_mass > 0 else -math.inf,
            escape_bias=float(escape_bias), relations=RELATIONS.index(relations),
            expressions=int(bool(expressions)),
        )
        handle = ctypes.c_void_p()
        if device_blob is None:
            blob = self._tables.blob
            rc = self._lib.xg_create(
                blob.ctypes.data_as(ctypes.c_void_p), ctypes.byref(self._tables.layout),
                ctypes.byref(self._options), int(max_sequences), ctypes.byref(handle))
        else:
            rc = self._lib.xg_create_from_device(
                ctypes.c_void_p(device_blob[0].data_ptr()), ctypes.byref(self._tables.layout),
                ctypes.byref(self._options), int(max_sequences), ctypes.byref(handle))
        _check(rc)
        self._handle = handle
        if expressions:
            from .tables import expression_tables

            delims, operators, lcp, entities, keys, verdicts = expression_tables(index, tokenizer, syntax)
            ptr = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
            _check(self._lib.xg_set_expressions(self._handle, ptr(delims), len(delims), operators, ptr(lcp),
                                                ptr(entities), ptr(keys), len(entities), ptr(verdicts)))
        if relations == "successor":
            from .relations import relation_successors

            tables = np.ascontiguousarray(relation_successors(index, versions), dtype=np.uint32)
            _check(self._lib.xg_set_relation_successors(self._handle, tables.ctypes.data_as(ctypes.c_void_p),
                                                        tables.shape[0]))
        self._stop_terms = None
        if stop:
            from .stopping import RelationTerms, label_word_table

            offsets, words = label_word_table(index, tokenizer)
            _check(self._lib.xg_enable_stop(self._handle, offsets.ctypes.data_as(ctypes.c_void_p),
                                            words.ctypes.data_as(ctypes.c_void_p), len(words)))
            self._stop_terms = RelationTerms.from_index(index, tokenizer)
        info = _Info()
        _check(self._lib.xg_info(self._handle, ctypes.byref(info)))
        self._info = info
        self.vocab_size = info.vocab
        self.words = info.words

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle and _lib is not None:
            _lib.xg_destroy(handle)
            self._handle = None

    @property
    def max_sequences(self) -> int:
        return self._info.max_sequences

    @property
    def layout(self) -> XgLayout:
        return self._tables.layout

    def reset(self, stream: int = 0) -> None:
        _check(self._lib.xg_reset(self._handle, _stream(stream)))

    def _slots(self, slots):
        import torch

        if not isinstance(slots, torch.Tensor) or not slots.is_cuda or slots.dtype != torch.int32 or slots.dim() != 1:
            raise ValueError("slots must be a 1-D int32 tensor on the GPU")
        if len(slots) > self.max_sequences:
            raise ValueError("more slots than max_sequences")
        return ctypes.c_void_p(slots.data_ptr()), len(slots)

    def begin(self, slots, stream: int = 0) -> None:
        ptr, n = self._slots(slots)
        _check(self._lib.xg_begin(self._handle, ptr, n, 1, _stream(stream)))

    def end(self, slots, stream: int = 0) -> None:
        ptr, n = self._slots(slots)
        _check(self._lib.xg_begin(self._handle, ptr, n, 0, _stream(stream)))

    def anchor(self, slot: int, entities: list[str], stream: int = 0) -> None:
        """Derivation/path mode: bind the slot's spans to these entities' label rows."""
        rows = self._anchor_rows(entities)
        _check(self._lib.xg_set_reached(self._handle, int(slot), rows.ctypes.data_as(ctypes.c_void_p),
                                        len(rows), _stream(stream)))

    def _anchor_rows(self, entities) -> np.ndarray:
        """The first 64 label rows (sorted) of these entities; ValueError when they have none."""
        labels = self._index.labels
        if self._entity_index is None:
            self._entity_index = {e: n for n, e in enumerate(labels.owner_ids)}
            owners = np.asarray(labels.owners, dtype=np.int64)
            self._rows_order = np.argsort(owners, kind="stable")
            self._rows_start = np.zeros(len(labels.owner_ids) + 1, dtype=np.int64)
            np.cumsum(np.bincount(owners, minlength=len(labels.owner_ids)), out=self._rows_start[1:])
        found = sorted(
            int(r)
            for e in dict.fromkeys(entities)
            if (n := self._entity_index.get(e)) is not None
            for r in self._rows_order[self._rows_start[n]: self._rows_start[n + 1]]
        )
        if not found:
            raise ValueError(f"anchor has no writable label rows: {entities!r}")
        return np.ascontiguousarray(found[:MAX_REACHED], dtype=np.int32)

    def _version_number(self, version: str | None) -> int:
        if version is None:
            return 0
        if version in self._added:
            return self._added[version][0]
        if self._versions is not None and version in self._versions.names:
            return self._versions.number(version)
        raise ValueError(f"no KG version {version!r}; the registered ones are {self.version_names()}")

    def version_names(self) -> list[str]:
        """Every KG version slots may select: those the engine was built with, then those
        added since (and not dropped)."""
        return [*(self._versions.names if self._versions is not None else ()), *self._added]

    def add_version(self, name: str, edits, stream: int = 0) -> int:
        """Register a KG version while the engine runs: the base with every edited (subject,
        relation) pair's objects replaced (the reference's pair-replacement edits,
        src/xgraph/kgversions.py:203-303), copied into the engine's device version arena on
        `stream` without rebuilding the shared tables.  Returns the version's number; slots
        then select it by name (set_version, Admission.version)."""
        from .kgversions import KGVersions, VersionBuilder

        if not isinstance(name, str) or not name:
            raise ValueError(f"a KG version needs a non-empty name, got {name!r}")
        if self._relations == "successor":
            raise ValueError("successor support reads the successor tables of the versions built in; "
                             "no version can be added while it runs")
        if name in self._added or (self._versions is not None and name in self._versions.names):
            raise ValueError(f"KG version {name!r} is registered already")
        if self._builder is None:
            self._builder = VersionBuilder(self._index)
        subjects, adjacency, relations, objects, stats = self._builder.overlay(name, edits)
        number = ctypes.c_int32()
        _check(self._lib.xg_add_version(
            self._handle, subjects.ctypes.data_as(ctypes.c_void_p), len(subjects),
            adjacency.ctypes.data_as(ctypes.c_void_p), relations.ctypes.data_as(ctypes.c_void_p),
            objects.ctypes.data_as(ctypes.c_void_p), _stream(stream), ctypes.byref(number)))
        single = KGVersions(names=(name,), stats=(stats,), offsets=np.array([0, len(subjects)], dtype=np.int64),
                            subjects=subjects, adjacency=adjacency, edge_relations=relations,
                            edge_objects=objects, base_fingerprint=self._index.base_fingerprint)
        self._added[name] = (int(number.value), single)
        return int(number.value)

    def drop_version(self, name: str, stream: int = 0) -> None:
        """Forget a version added with add_version (its number is reused later); slots still
        selecting it read the base KG from the next step on."""
        if name not in self._added:
            raise ValueError(f"no KG version {name!r} was added to this engine")
        _check(self._lib.xg_drop_version(self._handle, self._added[name][0], _stream(stream)))
        del self._added[name]

    def admission_records(self, admissions: Iterable[Admission]) -> np.ndarray:
        """XgAdmission records [n, ADMISSION_INTS] int32 for these admissions (anchor
        entities to label rows, version names to numbers), checked as the single calls check
        them; a device copy of the result can be handed to `admit` / `sync_apply` directly."""
        admissions = list(admissions)
        out = np.zeros((len(admissions), ADMISSION_INTS), dtype=np.int32)
        for k, a in enumerate(admissions):
            if not 0 <= int(a.slot) < self.max_sequences:
                raise ValueError(f"slot must be between 0 and max_sequences - 1, got {a.slot}")
            out[k, 0], out[k, 1] = int(a.slot), int(bool(a.on))
            if a.on:
                out[k, 2] = self._version_number(a.version)
                out[k, 3] = int(bool(a.open_span))
                if a.anchors:
                    rows = self._anchor_rows(a.anchors)
                    out[k, 4] = len(rows)
                    out[k, 5: 5 + len(rows)] = rows
        if len(set(out[:, 0].tolist())) != len(out):
            raise ValueError("two admissions name the same slot")
        return out

    def _admission_args(self, admissions):
        """(pointer, count, on_host, keep-alive) of admissions given as Admission objects, a
        host record array or a device int32 tensor of records."""
        import torch

        if admissions is None:
            return ctypes.c_void_p(0), 0, 0, None
        if isinstance(admissions, torch.Tensor):
            if (not admissions.is_cuda or admissions.dtype != torch.int32 or admissions.dim() != 2
                    or admissions.shape[1] != ADMISSION_INTS or not admissions.is_contiguous()):
                raise ValueError(f"device admissions must be a contiguous int32 [n, {ADMISSION_INTS}] GPU tensor")
            return ctypes.c_void_p(admissions.data_ptr()), admissions.shape[0], 0, admissions
        records = admissions if isinstance(admissions, np.ndarray) else self.admission_records(admissions)
        records = np.ascontiguousarray(records, dtype=np.int32)
        if records.ndim != 2 or records.shape[1] != ADMISSION_INTS:
            raise ValueError(f"admission records must be int32 [n, {ADMISSION_INTS}]")
        return records.ctypes.data_as(ctypes.c_void_p), records.shape[0], 1, records

    def admit(self, admissions, stream: int = 0) -> None:
        """Apply a batch of admissions (Admission objects, their records, or a device record
        tensor) in one kernel launch; each admitted slot's mask is rebuilt."""
        ptr, n, on_host, keep = self._admission_args(admissions)
        _check(self._lib.xg_admit(self._handle, ptr, n, on_host, _stream(stream)))
        del keep

    def faults(self) -> int:
        """Device-side faults since the last call (waits; value 2: a device admission out of
        range was skipped; value 4: a row the fused step wrote early left its relation
        segment, never expected); 0 normally."""
        out = ctypes.c_int32()
        _check(self._lib.xg_faults(self._handle, ctypes.byref(out)))
        return int(out.value)

    def set_version(self, slot: int, version: str | None, stream: int = 0) -> None:
        number = self._version_number(version)
        _check(self._lib.xg_set_version(self._handle, int(slot), number, _stream(stream)))

    def set_stop(self, slot: int, question: str, stream: int = 0) -> None:
        """Residual-goal STOP (src/xgraph/engine.py:946-967): compile this request's STOP
        relations from its question, after begin and before sync / open_span; the slot's
        next begin clears them; draft rows read them in place."""
        if self._stop_terms is None:
            raise ValueError("set_stop needs stop='residual-goal'")
        goal = self._stop_terms.for_question(question)
        relations, offsets, words = goal.arrays(len(self._index.relations.owner_ids))
        count = int(offsets[0])
        word_offsets = np.ascontiguousarray(offsets[1: count + 2], dtype=np.int32)
        buffer = np.frombuffer(words, dtype=np.uint8) if words else np.zeros(1, dtype=np.uint8)
        _check(self._lib.xg_set_stop(
            self._handle, int(slot), relations.ctypes.data_as(ctypes.c_void_p), relations.shape[0],
            buffer.ctypes.data_as(ctypes.c_void_p), len(words), word_offsets.ctypes.data_as(ctypes.c_void_p),
            len(word_offsets), _stream(stream)))

    def open_span(self, slot: int, stream: int = 0) -> None:
        _check(self._lib.xg_open_span(self._handle, int(slot), _stream(stream)))

    def view(self, version: str | None):
        if version is None:
            return self._index
        if version in self._added:
            return self._added[version][1].view(self._index, version)
        if self._versions is None or version not in self._versions.names:
            raise ValueError(f"no KG version {version!r}; the registered ones are {self.version_names()}")
        return self._versions.view(self._index, version)

    def advance(self, tokens, stream: int = 0) -> None:
        """Advance slots 0..len(tokens)-1 by these tokens (1-D int32, on the GPU or host)."""
        try:
            import torch
        except ImportError:  # pragma: no cover
            torch = None
        if torch is not None and isinstance(tokens, torch.Tensor):
            if tokens.dtype != torch.int32 or tokens.dim() != 1:
                raise ValueError("tokens must be a 1-D int32 array")
            if tokens.is_cuda:
                _check(self._lib.xg_advance(self._handle, ctypes.c_void_p(tokens.data_ptr()), len(tokens), 0,
                                            _stream(stream)))
                return
            tokens = tokens.numpy()
        host = np.ascontiguousarray(tokens, dtype=np.int32)
        if host.ndim != 1:
            raise ValueError("tokens must be a 1-D int32 array")
        _check(self._lib.xg_advance(self._handle, host.ctypes.data_as(ctypes.c_void_p), len(host), 1,
                                    _stream(stream)))

    def fill_mask(self, sequences: int | None = None, stream: int = 0) -> None:
        _check(self._lib.xg_fill_mask(self._handle, self._count(sequences), _stream(stream)))

    def sync(self, slots, history, prompt_len, total_len, stream: int = 0) -> None:
        import torch

        ptr, n = self._slots(slots)
        for name, lengths in (("prompt_len", prompt_len), ("total_len", total_len)):
            _device_ptr(lengths, name, ndim=1, dtype=torch.int32)
            if len(lengths) < self.max_sequences:
                raise ValueError("prompt_len and total_len need one entry per slot")
        _device_ptr(history, "history", ndim=2, dtype=torch.int32)
        if history.shape[0] < self.max_sequences or history.stride(1) != 1:
            raise ValueError("history needs one contiguous row per slot")
        _check(self._lib.xg_sync(
            self._handle, ptr, n, ctypes.c_void_p(history.data_ptr()), history.stride(0), history.shape[0],
            ctypes.c_void_p(prompt_len.data_ptr()), ctypes.c_void_p(total_len.data_ptr()),
            min(len(prompt_len), len(total_len)), _stream(stream)))

    def sync_apply(self, slots, history, prompt_len, total_len, logits, stream: int = 0, *, admissions=None) -> None:
        """`sync` then `apply_mask(logits, slots)` in one kernel launch, for a step without
        speculative draft rows (logits row i belongs to slots[i]); `admissions` (as for
        `admit`) are applied first in the same launch."""
        import torch

        ptr, n = self._slots(slots)
        for name, lengths in (("prompt_len", prompt_len), ("total_len", total_len)):
            _device_ptr(lengths, name, ndim=1, dtype=torch.int32)
            if len(lengths) < self.max_sequences:
                raise ValueError("prompt_len and total_len need one entry per slot")
        _device_ptr(history, "history", ndim=2, dtype=torch.int32)
        if history.shape[0] < self.max_sequences or history.stride(1) != 1:
            raise ValueError("history needs one contiguous row per slot")
        if not isinstance(logits, torch.Tensor) or not logits.is_cuda or logits.dim() != 2:
            raise ValueError("logits must be a 2-D tensor on the GPU")
        dtype = DTYPES.get(str(logits.dtype).removeprefix("torch."))
        if dtype is None:
            raise ValueError("logits must be float32, bfloat16 or float16")
        if logits.shape[0] != n or (logits.shape[1] > 1 and logits.stride(1) != 1):
            raise ValueError("logits need one contiguous row per entry of slots")
        aptr, an, on_host, keep = self._admission_args(admissions)
        _check(self._lib.xg_sync_apply_admit(
            self._handle, ptr, n, ctypes.c_void_p(history.data_ptr()), history.stride(0), history.shape[0],
            ctypes.c_void_p(prompt_len.data_ptr()), ctypes.c_void_p(total_len.data_ptr()),
            min(len(prompt_len), len(total_len)), ctypes.c_void_p(logits.data_ptr()), dtype, logits.shape[1],
            logits.stride(0) if n > 1 else logits.shape[1], aptr, an, on_host, _stream(stream)))
        del keep

    def apply_mask(self, logits, row_slots, stream: int = 0, *, local_pos=None, input_ids=None) -> None:
        """Set every logit its slot's mask disallows (and every column past the served
        vocabulary) to -inf, in place; rows of inactive slots and error rows are untouched.

        Under speculative decoding a request owns consecutive rows, one per draft position
        (src/xgraph/engine.py:1012-1031): local_pos[i] is row i's offset among its
        request's rows and input_ids[i] the token fed at row i (the last committed token at
        offset 0, then the drafts).  Row i is masked as if the tokens fed at its request's
        earlier rows after the first had been committed; the slot's state does not move.
        A row whose drafts leave the language (the error phase), or whose offset reaches
        before row 0, is left untouched."""
        import torch

        if (local_pos is None) != (input_ids is None):
            raise ValueError("local_pos and input_ids go together")
        if not isinstance(logits, torch.Tensor) or not logits.is_cuda or logits.dim() != 2:
            raise ValueError("logits must be a 2-D tensor on the GPU")
        dtype = DTYPES.get(str(logits.dtype).removeprefix("torch."))
        if dtype is None:
            raise ValueError("logits must be float32, bfloat16 or float16")
        ptr, n = self._row_slots(row_slots)
        if logits.shape[0] != n or (logits.shape[1] > 1 and logits.stride(1) != 1):
            raise ValueError("logits need one contiguous row per entry of row_slots")
        drafts = (ctypes.c_void_p(0), ctypes.c_void_p(0))
        if local_pos is not None:
            pos_ptr, pos_n = self._row_slots(local_pos, "local_pos")
            ids_ptr, ids_n = self._row_slots(input_ids, "input_ids")
            if pos_n != n or ids_n != n:
                raise ValueError("local_pos and input_ids need one entry per logits row")
            drafts = (pos_ptr, ids_ptr)
        _check(self._lib.xg_apply_mask(
            self._handle, ctypes.c_void_p(logits.data_ptr()), dtype, n, logits.shape[1],
            logits.stride(0) if n > 1 else logits.shape[1], ptr, drafts[0], drafts[1], _stream(stream)))

    def _row_slots(self, row_slots, name="row_slots"):
        import torch

        if (not isinstance(row_slots, torch.Tensor) or not row_slots.is_cuda
                or row_slots.dtype != torch.int32 or row_slots.dim() != 1 or not row_slots.is_contiguous()):
            raise ValueError(f"{name} must be a contiguous 1-D int32 tensor on the GPU")
        return ctypes.c_void_p(row_slots.data_ptr()), len(row_slots)

    @property
    def mask(self):
        """The mask buffer on the GPU, [max_sequences, words] int32 (a zero-copy view;
        fill_mask writes it)."""
        return self.mask_view()[:, : self.words]

    def mask_view(self):
        """Zero-copy torch view of the mask buffer, [max_sequences, words_padded] int32."""
        ptr = ctypes.c_void_p()
        _check(self._lib.xg_mask_device(self._handle, ctypes.byref(ptr)))
        wp = self._info.words_padded
        return _device_view(ptr.value, (self.max_sequences, wp), (wp * 4, 4), self._info.device, self)

    def states_view(self):
        """Zero-copy torch view of the device states, [max_sequences, 64] int32 (read-only use)."""
        ptr = ctypes.c_void_p()
        _check(self._lib.xg_states_device(self._handle, ctypes.byref(ptr)))
        return _device_view(ptr.value, (self.max_sequences, STATE_INTS), (STATE_INTS * 4, 4), self._info.device, self)

    def mask_host(self, sequences: int | None = None) -> np.ndarray:
        n = self._count(sequences)
        out = np.zeros((n, self.words), dtype=np.uint32)
        _check(self._lib.xg_mask_host(self._handle, n, out.ctypes.data_as(ctypes.c_void_p)))
        return out.view(np.int32)

    def states_host(self, sequences: int | None = None) -> dict[str, np.ndarray]:
        n = self._count(sequences)
        raw = np.zeros((n, STATE_INTS), dtype=np.int32)
        _check(self._lib.xg_states_host(self._handle, n, raw.ctypes.data_as(ctypes.c_void_p)))
        return {name: raw[:, i].copy() for i, name in enumerate(STATE_FIELDS)}

    def memory_host(self, sequences: int | None = None) -> np.ndarray:
        n = self._count(sequences)
        out = np.zeros((n, self._info.memory_ints), dtype=np.int32)
        _check(self._lib.xg_memory_host(self._handle, n, out.ctypes.data_as(ctypes.c_void_p)))
        return out

    def errors(self, sequences: int | None = None) -> int:
        return int(np.count_nonzero(self.states_host(sequences)["phase"] == PHASE_ERROR))

    def _count(self, sequences: int | None) -> int:
        n = self.max_sequences if sequences is None else int(sequences)
        if not 0 <= n <= self.max_sequences:
            raise ValueError(f"sequences must be between 0 and max_sequences ({self.max_sequences}), got {n}")
        return n


@dataclass(frozen=True)
class Admission:
    """One request joining (on=True) or leaving (on=False) a slot between steps, applied in
    the reference adapter's order (src/xgraph/vllm.py:569-605): begin or end, then the
    anchor entities (derivation / path mode), then the KG version by name (None = base),
    then open_span."""

    slot: int
    on: bool = True
    anchors: tuple[str, ...] = ()
    version: str | None = None
    open_span: bool = False


@dataclass(frozen=True)
class ClosedSpanRecord:
    kind: str
    entity_ids: tuple[str, ...] = ()
    triples: tuple[tuple[str, str, str], ...] = ()
    operator: str = ""
    operands: tuple[str, ...] = ()

    @property
    def resolved(self) -> bool:
        return self.kind in ("entity span", "fact span", "path span", "comparison")


def closed_span(index, states: dict[str, np.ndarray], seq: int) -> ClosedSpanRecord:
    """A slot's last closed span as KG ids, from the rows its state records
    (src/xgraph/engine.py:1091-1136).  For a slot reading a KG version, index is the
    version's view (Engine.view)."""
    kind = CLOSED[int(states["last_kind"][seq])]
    lo, hi = int(states["last_lo"][seq]), int(states["last_hi"][seq])
    if kind == "comparison":  # lo, hi: the operands' start rows; subj_lo the result, subj_hi the operator
        from .dates import VERDICTS

        operands = (index.labels.owner_id(lo), index.labels.owner_id(hi))
        result, operator = int(states["last_subj_lo"][seq]), int(states["last_subj_hi"][seq])
        if result >= 3:  # a value comparison's verdict: 3 yes, 4 no
            chosen = (VERDICTS["yes" if result == 3 else "no"],)
        else:  # a date comparison's operand: 0 A's, 1 B's, 2 both
            chosen = operands if result == 2 else operands[result: result + 1]
        return ClosedSpanRecord(kind, tuple(sorted(set(chosen))), (), COMPARISONS[operator - 1], operands)
    if kind == "entity span":
        owners = {index.labels.owner_id(r) for r in range(lo, hi)}
        if int(states["last_subj_lo"][seq]) == -1:  # an unbound span names no verdict entity
            from .dates import VERDICTS

            owners -= set(VERDICTS.values())
        return ClosedSpanRecord(kind, tuple(sorted(owners)))
    if kind != "fact span":
        return ClosedSpanRecord(kind)
    subjects = {index.labels.owner_id(r) for r in range(int(states["last_subj_lo"][seq]), int(states["last_subj_hi"][seq]))}
    relations = {index.relations.owner_id(r) for r in range(int(states["last_rel_lo"][seq]), int(states["last_rel_hi"][seq]))}
    triples = {
        (s, r, index.labels.owner_id(row))
        for s in subjects
        for r in relations
        for row in index.object_rows(s, r, lo, hi)
    }
    return ClosedSpanRecord(kind, (), tuple(sorted(triples)))
