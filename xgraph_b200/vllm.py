"""The engine in vLLM, as a Model Runner V2 logits processor (the reference's
src/xgraph/vllm.py, restated for this engine's served policies).

    XGRAPH_KG_INDEX=<index saved by xgraph_b200.index.save_kg_index> \\
    XGRAPH_TOKENIZER=<the model's tokenizer.json> \\
        vllm serve <model> --logits-processors xgraph_b200.vllm:XGraphLogitsProcessor

A request opts in with the per-request argument `xgraph` set to 1 (offline
`extra_args={"xgraph": 1}`, online `extra_body={"vllm_xargs": {"xgraph": 1}}`); other
requests are left alone.  One engine slot follows each of vLLM's request slots: vLLM keeps
every slot's token history on the GPU, and before each sampling step the engine advances
each opted-in slot over the tokens committed since the last step (from the end of the
prompt the first time, so a request resumed after preemption replays its output) and sets
every logit the slot's mask disallows to -inf, in place.  Without speculative drafts both
happen in one kernel launch (Engine.sync_apply); under speculative decoding each draft row
is masked as if the drafts before it had been committed (Engine.apply_mask's draft rows).

vLLM has no hook for a finished request; a slot is reset when its next request is added.

Per-request arguments, as in the reference: `xgraph_anchor` (entity ids where derivation
mode starts), `xgraph_kg_version` (a version of XGRAPH_KG_VERSIONS, a file written by
xgraph_b200.kgversions.write_kg_versions), `xgraph_open` (the prompt ends with the span
opener; the slot starts inside a span), `xgraph_prefill` (the prompt ends with this text,
which the engine replays as if the model had written it; a prompt whose last tokens do not
end with the text's bytes, or a replayed token the mask disallows, declines the request,
which is then left unmasked), `xgraph_replay_id` (the key under which a replay's outcome is
kept for `replay_statuses`).  Engine settings: XGRAPH_ESCAPES, XGRAPH_REPEATS,
XGRAPH_DERIVATION, XGRAPH_PATHS, XGRAPH_BOUND_ESCAPES, XGRAPH_COMMITTED_PATHS,
XGRAPH_START_RANK, XGRAPH_UNQUOTED_STARTS, XGRAPH_END_AFTER_ANSWER.  The reference's
research policies (release, escape bias, STOP, expressions, observations, menus, audit,
relation supports, per-request path options) are not served by this engine: a setting or
argument that asks for one is refused with a ValueError naming it.

This module imports only the standard library at import time: vLLM also calls
validate_params in its frontend process.
"""

from __future__ import annotations

import os
import sys
from typing import Any

try:
    from vllm.v1.worker.gpu.sample.logits_processor import LogitsProcessor as _Base
except ImportError:  # no vLLM of that API: the class still works with stand-ins
    _Base = object  # type: ignore[assignment,misc]

OPT_IN = "xgraph"
ANCHOR = "xgraph_anchor"
"""Per-request argument: the question's entity ids, where derivation mode starts."""
KG_VERSION = "xgraph_kg_version"
"""Per-request argument: the name of the KG version the request reads (XGRAPH_KG_VERSIONS)."""
VERSIONS = "XGRAPH_KG_VERSIONS"
OPEN = "xgraph_open"
"""Per-request argument: 1 starts the request inside a span (its prompt ends with the opener)."""
PREFILL = "xgraph_prefill"
"""Per-request argument: the text the prompt ends with, which the engine replays."""
REPLAY_ID = "xgraph_replay_id"
"""Per-request argument: the caller's key for the replay's outcome."""
QUESTION = "xgraph_question"
"""Per-request argument: the question text (accepted; no served policy reads it)."""
STOP = "xgraph_stop"
"""Per-request argument: 0 turns STOP off for the request (STOP is never on here)."""
REPLAYS = ("replayed", "tail mismatch", "disallowed")
"""The outcomes of a replayed prefill, which XGraphLogitsProcessor.replays counts."""

_UNSERVED_ARGS = ("xgraph_relation_ranks", "xgraph_path_options")
_UNSERVED_SETTINGS = {  # setting: the value that keeps the policy off
    "XGRAPH_RELEASE_MASS": "0", "XGRAPH_RELEASE_TOP": "0", "XGRAPH_ESCAPE_BIAS": "0",
    "XGRAPH_EXPRESSIONS": "0", "XGRAPH_STOP": "", "XGRAPH_OBSERVE": "0", "XGRAPH_OBSERVE_SELECT": "0",
    "XGRAPH_OBSERVE_ANSWER": "0", "XGRAPH_OBSERVE_WIDTH": "0", "XGRAPH_OBSERVE_DEFER": "0",
    "XGRAPH_OBSERVE_TERMINAL": "0", "XGRAPH_MENU": "0", "XGRAPH_MENU_CLOSE_NEXT": "0", "XGRAPH_AUDIT": "0",
    "XGRAPH_REQUEST_PATH_OPTIONS": "0", "XGRAPH_RELATIONS": "frontier",
}

_REGISTERED: dict[str, list[str]] = {}
_REPLAY_RESULTS: dict[str, str] = {}


def collect_replay_status(_worker, keys: list[str]) -> dict[str, str]:
    """vLLM worker RPC: hand over (and forget) the replay outcomes kept under `keys`."""
    from xgraph_b200.vllm import _REPLAY_RESULTS as results

    return {key: results.pop(key) for key in keys if key in results}


class XGraphWorkerExtension:
    """vLLM worker extension (``worker_extension_cls="xgraph_b200.vllm.XGraphWorkerExtension"``)
    through which `replay_statuses` collects replay outcomes from the workers."""

    def xgraph_collect_replay_status(self, keys: list[str]) -> dict[str, str]:
        from xgraph_b200.vllm import collect_replay_status

        return collect_replay_status(self, keys)


def replay_statuses(llm, keys: list[str]) -> dict[str, dict]:
    """The replay outcome of each key over all workers (src/xgraph/vllm.py:150-196): a
    decline on any worker wins; a key every worker confirms is replayed; anything else
    (no answer, a worker that did not see the key) is unconfirmed."""
    unavailable = "worker replay status unavailable"
    try:
        rpc = getattr(llm, "collective_rpc", None)
        results = rpc("xgraph_collect_replay_status", args=(keys,), timeout=30) if callable(rpc) else []
    except Exception as error:  # the outcome is reported, not raised
        results = []
        unavailable = f"worker replay status failed: {type(error).__name__}: {str(error)[:512]}"
    if not isinstance(results, (list, tuple)):
        results, unavailable = [], "invalid worker replay status response"
    statuses = {}
    for key in keys:
        values = [item[key] for item in results if isinstance(item, dict) and key in item]
        declined = next((v for v in values if v in ("tail mismatch", "disallowed")), None)
        if declined is not None:
            statuses[key] = {"replay_status": "declined", "replay_reason": declined, "declined": True}
        elif results and len(values) == len(results) and all(v == "replayed" for v in values):
            statuses[key] = {"replay_status": "replayed"}
        else:
            statuses[key] = {"replay_status": "unconfirmed", "replay_reason": unavailable, "error": True}
    return statuses


def _version_names(path: str) -> list[str]:
    """The version names of a version file, read once per process."""
    if path not in _REGISTERED:
        from xgraph_b200.kgversions import version_names

        _REGISTERED[path] = version_names(path)
    return _REGISTERED[path]


def replayed_tokens(tail: list[int], token_bytes, prefill: bytes) -> int | None:
    """How many of the last tokens of `tail` to replay for a prompt ending with `prefill`:
    the fewest whose bytes (token_bytes: a token's bytes, None for a special token) cover
    it, or None if their bytes do not end with it (src/xgraph/vllm.py:233-245)."""
    written = b""
    for count, token in enumerate(reversed(tail), start=1):
        data = token_bytes(token)
        if data is None:
            return None
        written = data + written
        if len(written) >= len(prefill):
            return count if written.endswith(prefill) else None
    return None


def _setting(name: str) -> str:
    value = os.environ.get(name)
    if not value:
        raise RuntimeError(f"{name} is not set; the xgraph logits processor needs it")
    return value


def check_served_settings(environ=os.environ) -> None:
    """Refuse settings that ask for a policy this engine does not serve."""
    asked = [name for name, off in _UNSERVED_SETTINGS.items()
             if environ.get(name) not in (None, "", off) and not _is_zero(environ.get(name), off)]
    if asked:
        raise ValueError(f"not served by the xgraph_b200 engine: {', '.join(asked)} "
                         "(the reference's research policies are out of its scope)")


def _is_zero(value: str | None, off: str) -> bool:
    if off != "0" or value is None:
        return False
    try:
        return float(value) == 0.0
    except ValueError:
        return False


class PendingRequest:
    """One slot's staged admission (in admission order), then its delayed prefill replay."""

    def __init__(self) -> None:
        self.admissions: list[tuple[int, bool]] = []
        self.anchor: list[str] | None = None
        self.version: str | None = None
        self.opened = False
        self.prefill: bytes | None = None
        self.replay_id: str | None = None
        self.order: dict[str, int] = {}

    def stage(self, name: str, value: Any, order: int) -> None:
        if value is None:
            self.order.pop(name, None)
        else:
            self.order.setdefault(name, order)
        setattr(self, name, value)


class XGraphLogitsProcessor(_Base):
    """vLLM Model Runner V2 logits processor over the B200 constraint engine.

    Construction reads XGRAPH_KG_INDEX and XGRAPH_TOKENIZER (and XGRAPH_KG_VERSIONS when
    set) and builds one engine with vLLM's `max_num_reqs` slots on the worker's GPU; it
    needs the engine's CUDA library.  The worker calls `add_request` for each admitted
    request, `apply_staged_writes` before a step, and `apply(logits, ctx)` per step.
    """

    def __init__(self, vllm_config: Any, req_states: Any) -> None:
        import torch

        from xgraph_b200.engine import Engine
        from xgraph_b200.index import load_kg_index
        from xgraph_b200.tokenizer import ServedTokenizer

        check_served_settings()
        index = load_kg_index(_setting("XGRAPH_KG_INDEX"))
        tokenizer = ServedTokenizer.from_file(_setting("XGRAPH_TOKENIZER"))
        versions = None
        if os.environ.get(VERSIONS):
            from xgraph_b200.kgversions import load_kg_versions

            versions = load_kg_versions(os.environ[VERSIONS], index)
            for stats in versions.stats:
                print(f"xgraph: KG version {stats}", file=sys.stderr, flush=True)
        self._torch = torch
        self._req_states = req_states
        self._tokenizer = tokenizer
        self._syntax = index.span_syntax
        end_after_answer = os.environ.get("XGRAPH_END_AFTER_ANSWER", "0") == "1"
        eos_token_ids: list[int] = []
        if end_after_answer:
            from vllm.tokenizers import cached_tokenizer_from_config

            # as vLLM's input processor: the served tokenizer's EOS plus every EOS in the
            # model's generation config
            model_config = vllm_config.model_config
            served = cached_tokenizer_from_config(model_config)
            generation = model_config.try_get_generation_config()
            for ids in (getattr(served, "eos_token_id", None), generation.get("eos_token_id")):
                if ids is not None:
                    eos_token_ids.extend([ids] if isinstance(ids, int) else ids)
        self._engine = Engine(
            index, tokenizer, index.span_syntax, req_states.max_num_reqs,
            escapes=os.environ.get("XGRAPH_ESCAPES", "1") != "0",
            repeats=os.environ.get("XGRAPH_REPEATS", "1") != "0",
            derivation=os.environ.get("XGRAPH_DERIVATION", "0") == "1",
            paths=os.environ.get("XGRAPH_PATHS", "0") == "1",
            bound_escapes=os.environ.get("XGRAPH_BOUND_ESCAPES", "1") == "1",
            committed_paths=os.environ.get("XGRAPH_COMMITTED_PATHS", "0") == "1",
            versions=versions,
            start_rank=os.environ.get("XGRAPH_START_RANK") or "degree",
            unquoted_starts=os.environ.get("XGRAPH_UNQUOTED_STARTS", "0") == "1",
            end_after_answer=end_after_answer,
            eos_token_ids=eos_token_ids,
        )
        self._pending: dict[int, PendingRequest] = {}
        self._replaying: dict[int, PendingRequest] = {}
        self._admission_order = 0
        self.replays = dict.fromkeys(REPLAYS, 0)

    @property
    def engine(self):
        """The engine the processor drives (one slot per vLLM request slot)."""
        return self._engine

    @property
    def engine_syntax(self):
        """The span syntax of the KG index the engine serves."""
        return self._syntax

    @classmethod
    def validate_params(cls, sampling_params: Any) -> None:
        """The reference's per-request argument checks (src/xgraph/vllm.py:442-516) for the
        served arguments; arguments of unserved policies are refused."""
        extra = sampling_params.extra_args or {}
        value = extra.get(OPT_IN)
        if value not in (None, 0, 1) or isinstance(value, float):
            raise ValueError(f"the per-request argument {OPT_IN!r} must be 0 or 1, got {value!r}")
        for name in _UNSERVED_ARGS:
            if name in extra:
                raise ValueError(f"the per-request argument {name!r} is not served by the xgraph_b200 engine")
        question = extra.get(QUESTION)
        if question is not None and (not isinstance(question, str) or not question.strip()):
            raise ValueError(f"the per-request argument {QUESTION!r} must be the question text")
        stop = extra.get(STOP)
        if stop is not None and (type(stop) is not int or stop != 0):
            raise ValueError(f"the per-request argument {STOP!r} only accepts 0, got {stop!r}")
        if stop is not None and value != 1:
            raise ValueError(f"{STOP} needs the engine: set {OPT_IN!r} to 1")
        opened = extra.get(OPEN)
        if opened not in (None, 0, 1) or isinstance(opened, float):
            raise ValueError(f"the per-request argument {OPEN!r} must be 0 or 1, got {opened!r}")
        if opened and value != 1:
            raise ValueError(f"{OPEN} needs the engine: set the per-request argument {OPT_IN!r} to 1")
        prefill = extra.get(PREFILL)
        if REPLAY_ID in extra and (not isinstance(extra[REPLAY_ID], str) or not extra[REPLAY_ID] or not prefill):
            raise ValueError(f"{REPLAY_ID} needs a nonempty string and {PREFILL}")
        if prefill is not None:
            if not isinstance(prefill, str) or not prefill:
                raise ValueError(f"the per-request argument {PREFILL!r} must be the text the prompt ends "
                                 f"with, got {prefill!r}")
            if value != 1:
                raise ValueError(f"{PREFILL} needs the engine: set the per-request argument {OPT_IN!r} to 1")
            if opened:
                raise ValueError(f"{PREFILL} and {OPEN} exclude each other: replay the opener")
        version = extra.get(KG_VERSION)
        if version is None:
            return
        if not isinstance(version, str):
            raise ValueError(f"the per-request argument {KG_VERSION!r} must be a KG version's name, got {version!r}")
        if not os.environ.get(VERSIONS):
            raise ValueError(f"{KG_VERSION} names {version!r}, but no KG versions are registered "
                             f"({VERSIONS} is not set)")
        names = _version_names(os.environ[VERSIONS])
        if version not in names:
            raise ValueError(f"no KG version {version!r}; the registered ones are {names}")

    def add_request(self, req_idx: int, sampling_params: Any) -> bool:
        """Stage the admission of a request to slot `req_idx`; True when it opted in."""
        extra = sampling_params.extra_args or {}
        on = bool(extra.get(OPT_IN))
        order = self._admission_order
        self._admission_order += 1
        pending = self._pending.setdefault(req_idx, PendingRequest())
        pending.admissions.append((order, on))
        if on and ANCHOR in extra:
            pending.stage("anchor", [str(e) for e in extra[ANCHOR]], order)
        pending.stage("version", str(extra[KG_VERSION]) if on and extra.get(KG_VERSION) else None, order)
        pending.opened = bool(on and extra.get(OPEN))
        if on and extra.get(PREFILL):
            pending.prefill = str(extra[PREFILL]).encode("utf-8")
            pending.replay_id = extra.get(REPLAY_ID) or None
            self._replaying[req_idx] = pending
        else:
            self._replaying.pop(req_idx, None)
        return on

    def apply_staged_writes(self) -> None:
        """Begin (or end) the admitted slots in admission order, then set their anchors and
        versions and open the spans of `xgraph_open` requests."""
        admissions = sorted((order, slot, on) for slot, pending in self._pending.items()
                            for order, on in pending.admissions)
        for on, start in ((True, self._engine.begin), (False, self._engine.end)):
            slots = [slot for _, slot, enabled in admissions if enabled == on]
            if slots:
                start(self._slots(slots), self._stream())
        for field, method in (("anchor", "anchor"), ("version", "set_version")):
            writes = sorted((pending.order[field], slot, getattr(pending, field))
                            for slot, pending in self._pending.items() if field in pending.order)
            for _, slot, value in writes:
                getattr(self._engine, method)(slot, value, self._stream())
        for slot in sorted(slot for slot, pending in self._pending.items() if pending.opened):
            self._engine.open_span(slot, self._stream())
        self._pending.clear()

    def apply(self, logits: Any, ctx: Any) -> Any:
        """Advance every opted-in slot of the step over its newly committed tokens and set the
        logits its mask disallows to -inf, in place (src/xgraph/vllm.py:607-631)."""
        int32 = self._torch.int32
        state = self._req_states
        stream = self._stream()
        if self._replaying:  # before the slots' first sync: their cursors are still unset
            self._replay(stream)
        slots = ctx.idx_mapping.to(int32)
        if ctx.expanded_idx_mapping.shape[0] == ctx.idx_mapping.shape[0]:  # no drafts: one launch
            self._engine.sync_apply(slots, state.all_token_ids.gpu, state.prompt_len.gpu, state.total_len.gpu,
                                    logits, stream)
        else:
            self._engine.sync(slots, state.all_token_ids.gpu, state.prompt_len.gpu, state.total_len.gpu, stream)
            self._engine.apply_mask(logits, ctx.expanded_idx_mapping.to(int32), stream,
                                    local_pos=ctx.expanded_local_pos.to(int32), input_ids=ctx.input_ids.to(int32))
        return logits

    def _replay(self, stream: int) -> None:
        """Advance each slot with a pending prefill over the prompt tokens that hold it, then
        decline (end) those whose tail does not match or whose replay hit a token outside the
        mask (src/xgraph/vllm.py:633-680)."""
        from xgraph_b200.engine import PHASE_ERROR
        from xgraph_b200.vllm import _REPLAY_RESULTS as results

        torch, state = self._torch, self._req_states
        pending, self._replaying = self._replaying, {}
        history = state.all_token_ids.gpu
        start = torch.zeros_like(state.prompt_len.gpu)
        stop = torch.zeros_like(state.prompt_len.gpu)
        replayed, declined = [], []
        for slot, request in sorted(pending.items()):
            prefill = request.prefill
            end = int(state.prompt_len.gpu[slot])
            tail = history[slot, max(0, end - len(prefill)): end].tolist()
            count = replayed_tokens(tail, self._tokenizer.token_bytes, prefill)
            if count is None:
                declined.append((slot, "tail mismatch"))
                continue
            start[slot], stop[slot] = end - count, end
            replayed.append(slot)
        if replayed:  # sync from start to stop: the cursors then stand at the prompt's end
            self._engine.sync(self._slots(replayed), history, start, stop, stream)
            phases = self._engine.states_host(max(replayed) + 1)["phase"]
            for slot in replayed:
                if phases[slot] == PHASE_ERROR:
                    declined.append((slot, "disallowed"))
                else:
                    self.replays["replayed"] += 1
                    if key := pending[slot].replay_id:
                        results.setdefault(key, "replayed")  # a re-admission never erases a decline
        if declined:
            self._engine.end(self._slots([slot for slot, _ in declined]), stream)
            for slot, reason in declined:
                self.replays[reason] += 1
                if key := pending[slot].replay_id:
                    results[key] = reason
                print(f"xgraph: declined the replayed prefill of the request in slot {slot} ({reason}); "
                      f"it is left unmasked. Replays so far: {self.replays}", file=sys.stderr, flush=True)

    def _slots(self, slots: list[int]) -> Any:
        return self._torch.tensor(slots, dtype=self._torch.int32, device=self._req_states.device)

    def _stream(self) -> int:
        return self._torch.cuda.current_stream().cuda_stream
