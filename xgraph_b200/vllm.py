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
XGRAPH_RELEASE_MASS, XGRAPH_RELEASE_TOP, XGRAPH_DERIVATION, XGRAPH_ESCAPE_BIAS, XGRAPH_PATHS,
XGRAPH_BOUND_ESCAPES, XGRAPH_COMMITTED_PATHS, XGRAPH_START_RANK, XGRAPH_UNQUOTED_STARTS,
XGRAPH_END_AFTER_ANSWER, XGRAPH_STOP (residual-goal: each opted-in request supplies its
question as `xgraph_question`; `xgraph_stop` 0 turns STOP off for a request),
XGRAPH_RELATIONS (frontier, vocabulary or successor relation support), XGRAPH_EXPRESSIONS
(1: date and value comparisons; needs XGRAPH_PATHS=1, XGRAPH_COMMITTED_PATHS=1 and an index
with the date table).  The reference's other research policies (observations, menus, audit,
per-request path options) are not served by this engine: a setting or argument
that asks for one is refused with a ValueError naming it.

This module imports only the standard library at import time: vLLM also calls
validate_params in its frontend process.
"""

from __future__ import annotations

import os
import sys
from dataclasses import dataclass
from typing import Any

try:
    from vllm.v1.worker.gpu.sample.logits_processor import LogitsProcessor as _Base
except ImportError:  # no vLLM of that API: the class still works with stand-ins
    _Base = object  # type: ignore[assignment,misc]

OPT_IN = "xgraph"
ANCHOR = "xgraph_anchor"
"""Request extra arg: entity ids bound before the first span (derivation and path mode start there)."""
KG_VERSION = "xgraph_kg_version"
"""Request extra arg: which version of the XGRAPH_KG_VERSIONS file this request's KG reads."""
VERSIONS = "XGRAPH_KG_VERSIONS"
OPEN = "xgraph_open"
"""Request extra arg: 1 when the prompt already ends in the span opener (decoding begins in a span)."""
PREFILL = "xgraph_prefill"
"""Request extra arg: trailing prompt text to run through the engine before decoding."""
REPLAY_ID = "xgraph_replay_id"
"""Request extra arg: key under which the replay outcome is kept for replay_statuses."""
QUESTION = "xgraph_question"
"""Request extra arg: the question, which STOP needs (XGRAPH_STOP=residual-goal)."""
STOP = "xgraph_stop"
"""Request extra arg: 0 disables STOP for this one request."""
REPLAYS = ("replayed", "tail mismatch", "disallowed")
"""What a replayed prefill can end as (the keys of XGraphLogitsProcessor.replays)."""

_UNSERVED_ARGS = ("xgraph_relation_ranks", "xgraph_path_options")
_UNSERVED_SETTINGS = {  # setting: the value that keeps the policy off
    "XGRAPH_OBSERVE": "0", "XGRAPH_OBSERVE_SELECT": "0",
    "XGRAPH_OBSERVE_ANSWER": "0", "XGRAPH_OBSERVE_WIDTH": "0", "XGRAPH_OBSERVE_DEFER": "0",
    "XGRAPH_OBSERVE_TERMINAL": "0", "XGRAPH_MENU": "0", "XGRAPH_MENU_CLOSE_NEXT": "0", "XGRAPH_AUDIT": "0",
    "XGRAPH_REQUEST_PATH_OPTIONS": "0",
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


DECLINES = ("tail mismatch", "disallowed")


def _worker_receipts(llm, keys: list[str]) -> tuple[list, str]:
    """Every worker's {key: outcome} answer to the replay-status RPC, with the reason to give
    for a key no answer settles."""
    call = getattr(llm, "collective_rpc", None)
    if not callable(call):
        return [], "worker replay status unavailable"
    try:
        answers = call("xgraph_collect_replay_status", args=(keys,), timeout=30)
    except Exception as error:  # the outcome is reported, not raised
        return [], f"worker replay status failed: {type(error).__name__}: {str(error)[:512]}"
    if not isinstance(answers, (list, tuple)):
        return [], "invalid worker replay status response"
    return list(answers), "worker replay status unavailable"


def replay_statuses(llm, keys: list[str]) -> dict[str, dict]:
    """The replay outcome of each key over all workers (the reference's
    src/xgraph/vllm.py:150-196 reports the same three kinds): declined when some worker
    declined it (that worker's reason), replayed when every worker answered and each says
    replayed, else unconfirmed (an answer missing or unreadable)."""
    answers, missing = _worker_receipts(llm, keys)
    readable = [a for a in answers if isinstance(a, dict)]
    out: dict[str, dict] = {}
    for key in keys:
        outcomes = [a.get(key) for a in readable]
        reason = next((o for o in outcomes if o in DECLINES), None)
        if reason is not None:
            out[key] = {"replay_status": "declined", "replay_reason": reason, "declined": True}
        elif answers and len(readable) == len(answers) and all(o == "replayed" for o in outcomes):
            out[key] = {"replay_status": "replayed"}
        else:
            out[key] = {"replay_status": "unconfirmed", "replay_reason": missing, "error": True}
    return out


def _version_names(path: str) -> list[str]:
    """Version names of the file at `path`, cached for the life of the process."""
    if path not in _REGISTERED:
        from xgraph_b200.kgversions import version_names

        _REGISTERED[path] = version_names(path)
    return _REGISTERED[path]


def tail_cover(tail: list[int], token_bytes, prefill: bytes) -> int | None:
    """The number k of trailing tokens of `tail` to replay so that the prompt's end holds
    `prefill`: the smallest k whose tokens' bytes are at least as long as it, accepted only
    if those bytes end with it and none of the k tokens is special (token_bytes(t) is None
    for a special token); None declines the replay."""
    sizes = []
    for token in reversed(tail):
        data = token_bytes(token)
        if data is None:
            return None
        sizes.append(data)
        if sum(map(len, sizes)) >= len(prefill):
            return len(sizes) if b"".join(reversed(sizes)).endswith(prefill) else None
    return None


def _required_env(name: str) -> str:
    """An environment setting the processor cannot start without."""
    if value := os.environ.get(name):
        return value
    raise RuntimeError(f"the xgraph logits processor needs the environment setting {name}")


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


def _flag(extra: dict, name: str):
    """A 0/1 per-request argument (absent: None); any other value is refused."""
    value = extra.get(name)
    if value is None or (not isinstance(value, float) and value in (0, 1)):
        return value
    raise ValueError(f"the per-request argument {name!r} takes 0 or 1, not {value!r}")


def _needs_engine(engine: bool, name: str) -> None:
    if not engine:
        raise ValueError(f"{name!r} only applies to requests that set {OPT_IN!r} to 1")


def _check_version_argument(version) -> None:
    """A KG version named by a request must be one of XGRAPH_KG_VERSIONS."""
    if version is None:
        return
    if not isinstance(version, str):
        raise ValueError(f"{KG_VERSION!r} is a KG version's name, not {version!r}")
    path = os.environ.get(VERSIONS)
    if not path:
        raise ValueError(f"{KG_VERSION!r} asks for {version!r} but {VERSIONS} registers no KG versions")
    names = _version_names(path)
    if version not in names:
        raise ValueError(f"{version!r} is not a registered KG version (those are {names})")


@dataclass
class Staged:
    """What a slot's admissions since the last step leave it with: the latest admitted
    request (Admission: begin or end, anchors, version, open) and its prefill to replay.
    A slot that was also ended during the step ends (the adapter begins before it ends)."""

    admission: Any
    ended: bool = False
    prefill: bytes | None = None
    replay_id: str | None = None
    question: str | None = None  # residual-goal STOP: the request's question


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
        index = load_kg_index(_required_env("XGRAPH_KG_INDEX"))
        tokenizer = ServedTokenizer.from_file(_required_env("XGRAPH_TOKENIZER"))
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
        self._stop = os.environ.get("XGRAPH_STOP") or None
        # XGRAPH_EXPRESSIONS=1: a span may be a date or value comparison (src/xgraph/vllm.py:342-383)
        expressions = os.environ.get("XGRAPH_EXPRESSIONS", "0") == "1"
        if expressions and not (os.environ.get("XGRAPH_PATHS", "0") == "1"
                                and os.environ.get("XGRAPH_COMMITTED_PATHS", "0") == "1"):
            raise ValueError("XGRAPH_EXPRESSIONS=1 needs path mode with committed paths: "
                             "XGRAPH_PATHS=1 and XGRAPH_COMMITTED_PATHS=1")
        self._engine = Engine(
            index, tokenizer, index.span_syntax, req_states.max_num_reqs,
            escapes=os.environ.get("XGRAPH_ESCAPES", "1") != "0",
            repeats=os.environ.get("XGRAPH_REPEATS", "1") != "0",
            # release a span's step to the escape marker when the model puts less than
            # XGRAPH_RELEASE_MASS on the allowed set, or (XGRAPH_RELEASE_TOP=1) when its
            # own top token is disallowed; XGRAPH_ESCAPE_BIAS is added to the logits of
            # the tokens that commit to the escape (src/xgraph/vllm.py:319-329)
            release_mass=float(os.environ.get("XGRAPH_RELEASE_MASS", "0")),
            release_top=os.environ.get("XGRAPH_RELEASE_TOP", "0") == "1",
            derivation=os.environ.get("XGRAPH_DERIVATION", "0") == "1",
            escape_bias=float(os.environ.get("XGRAPH_ESCAPE_BIAS", "0")),
            paths=os.environ.get("XGRAPH_PATHS", "0") == "1",
            bound_escapes=os.environ.get("XGRAPH_BOUND_ESCAPES", "1") == "1",
            committed_paths=os.environ.get("XGRAPH_COMMITTED_PATHS", "0") == "1",
            versions=versions,
            start_rank=os.environ.get("XGRAPH_START_RANK") or "degree",
            unquoted_starts=os.environ.get("XGRAPH_UNQUOTED_STARTS", "0") == "1",
            end_after_answer=end_after_answer,
            eos_token_ids=eos_token_ids,
            stop=self._stop,
            relations=os.environ.get("XGRAPH_RELATIONS") or "frontier",
            expressions=expressions,
        )
        self._staged: dict[int, Staged] = {}   # slot -> admissions since the last apply_staged_writes
        self._folded = None                    # admission records the next step's launch applies
        self._prefills: dict[int, Staged] = {}  # slot -> a prefill to replay before its first sync
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
        """Refuse a request whose per-request arguments the engine cannot honour (the
        arguments and what they accept are the reference's, src/xgraph/vllm.py:442-516, for
        the served policies); arguments of unserved policies are refused by name."""
        extra = sampling_params.extra_args or {}
        engine = _flag(extra, OPT_IN) == 1
        unserved = [name for name in _UNSERVED_ARGS if name in extra]
        if unserved:
            raise ValueError(f"{unserved[0]!r} belongs to a policy the xgraph_b200 engine does not serve")
        question = extra.get(QUESTION)
        if STOP in extra:
            if type(extra[STOP]) is not int or extra[STOP] != 0:
                raise ValueError(f"the per-request argument {STOP!r} only accepts 0, got {extra[STOP]!r}")
            _needs_engine(engine, STOP)
        if ((engine and extra.get(STOP) != 0 and os.environ.get("XGRAPH_STOP")) or question is not None) and not (
                isinstance(question, str) and question.strip()):
            raise ValueError(f"the per-request argument {QUESTION!r} must be the question text")
        opened = _flag(extra, OPEN)
        if opened:
            _needs_engine(engine, OPEN)
        prefill = extra.get(PREFILL)
        if REPLAY_ID in extra:
            key = extra[REPLAY_ID]
            if not (isinstance(key, str) and key) or not prefill:
                raise ValueError(f"{REPLAY_ID!r} is a nonempty string key and goes with {PREFILL!r}")
        if prefill is not None:
            if not (isinstance(prefill, str) and prefill):
                raise ValueError(f"{PREFILL!r} is the text the prompt ends with, not {prefill!r}")
            _needs_engine(engine, PREFILL)
            if opened:
                raise ValueError(f"{PREFILL!r} replays the opener itself; it cannot go with {OPEN!r}")
        _check_version_argument(extra.get(KG_VERSION))

    def add_request(self, req_idx: int, sampling_params: Any) -> bool:
        """Stage the admission of a request to slot `req_idx`; True when it opted in."""
        from xgraph_b200.engine import Admission

        extra = sampling_params.extra_args or {}
        on = bool(extra.get(OPT_IN))
        earlier = self._staged.get(req_idx)
        entry = Staged(Admission(req_idx, False), ended=True) if not on else Staged(Admission(
            req_idx, True, tuple(str(e) for e in extra.get(ANCHOR) or ()),
            str(extra[KG_VERSION]) if extra.get(KG_VERSION) else None, bool(extra.get(OPEN))))
        entry.ended |= bool(earlier and earlier.ended)
        if on and self._stop and extra.get(STOP) != 0:
            question = extra.get(QUESTION)
            if not isinstance(question, str) or not question.strip():
                raise ValueError(f"residual-goal STOP needs the per-request argument {QUESTION!r}")
            entry.question = question
        if on and extra.get(PREFILL):
            entry.prefill = str(extra[PREFILL]).encode("utf-8")
            entry.replay_id = extra.get(REPLAY_ID) or None
        self._staged[req_idx] = entry
        return on

    def apply_staged_writes(self) -> None:
        """Turn the staged admissions into one admission record per slot.  They are applied
        in the next step's launch (Engine.sync_apply with admissions), or by one admit launch
        when that step needs them earlier (a prefill to replay, draft rows)."""
        from xgraph_b200.engine import Admission

        if not self._staged:
            return
        if self._folded is not None:  # a second round before any step: the first goes now
            self._engine.admit(self._folded, self._stream())
            self._folded = None
        admissions, questions = [], []
        for slot, entry in sorted(self._staged.items()):
            admissions.append(Admission(slot, False) if entry.ended else entry.admission)
            if entry.prefill is not None and not entry.ended:
                self._prefills[slot] = entry
            else:
                self._prefills.pop(slot, None)
            if entry.question is not None and not entry.ended:
                questions.append((slot, entry.question))
        self._staged.clear()
        records = self._engine.admission_records(admissions)
        if questions:  # a STOP table goes in after its slot's begin: admit now, then install
            self._engine.admit(records, self._stream())
            for slot, question in questions:
                self._engine.set_stop(slot, question, self._stream())
        else:
            self._folded = records

    def apply(self, logits: Any, ctx: Any) -> Any:
        """Advance every opted-in slot of the step over its newly committed tokens and set the
        logits its mask disallows to -inf, in place (the reference adapter's step,
        src/xgraph/vllm.py:607-631), with the step's admissions applied first."""
        int32 = self._torch.int32
        state = self._req_states
        stream = self._stream()
        drafts = ctx.expanded_idx_mapping.shape[0] != ctx.idx_mapping.shape[0]
        if self._folded is not None and (drafts or self._prefills):
            self._engine.admit(self._folded, stream)
            self._folded = None
        if self._prefills:  # before the slots' first sync: their cursors are still unset
            self._replay_prefills(stream)
        slots = ctx.idx_mapping.to(int32)
        if not drafts:  # one launch: admissions, sync and the masks
            folded, self._folded = self._folded, None
            self._engine.sync_apply(slots, state.all_token_ids.gpu, state.prompt_len.gpu, state.total_len.gpu,
                                    logits, stream, admissions=folded)
        else:
            self._engine.sync(slots, state.all_token_ids.gpu, state.prompt_len.gpu, state.total_len.gpu, stream)
            self._engine.apply_mask(logits, ctx.expanded_idx_mapping.to(int32), stream,
                                    local_pos=ctx.expanded_local_pos.to(int32), input_ids=ctx.input_ids.to(int32))
        return logits

    def _replay_prefills(self, stream: int) -> None:
        """Each admitted slot with a prefill consumes the prompt tokens that spell it (sync
        over [prompt_len - k, prompt_len)), as if the model had written them; a prompt that
        does not end with the prefill's bytes, or a replay that leaves the language, ends
        the slot (the request is served unmasked) and is counted and reported."""
        from xgraph_b200.engine import PHASE_ERROR
        from xgraph_b200.vllm import _REPLAY_RESULTS as outcomes

        torch, state = self._torch, self._req_states
        todo, self._prefills = sorted(self._prefills.items()), {}
        prompt_end = state.prompt_len.gpu
        begin_at, end_at = torch.zeros_like(prompt_end), torch.zeros_like(prompt_end)
        outcome: dict[int, str] = {}
        live = []
        for slot, entry in todo:
            end = int(prompt_end[slot])
            tail = state.all_token_ids.gpu[slot, max(0, end - len(entry.prefill)): end].tolist()
            k = tail_cover(tail, self._tokenizer.token_bytes, entry.prefill)
            if k is None:
                outcome[slot] = "tail mismatch"
                continue
            begin_at[slot], end_at[slot] = end - k, end
            live.append(slot)
        if live:  # afterwards the slots' cursors stand at their prompts' ends
            self._engine.sync(self._slots(live), state.all_token_ids.gpu, begin_at, end_at, stream)
            phase = self._engine.states_host(max(live) + 1)["phase"]
            for slot in live:
                outcome[slot] = "disallowed" if phase[slot] == PHASE_ERROR else "replayed"
        ended = sorted(slot for slot, result in outcome.items() if result != "replayed")
        if ended:
            self._engine.end(self._slots(ended), stream)
        for slot, entry in todo:
            result = outcome[slot]
            self.replays[result] += 1
            if entry.replay_id:
                if result == "replayed":
                    outcomes.setdefault(entry.replay_id, result)  # a decline stays a decline
                else:
                    outcomes[entry.replay_id] = result
            if result != "replayed":
                print(f"xgraph: slot {slot}: the replayed prefill was declined ({result}); the request "
                      f"runs unmasked. Replays: {self.replays}", file=sys.stderr, flush=True)

    def _slots(self, slots: list[int]) -> Any:
        return self._torch.tensor(slots, dtype=self._torch.int32, device=self._req_states.device)

    def _stream(self) -> int:
        return self._torch.cuda.current_stream().cuda_stream
