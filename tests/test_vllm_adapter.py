"""The vLLM Model Runner V2 processor (xgraph_b200.vllm) with stand-ins for vLLM's request
state and step context, as the reference's adapter tests do (tests/test_vllm_adapter.py:
44-70, 297-320).  CPU tests cover argument checks, settings, the replay helpers and the
admission bookkeeping; GPU tests drive golden walks through `apply` and compare every
masked row with the reference's allowed sets, with one row per request and with draft rows,
and replay a prefill."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest

from tests.conftest import case_versions, golden_masks, golden_walks, golden_worlds, unpack, world_index
from xgraph_b200 import vllm as adapter


def params(**extra):
    return SimpleNamespace(extra_args=extra)


# -- CPU ---------------------------------------------------------------------------------

@pytest.mark.parametrize("extra", [{}, {"xgraph": 0}, {"xgraph": 1}, {"xgraph": 1, "xgraph_open": 1},
                                   {"xgraph": 1, "xgraph_prefill": "⟦ Ada", "xgraph_replay_id": "k"},
                                   {"xgraph": 1, "xgraph_question": "who?", "xgraph_stop": 0}])
def test_valid_arguments(extra):
    adapter.XGraphLogitsProcessor.validate_params(params(**extra))


@pytest.mark.parametrize("extra", [{"xgraph": 2}, {"xgraph": 1.0}, {"xgraph_open": 1}, {"xgraph": 1, "xgraph_open": 2},
                                   {"xgraph_prefill": "x"}, {"xgraph": 1, "xgraph_prefill": ""},
                                   {"xgraph": 1, "xgraph_prefill": "x", "xgraph_open": 1},
                                   {"xgraph": 1, "xgraph_replay_id": "k"}, {"xgraph": 1, "xgraph_stop": 1},
                                   {"xgraph": 1, "xgraph_question": None, "xgraph_stop": 2},
                                   {"xgraph_stop": 0}, {"xgraph": 1, "xgraph_question": " "},
                                   {"xgraph": 1, "xgraph_relation_ranks": []}, {"xgraph": 1, "xgraph_path_options": "{}"},
                                   {"xgraph": 1, "xgraph_kg_version": 3}, {"xgraph": 1, "xgraph_kg_version": "v"}])
def test_invalid_arguments_raise(extra, monkeypatch):
    monkeypatch.delenv(adapter.VERSIONS, raising=False)
    with pytest.raises(ValueError):
        adapter.XGraphLogitsProcessor.validate_params(params(**extra))


def test_unserved_settings_are_refused():
    adapter.check_served_settings({"XGRAPH_PATHS": "1", "XGRAPH_RELEASE_MASS": "0.2", "XGRAPH_RELATIONS": "frontier",
                                   "XGRAPH_ESCAPE_BIAS": "-2.5", "XGRAPH_RELEASE_TOP": "1", "XGRAPH_OBSERVE": "0.0",
                                   "XGRAPH_STOP": "residual-goal"})
    adapter.check_served_settings({"XGRAPH_RELATIONS": "successor"})  # the relation supports are served
    adapter.check_served_settings({"XGRAPH_EXPRESSIONS": "1"})  # and expressions
    for name, value in [("XGRAPH_MENU", "3"), ("XGRAPH_AUDIT", "1"), ("XGRAPH_OBSERVE", "4")]:
        with pytest.raises(ValueError, match=name):
            adapter.check_served_settings({name: value})


def test_tail_cover():
    table = {1: b"ab", 2: b"c", 3: b" \xe2\x9f\xa6", 4: None}
    tb = table.get
    assert adapter.tail_cover([1, 2], tb, b"c") == 1
    assert adapter.tail_cover([1, 2], tb, b"bc") == 2  # the first token is replayed whole
    assert adapter.tail_cover([1, 2], tb, b"abc") == 2
    assert adapter.tail_cover([1, 2], tb, b"xc") is None
    assert adapter.tail_cover([4, 2], tb, b"bc") is None
    assert adapter.tail_cover([2], tb, b"abc") is None


def test_replay_statuses():
    class LLM:
        def __init__(self, results):
            self.results = results

        def collective_rpc(self, name, args, timeout):
            assert name == "xgraph_collect_replay_status"
            return self.results

    keys = ["a", "b", "c"]
    got = adapter.replay_statuses(LLM([{"a": "replayed", "b": "replayed"}, {"a": "replayed", "b": "disallowed"}]), keys)
    assert got["a"] == {"replay_status": "replayed"}
    assert got["b"]["declined"] and got["b"]["replay_reason"] == "disallowed"
    assert got["c"]["replay_status"] == "unconfirmed"
    assert all(v["replay_status"] == "unconfirmed" for v in adapter.replay_statuses(object(), keys).values())
    adapter._REPLAY_RESULTS.update({"x": "replayed"})
    assert adapter.collect_replay_status(None, ["x", "y"]) == {"x": "replayed"} and "x" not in adapter._REPLAY_RESULTS


def test_version_file_round_trip(tmp_path):
    from xgraph_b200.kgversions import build_kg_versions, load_kg_versions, version_names, write_kg_versions

    case = next(c for c in golden_walks() if c["versions"])
    index = world_index(case["world"], False)
    edits = case_versions(case)
    write_kg_versions(tmp_path, edits, index)
    assert version_names(tmp_path) == list(edits)
    loaded, built = load_kg_versions(tmp_path, index), build_kg_versions(index, edits)
    assert loaded.names == built.names
    for field in ("offsets", "subjects", "adjacency", "edge_relations", "edge_objects"):
        np.testing.assert_array_equal(getattr(loaded, field), getattr(built, field))


def test_admissions_become_one_record_per_slot():
    """The step's admissions: one record per slot (the latest request; a slot also ended in
    the round ends), applied in the next step's launch, or by one admit launch when a second
    round comes first."""
    from xgraph_b200.engine import Admission

    admitted = []

    class FakeEngine:
        def admission_records(self, admissions):
            return list(admissions)

        def admit(self, records, stream):
            admitted.append(records)

    proc = object.__new__(adapter.XGraphLogitsProcessor)
    proc._engine, proc._stream, proc._stop = FakeEngine(), lambda: 0, None
    proc._staged, proc._folded, proc._prefills = {}, None, {}
    assert proc.add_request(3, params(xgraph=1, xgraph_anchor=["Q1"], xgraph_kg_version="v1"))
    assert not proc.add_request(1, params())
    assert proc.add_request(0, params(xgraph=1, xgraph_open=1))
    assert proc.add_request(2, params(xgraph=1, xgraph_prefill="\u27e6 Ada"))
    proc.apply_staged_writes()
    assert proc._folded == [Admission(0, True, (), None, True), Admission(1, False),
                            Admission(2, True), Admission(3, True, ("Q1",), "v1", False)]
    assert list(proc._prefills) == [2] and not proc._staged and not admitted
    assert not proc.add_request(2, params())  # slot 2's next request opts out: no replay
    assert proc.add_request(1, params(xgraph=1))
    proc.apply_staged_writes()
    assert admitted == [[Admission(0, True, (), None, True), Admission(1, False), Admission(2, True),
                         Admission(3, True, ("Q1",), "v1", False)]]
    assert proc._folded == [Admission(1, True), Admission(2, False)] and not proc._prefills
    proc.add_request(4, params(xgraph=1))
    proc.add_request(4, params())  # admitted and ended in one round: it ends
    proc.add_request(4, params(xgraph=1))
    assert proc._staged[4].ended


def test_stop_questions_are_installed_after_their_admissions(monkeypatch):
    """With XGRAPH_STOP=residual-goal a request's question becomes its slot's STOP table
    (Engine.set_stop) right after an admit launch of the round's admissions (the table must
    follow the slot's begin); a request with xgraph_stop=0 gets none."""
    from xgraph_b200.engine import Admission

    calls = []

    class FakeEngine:
        def admission_records(self, admissions):
            return list(admissions)

        def admit(self, records, stream):
            calls.append(("admit", records))

        def set_stop(self, slot, question, stream):
            calls.append(("set_stop", slot, question))

    monkeypatch.setenv("XGRAPH_STOP", "residual-goal")
    proc = object.__new__(adapter.XGraphLogitsProcessor)
    proc._engine, proc._stream, proc._stop = FakeEngine(), lambda: 0, "residual-goal"
    proc._staged, proc._folded, proc._prefills = {}, None, {}
    with pytest.raises(ValueError, match="xgraph_question"):
        proc.add_request(0, params(xgraph=1))
    assert proc.add_request(0, params(xgraph=1, xgraph_question="Which employer has Marie Curie?"))
    assert proc.add_request(1, params(xgraph=1, xgraph_stop=0))
    proc.apply_staged_writes()
    assert calls == [("admit", [Admission(0, True), Admission(1, True)]),
                     ("set_stop", 0, "Which employer has Marie Curie?")]
    assert proc._folded is None
    adapter.XGraphLogitsProcessor.validate_params(params(xgraph=1, xgraph_question="Which spouse has Ada?"))
    with pytest.raises(ValueError, match="xgraph_question"):
        adapter.XGraphLogitsProcessor.validate_params(params(xgraph=1))
    adapter.XGraphLogitsProcessor.validate_params(params(xgraph=1, xgraph_stop=0))


# -- GPU ---------------------------------------------------------------------------------

CASES = ["toy_ordinary", "toy_opened", "bpe_norepeat", "bpe_committed", "bpe_paths", "crowd_committed"]


def processor_for(case, tmp_path, monkeypatch, slots):
    from xgraph_b200.index import save_kg_index
    from xgraph_b200.kgversions import write_kg_versions

    index = world_index(case["world"], case["options"].get("start_rank") == "sitelinks")
    save_kg_index(index, tmp_path / "index")
    (tmp_path / "tokenizer.json").write_text(golden_worlds()[case["world"]]["tokenizer"], encoding="utf-8")
    for name in list(adapter._UNSERVED_SETTINGS) + [adapter.VERSIONS]:
        monkeypatch.delenv(name, raising=False)
    monkeypatch.setenv("XGRAPH_KG_INDEX", str(tmp_path / "index"))
    monkeypatch.setenv("XGRAPH_TOKENIZER", str(tmp_path / "tokenizer.json"))
    options = case["options"]
    flags = {"escapes": "XGRAPH_ESCAPES", "repeats": "XGRAPH_REPEATS", "derivation": "XGRAPH_DERIVATION",
             "paths": "XGRAPH_PATHS", "bound_escapes": "XGRAPH_BOUND_ESCAPES",
             "committed_paths": "XGRAPH_COMMITTED_PATHS", "unquoted_starts": "XGRAPH_UNQUOTED_STARTS"}
    for key, name in flags.items():
        if key in options:
            monkeypatch.setenv(name, "1" if options[key] else "0")
    if "start_rank" in options:
        monkeypatch.setenv("XGRAPH_START_RANK", options["start_rank"])
    if case_versions(case):
        write_kg_versions(tmp_path / "versions", case_versions(case), index)
        monkeypatch.setenv(adapter.VERSIONS, str(tmp_path / "versions"))
        adapter._REGISTERED.clear()
    import torch

    width = 3 + len(case["sequences"][0]["tokens"]) + 8
    state = SimpleNamespace(max_num_reqs=slots, device=torch.device("cuda"),
                            all_token_ids=SimpleNamespace(gpu=torch.zeros((slots, width), dtype=torch.int32, device="cuda")),
                            prompt_len=SimpleNamespace(gpu=torch.zeros(slots, dtype=torch.int32, device="cuda")),
                            total_len=SimpleNamespace(gpu=torch.zeros(slots, dtype=torch.int32, device="cuda")))
    return adapter.XGraphLogitsProcessor(None, state), state


def admit(proc, case, prefill=None):
    for k, seq in enumerate(case["sequences"]):
        extra = {"xgraph": 1}
        if seq["anchor"]:
            extra["xgraph_anchor"] = seq["anchor"]
        if seq["version"]:
            extra["xgraph_kg_version"] = seq["version"]
        if seq["opened"]:
            extra["xgraph_open"] = 1
        if prefill is not None and not seq["opened"]:
            extra["xgraph_prefill"] = prefill[k]
        adapter.XGraphLogitsProcessor.validate_params(params(**extra))
        assert proc.add_request(k, params(**extra))
    proc.apply_staged_writes()


def check_rows(got, was, expected_sets, cols):
    for r, want in enumerate(expected_sets):
        allowed = np.zeros(cols, dtype=bool)
        allowed[sorted(want)] = True
        assert np.all(np.isneginf(got[r][~allowed])), r
        np.testing.assert_array_equal(got[r][allowed], was[r][allowed])


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_one_row_per_request_follows_the_golden_walks(name, tmp_path, monkeypatch):
    import torch

    case = next(c for c in golden_walks() if c["name"] == name)
    seqs = case["sequences"]
    n = len(seqs)
    proc, state = processor_for(case, tmp_path, monkeypatch, n + 1)  # one slot stays unused
    admit(proc, case)
    prompt = 3
    state.prompt_len.gpu[:n] = prompt
    state.all_token_ids.gpu[:n, :prompt] = 7  # the prompt is never advanced over
    gen = torch.Generator(device="cuda").manual_seed(5)
    steps = len(seqs[0]["tokens"])
    from tests.conftest import world

    _, served, _ = world(case["world"])
    for step in range(0, steps, 5):
        state.total_len.gpu[:n] = prompt + step
        for k, seq in enumerate(seqs):
            if step:
                state.all_token_ids.gpu[k, prompt: prompt + step] = torch.tensor(seq["tokens"][:step], dtype=torch.int32)
        rows = torch.arange(n, dtype=torch.int32, device="cuda")
        ctx = SimpleNamespace(idx_mapping=rows, expanded_idx_mapping=rows, expanded_local_pos=torch.zeros_like(rows),
                              input_ids=torch.zeros_like(rows))
        logits = torch.randn((n, served.vocab_size + 2), generator=gen, device="cuda")
        was = logits.clone()
        proc.apply(logits, ctx)
        check_rows(logits.cpu().numpy(), was.cpu().numpy(),
                   [unpack(golden_masks()[f"{name}/{k}"][step], served.vocab_size) for k in range(n)],
                   served.vocab_size + 2)


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["bpe_committed", "bpe_norepeat"])
def test_draft_rows_follow_the_golden_walks(name, tmp_path, monkeypatch):
    import torch

    from tests.conftest import world

    case = next(c for c in golden_walks() if c["name"] == name)
    seqs = case["sequences"]
    n, drafts, prompt = len(seqs), 3, 2
    proc, state = processor_for(case, tmp_path, monkeypatch, n)
    admit(proc, case)
    _, served, _ = world(case["world"])
    state.prompt_len.gpu[:] = prompt
    gen = torch.Generator(device="cuda").manual_seed(9)
    for committed in (1, 20, 41):
        state.total_len.gpu[:] = prompt + committed
        for k, seq in enumerate(seqs):
            state.all_token_ids.gpu[k, prompt: prompt + committed] = torch.tensor(seq["tokens"][:committed],
                                                                                 dtype=torch.int32)
        slots, local, fed, want = [], [], [], []
        for k, seq in enumerate(seqs):
            for j in range(drafts + 1):
                slots.append(k)
                local.append(j)
                fed.append(seq["tokens"][committed + j - 1])
                want.append(unpack(golden_masks()[f"{name}/{k}"][committed + j], served.vocab_size))
        as_t = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")  # noqa: E731
        ctx = SimpleNamespace(idx_mapping=as_t(list(range(n))), expanded_idx_mapping=as_t(slots),
                              expanded_local_pos=as_t(local), input_ids=as_t(fed))
        logits = torch.randn((len(slots), served.vocab_size), generator=gen, device="cuda")
        was = logits.clone()
        proc.apply(logits, ctx)
        check_rows(logits.cpu().numpy(), was.cpu().numpy(), want, served.vocab_size)


@pytest.mark.gpu
def test_replayed_prefill_continues_from_the_replayed_state(tmp_path, monkeypatch):
    """Prompts ending with the start of a span (`⟦ <label>`): the replay leaves each slot
    where advancing a fresh slot over the replayed tokens leaves it; a prompt whose tail
    does not hold its prefill and one whose prefill leaves the language are declined and
    left unmasked."""
    import torch

    from tests.conftest import world
    from xgraph_b200.engine import Engine

    case = next(c for c in golden_walks() if c["name"] == "bpe_committed")
    kg, served, _ = world(case["world"])
    n = 6
    proc, state = processor_for(case, tmp_path, monkeypatch, n)
    labels = [e.labels[0] for e in kg.entities[:n - 2]]
    texts = [f"{'so it goes,' * (k + 1)} \u27e6 {label}" for k, label in enumerate(labels)]
    texts += ["plain prose at the end", "then \u27e6 Zqxzqxzq"]
    prefills = [t[t.index("\u27e6"):] for t in texts[: n - 2]] + ["\u27e6 never written", "\u27e6 Zqxzqxzq"]
    for k in range(n):
        extra = {"xgraph": 1, "xgraph_prefill": prefills[k]}
        adapter.XGraphLogitsProcessor.validate_params(params(**extra))
        proc.add_request(k, params(**extra))
    proc.apply_staged_writes()
    encoded = [served.encode(t) for t in texts]
    for k, ids in enumerate(encoded):
        state.all_token_ids.gpu[k, : len(ids)] = torch.tensor(ids, dtype=torch.int32)
        state.prompt_len.gpu[k] = len(ids)
        state.total_len.gpu[k] = len(ids)
    rows = torch.arange(n, dtype=torch.int32, device="cuda")
    ctx = SimpleNamespace(idx_mapping=rows, expanded_idx_mapping=rows, expanded_local_pos=torch.zeros_like(rows),
                          input_ids=torch.zeros_like(rows))
    logits = torch.randn((n, served.vocab_size), device="cuda")
    was = logits.clone()
    proc.apply(logits, ctx)
    assert proc.replays == {"replayed": n - 2, "tail mismatch": 1, "disallowed": 1}
    # the expected masks: a fresh slot advanced over the same replayed tokens
    options = {k: v for k, v in case["options"].items()}
    plain = Engine(world_index(case["world"], False), served, proc.engine_syntax, 1, **options)
    want = []
    for k in range(n - 2):
        count = adapter.tail_cover(encoded[k], served.token_bytes, prefills[k].encode("utf-8"))
        plain.reset()
        plain.begin(torch.zeros(1, dtype=torch.int32, device="cuda"))
        for token in encoded[k][len(encoded[k]) - count:]:
            plain.advance(np.array([token], dtype=np.int32))
        plain.fill_mask(1)
        want.append(unpack(plain.mask_host(1).view(np.uint32)[0], served.vocab_size))
    got = logits.cpu().numpy()
    check_rows(got[: n - 2], was.cpu().numpy()[: n - 2], want, served.vocab_size)
    np.testing.assert_array_equal(got[n - 2:], was.cpu().numpy()[n - 2:])  # declined: left unmasked
