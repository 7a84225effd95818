"""The committed token streams the benchmark replays, checked on the CPU.

tests/golden/make_streams.py sampled them on a GPU with the engine's masks; here every token
of every stream, up to its replay length, must be allowed by the oracle (so both arms of
bench.py replay valid decodes, and the reference arm needs nothing of the engine), and the
recorded allowed counts must equal the oracle's allowed-set sizes at seeded positions.
"""

from __future__ import annotations

from functools import cache

import numpy as np
import pytest

from tests.conftest import ROOT

FIXTURE = ROOT / "tests" / "golden" / "streams_paths100k.npz"


@cache
def fixture():
    return np.load(FIXTURE)


@cache
def workload():
    from xgraph_b200.synthetic import build_workload

    return build_workload(int(fixture()["config"]), int(fixture()["seed"]))


def oracle():
    from oracle.oracle import Oracle

    w = workload()
    return Oracle(w.index, w.served, w.syntax, **w.config.options)


def test_fixture_matches_its_workload():
    data, w = fixture(), workload()
    assert int(data["vocab"]) == w.served.vocab_size
    assert str(data["fingerprint"]) == w.served.fingerprint
    tokens, lengths = data["tokens"], data["lengths"]
    lo, hi = w.config.lengths
    assert tokens.shape[1] >= hi and lengths.min() >= lo and lengths.max() <= hi
    assert data["allowed"].shape == (tokens.shape[0], tokens.shape[1] + 1)


def test_every_replayed_token_is_allowed_by_the_oracle():
    from oracle.oracle import TokenNotAllowed

    data = fixture()
    tokens, lengths = data["tokens"].astype(np.int64), data["lengths"]
    o = oracle()
    for sid in range(len(lengths)):
        state = o.initial_state()
        for pos in range(int(lengths[sid])):
            try:
                state = o.advance(state, int(tokens[sid, pos]))
            except TokenNotAllowed as error:  # pragma: no cover - the failure message
                pytest.fail(f"stream {sid} position {pos}: {error}")


def test_recorded_allowed_counts_equal_the_oracle():
    data = fixture()
    tokens, lengths, allowed = data["tokens"].astype(np.int64), data["lengths"], data["allowed"]
    o = oracle()
    rng = np.random.default_rng(17)
    for sid in rng.choice(len(lengths), size=6, replace=False).tolist():
        stops = sorted(set(rng.integers(0, int(lengths[sid]), size=2).tolist()))
        state = o.initial_state()
        for pos in range(max(stops) + 1):
            if pos in stops:
                assert len(o.allowed(state)) == int(allowed[sid, pos]), (sid, pos)
            state = o.advance(state, int(tokens[sid, pos]))
