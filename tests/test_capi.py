"""The C ABI library: it loads, exports every function include/xgraph_b200.h declares, and
its host-side argument checks raise the reference's error types (no GPU work)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared() -> list[str]:
    text = (ROOT / "include" / "xgraph_b200.h").read_text()
    return sorted(set(re.findall(r"^XG_API\s+(?:int|const char\*|int32_t)\s+(xg_\w+)\(", text, flags=re.M)))


def test_header_declares_the_engine_lifecycle():
    names = declared()
    for name in ("xg_create", "xg_begin", "xg_sync", "xg_advance", "xg_apply_mask", "xg_states_host"):
        assert name in names


def test_library_exports_every_declared_function():
    from xgraph_b200.build import build

    path = build()
    lib = ctypes.CDLL(str(path))
    for name in declared():
        assert hasattr(lib, name), name
    lib.xg_abi_version.restype = ctypes.c_int32
    from xgraph_b200.engine import ABI_VERSION

    assert lib.xg_abi_version() == ABI_VERSION
    assert f"#define XG_ABI_VERSION {ABI_VERSION}\n" in (ROOT / "include" / "xgraph_b200.h").read_text()


def test_ctypes_structures_match_the_header(tmp_path):
    """The ctypes mirrors of XgOptions and XgLayout have the header's field offsets and
    sizes (a C program built with gcc against the header prints them)."""
    import subprocess

    from xgraph_b200.tables import XgLayout, XgOptions

    lines = []
    for struct in (XgOptions, XgLayout):
        name = struct.__name__
        lines.append(f'printf("{name} size %zu\\n", sizeof({name}));')
        for field, _ in struct._fields_:
            lines.append(f'printf("{name} {field} %zu\\n", offsetof({name}, {field}));')
    source = tmp_path / "offsets.c"
    source.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "xgraph_b200.h"\nint main(void) {\n'
                      + "\n".join(lines) + "\nreturn 0;\n}\n")
    binary = tmp_path / "offsets"
    subprocess.run(["gcc", "-std=c11", "-I", str(ROOT / "include"), str(source), "-o", str(binary)], check=True)
    printed = subprocess.run([str(binary)], check=True, capture_output=True, text=True).stdout.split("\n")
    for struct in (XgOptions, XgLayout):
        name = struct.__name__
        assert f"{name} size {ctypes.sizeof(struct)}" in printed
        for field, _ in struct._fields_:
            assert f"{name} {field} {getattr(struct, field).offset}" in printed, (name, field)


def test_null_engine_calls_fail_with_einval():
    from xgraph_b200.build import build

    lib = ctypes.CDLL(str(build()))
    lib.xg_reset.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    lib.xg_last_error.restype = ctypes.c_char_p
    assert lib.xg_reset(None, None) == 1
    assert b"null" in lib.xg_last_error()


def test_engine_constructor_fails_loudly_without_the_library(monkeypatch, tmp_path):
    import xgraph_b200.engine as engine

    monkeypatch.setattr(engine, "_lib", None)
    with pytest.raises(engine.EngineUnavailable):
        engine.load_library(tmp_path / "missing.so")


def test_adjacency_build_rejects_bad_arguments_before_any_device_work():
    """xg_build_adjacency checks its outputs, sizes and pointers on the host and fails with
    XG_EINVAL (ValueError) before touching the GPU."""
    from xgraph_b200.engine import _check, load_library

    lib = load_library()
    edges, unwritable = ctypes.c_int64(), ctypes.c_int64()
    fake = ctypes.c_void_p(16)  # never dereferenced: every call below fails its host checks first
    cases = [
        ((fake, fake, fake, 1, fake, fake, 2, 2, fake, 1, 0, None, None, None, None, ctypes.byref(unwritable), None),
         "null edges"),
        ((fake, fake, fake, -1, fake, fake, 2, 2, fake, 1, 0, None, None, None, ctypes.byref(edges),
          ctypes.byref(unwritable), None), "negative size"),
        ((None, fake, fake, 3, fake, fake, 2, 2, fake, 1, 0, None, None, None, ctypes.byref(edges),
          ctypes.byref(unwritable), None), "null triples"),
        ((fake, fake, fake, 3, None, fake, 2, 2, fake, 1, 0, None, None, None, ctypes.byref(edges),
          ctypes.byref(unwritable), None), "null label rows"),
        ((fake, fake, fake, 3, fake, fake, 1 << 30, 1 << 30, fake, 1 << 30, 0, None, None, None, ctypes.byref(edges),
          ctypes.byref(unwritable), None), "too large"),
    ]
    for args, message in cases:
        with pytest.raises(ValueError, match=message):
            _check(lib.xg_build_adjacency(*args))
