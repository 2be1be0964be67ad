"""C ABI library: builds, loads and exports every symbol of include/gpa_b200.h.
These tests launch nothing (no GPU needed)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "gpa_b200.h"


@pytest.fixture(scope="module")
def lib():
    from gpa_vggt_b200 import build, _lib
    build.build()
    return _lib.load()


def header_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^GPA_API\s+[\w\s\*]+?\b(gpa_\w+)\s*\(", text, flags=re.M)))


def test_every_header_symbol_is_exported(lib):
    syms = header_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in the header but not exported"


def test_binding_covers_header():
    from gpa_vggt_b200 import _lib
    assert set(header_symbols()) <= set(_lib.SIGNATURES)


def test_version_and_host_only_entry_points(lib):
    assert lib.gpa_version() >= 100
    nd, ns = ctypes.c_int(), ctypes.c_int()
    assert lib.gpa_merge_counts(200, 37, 37, 2, 2, 5, 0, ctypes.byref(nd), ctypes.byref(ns)) == 0
    assert (nd.value, ns.value) == (66845, 207955)   # the S=200 split of the survey table
    assert lib.gpa_merge_counts(4, 37, 37, 2, 2, 5, 0, ctypes.byref(nd), ctypes.byref(ns)) == 0
    assert (nd.value, ns.value) == (2361, 3135)
    assert lib.gpa_merge_plan_workspace_bytes(207955, 66845) > 0


def test_argument_errors_are_reported_without_launching(lib):
    from gpa_vggt_b200 import _lib
    rc = lib.gpa_attention_keybias(None, None, None, None, 1, 1, 4, 4, 32, *([0] * 11), 0.1,
                                   None, 0, 0, 0, None, 0, 0, None, None)
    assert rc == 3
    assert b"head_dim" in lib.gpa_last_error()
    rc = lib.gpa_sim_argmax(None, None, 1, 4, 4, 100, 0, 0, 0, 0, None, None, None, None)
    assert rc == 3
    with pytest.raises(_lib.GpaError):
        _lib.check(rc, "gpa_sim_argmax")
