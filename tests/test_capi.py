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


def test_argument_errors_of_the_block_kernels(lib):
    """The fused block/head kernels validate shapes and alignment before any
    launch (a misaligned pointer never reaches a 16-byte vector access)."""
    from gpa_vggt_b200 import _lib
    lib = _lib.load()
    odd = ctypes.c_void_p(8)      # not 16-byte aligned
    ok = ctypes.c_void_p(256)
    # GELU: element count must be a multiple of 8; buffers 16-byte aligned
    assert lib.gpa_gelu_bf16(ok, 12, ok, None) == 3
    assert b"multiple of 8" in lib.gpa_last_error()
    assert lib.gpa_gelu_bf16(odd, 16, ok, None) == 1
    assert lib.gpa_gelu_bf16(ok, 0, ok, None) == 0          # empty: nothing to do
    # residual + LayerScale: cols % 8, aligned rows
    assert lib.gpa_residual_scale_bf16(ok, 1024, ok, 1024, ok, 4, 1020, ok, 1024, None) == 3
    assert lib.gpa_residual_scale_bf16(ok, 1021, ok, 1024, ok, 4, 1024, ok, 1024, None) == 1
    # DPT resize: dtype, channels % 8, channels-last alignment
    f32, bf16 = _lib.GPA_DTYPE_F32, _lib.GPA_DTYPE_BF16
    assert lib.gpa_upsample_bilinear_bf16(ok, 7, 1, 8, 4, 4, 128, 32, 8, None, 0, 0, 0, 8, 8, ok,
                                          512, 64, 8, None) == 1
    assert lib.gpa_upsample_bilinear_bf16(ok, bf16, 1, 12, 4, 4, 192, 48, 12, None, 0, 0, 0, 8, 8, ok,
                                          768, 96, 12, None) == 3
    assert lib.gpa_upsample_bilinear_bf16(ok, f32, 1, 8, 4, 4, 130, 32, 8, None, 0, 0, 0, 8, 8, ok,
                                          512, 64, 8, None) == 1
    assert b"aligned" in lib.gpa_last_error()
    # LSE combine: strides in multiples of 8 elements
    A = _lib.i64array
    assert lib.gpa_lse_combine(2, 2, 4, 64, ok, A([64, 512, 4]), ok, A([8, 4, 1]), ok, A([64, 512, 128]),
                               ok, A([8, 4, 1]), ok, A([64, 512, 128]), None) == 1


def test_argument_errors_of_the_exchange_entry_points(lib):
    """The peer-memory exchange and its IPC helpers reject bad arguments before
    any CUDA call (so this runs without a GPU)."""
    I, I64, P = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p
    fake = P(16)   # never dereferenced: every call below fails validation first

    def xch(world, rank, dtype, rows, elems, unm, nd, lo, hi, seg_src=fake):
        return lib.gpa_merge_exchange_p2p(fake, fake, I(world), I(rank), I(dtype), I(rows), I(elems),
                                          fake, fake, fake, I(unm), fake, seg_src, I(nd), I(lo), I(hi),
                                          None, None)
    assert xch(0, 0, 1, 10, 2048, 0, 4, 0, 4) == 1            # world < 1
    assert xch(9, 0, 1, 10, 2048, 0, 4, 0, 4) == 1            # world > 8
    assert xch(2, 2, 1, 10, 2048, 0, 4, 0, 4) == 1            # rank outside the world
    assert b"world" in lib.gpa_last_error()
    assert xch(2, 0, 1, 10, 2052, 0, 4, 0, 4) == 3            # row not a multiple of 8
    assert xch(2, 0, 1, 10, 4096, 0, 4, 0, 4) == 3            # row above 2048 elements
    assert xch(2, 0, 7, 10, 2048, 0, 4, 0, 4) == 1            # dtype
    assert xch(2, 0, 1, 10, 2048, 0, 4, 3, 2) == 1            # dst range reversed
    assert xch(2, 0, 1, 10, 2048, 0, 4, 0, 5) == 1            # dst range past num_dst
    assert xch(2, 0, 1, 0, 2048, 0, 4, 0, 4) == 1             # no rows per rank
    assert xch(2, 0, 1, 10, 2048, 0, 4, 0, 4, seg_src=None) == 1   # null member list
    assert b"null" in lib.gpa_last_error()
    assert lib.gpa_merge_exchange_p2p(P(17), fake, I(2), I(0), I(1), I(10), I(2048), fake, fake, fake,
                                      I(0), fake, fake, I(4), I(0), I(4), None, None) == 1   # unaligned table
    assert lib.gpa_ipc_export(None, None, None) == 1
    assert lib.gpa_ipc_open(None, I64(0), None) == 1
    assert lib.gpa_ipc_open(ctypes.create_string_buffer(64), I64(-1), ctypes.byref(P())) == 1
    assert lib.gpa_ipc_close(None, I64(0)) == 1
