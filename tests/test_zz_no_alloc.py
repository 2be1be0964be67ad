"""gpa_merge_plan_noalloc: the merge plan for callers that cannot allocate
device memory (hosts whose own arena owns the GPU's memory, FFI callers with no
allocator).  It must produce exactly what gpa_merge_plan produces with a
caller-provided workspace, call after call, although its scratch is one fixed
array that every call reuses.

This file is collected last on purpose; it runs alone or after the others.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def lib():
    from gpa_vggt_b200 import build, _lib
    build.build()
    return _lib.load()


def _inputs(ns, nd, seed):
    g = torch.Generator().manual_seed(seed)
    node_max = torch.randint(0, 64, (ns,), generator=g).float() / 64   # many ties at the cut
    node_idx = torch.randint(0, nd, (ns,), generator=g)
    node_idx[: ns // 20] = 7                                             # one hub group
    return node_max.to(DEV), node_idx.int().to(DEV)


def _noalloc_plan(lib, node_max, node_idx, nd, r):
    """Call the no-allocation entry point through the C ABI."""
    from gpa_vggt_b200 import _lib
    ns = node_max.numel()
    r = max(0, min(r, ns))
    unm = torch.full((max(ns - r, 1),), -1, device=DEV, dtype=torch.int32)
    seg_start = torch.full((nd + 1,), -1, device=DEV, dtype=torch.int32)
    seg_src = torch.full((max(r, 1),), -1, device=DEV, dtype=torch.int32)
    counts = torch.full((ns - r + nd,), -1.0, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.gpa_merge_plan_noalloc(_lib.ptr(node_max), _lib.ptr(node_idx), ns, nd, r,
                                    _lib.ptr(unm), _lib.ptr(seg_start), _lib.ptr(seg_src),
                                    _lib.ptr(counts), stream)
    _lib.check(rc, "gpa_merge_plan_noalloc")
    return unm[: ns - r], seg_start, seg_src[:r], counts


@pytest.mark.parametrize("ns,nd,ratios,seeds", [
    (207955, 66845, (0.2, 0.98), (1, 2)),   # the S=200 split: core block, then aggressive
    (3135, 2361, (0.5, 0.05), (3, 4)),      # S=4
])
def test_noalloc_plan_matches_workspace_plan_twice_in_a_row(lib, ns, nd, ratios, seeds):
    from gpa_vggt_b200 import kernels
    dst_pos = torch.arange(nd, device=DEV, dtype=torch.int32)
    src_pos = torch.arange(nd, nd + ns, device=DEV, dtype=torch.int32)
    for ratio, seed in zip(ratios, seeds):   # two calls in a row on the same scratch
        node_max, node_idx = _inputs(ns, nd, seed)
        r = int((ns + nd) * ratio)
        want = kernels.merge_plan(node_max, node_idx, r, dst_pos, src_pos)
        unm, seg_start, seg_src, counts = _noalloc_plan(lib, node_max, node_idx, nd, r)
        torch.cuda.synchronize()
        assert torch.equal(unm, want.unm_src)
        assert torch.equal(seg_start, want.seg_start)
        assert torch.equal(seg_src, want.seg_src)
        assert torch.equal(counts, want.counts)


def test_noalloc_plan_allocates_nothing(lib):
    """After a first call, a call changes neither torch's allocation count nor
    the device's free memory (cudaMemGetInfo): the scratch is the library's
    fixed array, not an allocation."""
    from gpa_vggt_b200 import _lib
    ns, nd = 207955, 66845
    node_max, node_idx = _inputs(ns, nd, 5)
    r = int((ns + nd) * 0.2)
    unm = torch.empty(ns - r, device=DEV, dtype=torch.int32)
    seg_start = torch.empty(nd + 1, device=DEV, dtype=torch.int32)
    seg_src = torch.empty(r, device=DEV, dtype=torch.int32)
    counts = torch.empty(ns - r + nd, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = (_lib.ptr(node_max), _lib.ptr(node_idx), ns, nd, r, _lib.ptr(unm), _lib.ptr(seg_start),
            _lib.ptr(seg_src), _lib.ptr(counts), stream)
    _lib.check(lib.gpa_merge_plan_noalloc(*args), "gpa_merge_plan_noalloc")   # warm-up
    torch.cuda.synchronize()
    n_alloc = torch.cuda.memory_stats()["allocation.all.allocated"]
    free0, _ = torch.cuda.mem_get_info()
    _lib.check(lib.gpa_merge_plan_noalloc(*args), "gpa_merge_plan_noalloc")
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_stats()["allocation.all.allocated"] == n_alloc
    assert free1 == free0


def test_noalloc_plan_rejects_sizes_beyond_its_scratch(lib):
    from gpa_vggt_b200 import _lib
    big = 4_000_000
    assert lib.gpa_merge_plan_workspace_bytes(big, 100) > (16 << 20)
    rc = lib.gpa_merge_plan_noalloc(None, None, big, 100, 10, None, None, None, None, None)
    assert rc == 3
    assert b"scratch" in lib.gpa_last_error()
    with pytest.raises(_lib.GpaError):
        _lib.check(rc, "gpa_merge_plan_noalloc")
