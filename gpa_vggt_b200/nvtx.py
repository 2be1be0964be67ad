"""Markers around the forward's blocks, off by default (a no-op then):

* GPA_NVTX=1: NVTX ranges, for profilers (ncu --nvtx, nsys);
* GPA_BLOCK_TIMING=1: CUDA events around each marked range on the current
  stream; block_times() returns the device milliseconds per range name,
  summed over calls since the last reset (synchronises when read)."""
from __future__ import annotations

import contextlib
import os

import torch

ENABLED = os.environ.get("GPA_NVTX", "0") == "1"
TIMING = os.environ.get("GPA_BLOCK_TIMING", "0") == "1"
_events = []


@contextlib.contextmanager
def nvtx(name: str):
    if not (ENABLED or TIMING):
        yield
        return
    if ENABLED:
        torch.cuda.nvtx.range_push(name)
    if TIMING:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    try:
        yield
    finally:
        if TIMING:
            e1.record()
            _events.append((name, e0, e1))
        if ENABLED:
            torch.cuda.nvtx.range_pop()


def block_times(reset: bool = True) -> dict:
    """{range name: device ms summed over its calls} of the timed ranges."""
    torch.cuda.synchronize()
    out = {}
    for name, e0, e1 in _events:
        out[name] = out.get(name, 0.0) + e0.elapsed_time(e1)
    if reset:
        _events.clear()
    return out
