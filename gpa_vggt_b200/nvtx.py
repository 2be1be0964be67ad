"""NVTX ranges around the forward's blocks, for profilers (ncu --nvtx,
nsys): set GPA_NVTX=1.  Off by default, where a range costs nothing."""
from __future__ import annotations

import contextlib
import os

import torch

ENABLED = os.environ.get("GPA_NVTX", "0") == "1"


@contextlib.contextmanager
def nvtx(name: str):
    if not ENABLED:
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
