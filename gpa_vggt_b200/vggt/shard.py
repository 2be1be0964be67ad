"""Query-frame sharding of the GPA-VGGT forward across the GPUs of one node.

Each rank owns a contiguous range of S / world frames: the DINO patch embed,
the frame blocks and the DPT head are frame-local; a global block's queries
are the rank's own tokens, and the keys/values every query needs are exchanged
with NCCL all-gathers (one process per GPU, torch.distributed):

* merged blocks: the dst metric rows (so each rank matches its own src tokens
  against all dst tokens), the (node_max, node_idx) pairs of every src token
  (so every rank builds the identical global merge plan, top-r cut included),
  then K and V, which every rank merges itself;
* frame + shared-set blocks: the shared set only (special tokens and pooled
  summaries of every frame, 30 per frame and head);
* plain global attention: K and V;
* camera head: the camera tokens of every frame.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist


class FrameShard:
    """Frames [f0, f1) of S on this rank; collectives over `group`."""

    def __init__(self, frames: int, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if frames % self.world:
            raise ValueError(f"FrameShard: {frames} frames do not split over {self.world} ranks")
        self.frames = frames
        self.local = frames // self.world
        self.f0 = self.rank * self.local
        self.f1 = self.f0 + self.local
        # a second communicator for the bulk key/value exchange, so it runs on its
        # own stream while the small match-result gathers and kernels proceed
        # (every rank constructs the shard, so every rank joins the new group)
        self.kv_group = None
        if self.world > 1:
            ranks = dist.get_process_group_ranks(group) if group is not None else list(range(self.world))
            self.kv_group = dist.new_group(ranks)

    @property
    def active(self) -> bool:
        return self.world > 1

    def gather(self, t: torch.Tensor) -> torch.Tensor:
        """All-gather equal-size tensors along dim 0 (rank order)."""
        t = t.contiguous()
        out = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), device=t.device, dtype=t.dtype)
        dist.all_gather_into_tensor(out, t, group=self.group)
        return out

    def gather_async(self, t: torch.Tensor):
        """Start an all-gather of equal-size tensors along dim 0 on the key/value
        communicator; returns (output, work).  work.wait() orders the current
        stream after the exchange."""
        t = t.contiguous()
        out = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), device=t.device, dtype=t.dtype)
        work = dist.all_gather_into_tensor(out, t, group=self.kv_group, async_op=True)
        return out, work

    def gather_varlen(self, t: torch.Tensor, counts: Sequence[int]) -> torch.Tensor:
        """All-gather along dim 0 when rank i holds counts[i] rows."""
        m = max(counts)
        pad = torch.zeros((m,) + tuple(t.shape[1:]), device=t.device, dtype=t.dtype)
        pad[: t.shape[0]] = t
        full = self.gather(pad).view((self.world, m) + tuple(t.shape[1:]))
        return torch.cat([full[i, : counts[i]] for i in range(self.world)], 0)

    # -- the bipartite split's per-frame counts (merging/merge.py:87-166) --------
    @staticmethod
    def role_counts(frame: int, P: int, dst_per_frame: int):
        """(dst, src) tokens of one frame: frame 0 is all dst."""
        return (P, 0) if frame == 0 else (dst_per_frame, P - dst_per_frame)

    def role_ranges(self, P: int, dst_per_frame: int):
        """Per rank: (dst ordinal range, src ordinal range), frame-major ordinals."""
        out = []
        d = s = 0
        for r in range(self.world):
            d0, s0 = d, s
            for f in range(r * self.local, (r + 1) * self.local):
                nd, ns = self.role_counts(f, P, dst_per_frame)
                d += nd
                s += ns
            out.append(((d0, d), (s0, s)))
        return out
