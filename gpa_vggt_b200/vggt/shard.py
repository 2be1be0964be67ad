"""Query-frame sharding of the GPA-VGGT forward across the GPUs of one node.

Each rank owns a contiguous range of S / world frames: the DINO patch embed,
the frame blocks and the DPT head are frame-local; a global block's queries
are the rank's own tokens, and the keys/values every query needs are exchanged
with NCCL all-gathers (one process per GPU, torch.distributed):

* merged blocks: the dst metric rows (so each rank matches its own src tokens
  against all dst tokens), the (node_max, node_idx) pairs of every src token
  (so every rank builds the identical global merge plan, top-r cut included);
  then each rank merges the output slots whose tokens sit in its own frames:
  an all-to-all brings it the K/V rows of the members it lacks, and the merged
  K/V of every slot is all-gathered (merge_exchange);
* frame + shared-set blocks: the shared set only (special tokens and pooled
  summaries of every frame, 30 per frame and head);
* plain global attention: K and V;
* camera head: the camera tokens of every frame.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from ..nvtx import nvtx


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
        self._flag = None
        self._peer = None

    def device_barrier(self, device=None) -> None:
        """Order the current stream against every rank's: a one-element
        all-reduce on the stream (later work waits for every rank's earlier
        work)."""
        if self._flag is None:
            self._flag = torch.zeros(1, dtype=torch.int32, device=device or torch.cuda.current_device())
        dist.all_reduce(self._flag, group=self.group)

    def peer_buffers(self, rows_bytes: int, out_bytes: int, device) -> "PeerBuffers":
        """The IPC-mapped exchange buffers, (re)created collectively when a call
        needs more room (every rank asks for the same sizes at the same call)."""
        pb = self._peer
        if pb is None or pb.rows.numel() < rows_bytes or pb.out.numel() < out_bytes:
            if pb is not None:
                rows_bytes, out_bytes = max(rows_bytes, pb.rows.numel()), max(out_bytes, pb.out.numel())
                pb.close()
            self._peer = PeerBuffers(self, rows_bytes, out_bytes, device)
        return self._peer

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

    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor, out_splits: List[int],
                   in_splits: List[int]) -> torch.Tensor:
        """Rows of inp go to the ranks in order (in_splits[i] to rank i); out
        receives out_splits[i] rows from rank i, in rank order."""
        dist.all_to_all_single(out, inp.contiguous(), out_splits, in_splits, group=self.group)
        return out

    def gather_varlen2(self, a: torch.Tensor, b: torch.Tensor, counts_a: Sequence[int],
                       counts_b: Sequence[int]):
        """Two variable-length all-gathers along dim 0 in one collective: rank i
        holds counts_a[i] rows of a and counts_b[i] rows of b (same row shape)."""
        ma, mb = max(counts_a), max(counts_b)
        pad = torch.zeros((ma + mb,) + tuple(a.shape[1:]), device=a.device, dtype=a.dtype)
        pad[: a.shape[0]] = a
        pad[ma: ma + b.shape[0]] = b
        full = self.gather(pad).view((self.world, ma + mb) + tuple(a.shape[1:]))
        ga = torch.cat([full[i, : counts_a[i]] for i in range(self.world)], 0)
        gb = torch.cat([full[i, ma: ma + counts_b[i]] for i in range(self.world)], 0)
        return ga, gb

    def gather_varlen2_async(self, a: torch.Tensor, b: torch.Tensor, counts_a: Sequence[int],
                             counts_b: Sequence[int]):
        """gather_varlen2 started on the key/value communicator.  Returns (full,
        work): after work.wait(), rank i's rows of a are full[i, :counts_a[i]]
        and its rows of b full[i, max(counts_a):max(counts_a) + counts_b[i]]."""
        ma, mb = max(counts_a), max(counts_b)
        pad = torch.zeros((ma + mb,) + tuple(a.shape[1:]), device=a.device, dtype=a.dtype)
        pad[: a.shape[0]] = a
        pad[ma: ma + b.shape[0]] = b
        full, work = self.gather_async(pad)
        return full.view((self.world, ma + mb) + tuple(a.shape[1:])), work

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


class PeerBuffers:
    """Token-row and merged-row buffers of the merged-block exchange, mapped by
    every rank of the shard (CUDA IPC over NVLink), and the device tables of
    their addresses as this process sees them (for gpa_merge_exchange_p2p).
    Created collectively; the mappings stay until close()."""

    def __init__(self, sh: FrameShard, rows_bytes: int, out_bytes: int, device):
        from .. import kernels
        self.sh = sh
        self.rows = torch.empty(rows_bytes, dtype=torch.uint8, device=device)
        self.out = torch.empty(out_bytes, dtype=torch.uint8, device=device)
        mine = (kernels.ipc_export(self.rows), kernels.ipc_export(self.out))
        every = [None] * sh.world
        dist.all_gather_object(every, mine, group=sh.group)
        self._opened = []
        rows_at, out_at = [], []
        for r, ((h_rows, o_rows), (h_out, o_out)) in enumerate(every):
            if r == sh.rank:
                rows_at.append(self.rows.data_ptr())
                out_at.append(self.out.data_ptr())
                continue
            a = kernels.ipc_open(h_rows, o_rows)
            self._opened.append((a, o_rows))
            b = kernels.ipc_open(h_out, o_out)
            self._opened.append((b, o_out))
            rows_at.append(a)
            out_at.append(b)
        self.peer_rows = torch.tensor(rows_at, dtype=torch.int64, device=device)
        self.peer_out = torch.tensor(out_at, dtype=torch.int64, device=device)

    def close(self) -> None:
        """Unmap the peers' buffers once no rank uses them (collective)."""
        from .. import kernels
        self.sh.device_barrier()
        torch.cuda.synchronize()
        for a, off in self._opened:
            kernels.ipc_close(a, off)
        self._opened = []
        self.sh.device_barrier()
        torch.cuda.synchronize()


def merge_exchange_p2p(sh: FrameShard, k: torch.Tensor, v: torch.Tensor, plan, tokens_per_frame: int,
                       dst_range, kernels) -> torch.Tensor:
    """Merged K/V rows of every output slot of `plan` on every rank, through
    peer memory: this rank's token rows [local_frames * P] of k and v ([Nl, H,
    D]) go into its shared row buffer, then one kernel per rank merges the
    slots whose token it owns (its dst ordinals `dst_range`, its unmerged src)
    from whichever rank holds the member rows and stores them into every
    rank's merged buffer -- the all-to-all, the scatter-mean and the
    all-gather of merge_exchange in one launch, bit-identical to one GPU's
    merge.  Returns [N_m, 2 * H * D] in k's dtype (K then V per slot), a view
    of the shared buffer that the next exchange overwrites."""
    Nl, H, D = k.shape
    dt = k.dtype
    C = 2 * H * D
    row_bytes = C * k.element_size()
    N = sh.frames * tokens_per_frame
    pb = sh.peer_buffers(Nl * row_bytes, N * row_bytes, k.device)
    with nvtx("exch_stage"):
        rows = pb.rows[: Nl * row_bytes].view(dt).view(Nl, 2, H, D)
        if (v.dtype == dt and k.stride() == v.stride() and k.stride(2) == 1 and k.stride(1) == D
                and v.data_ptr() == k.data_ptr() + H * D * k.element_size()):
            # K and V side by side in each token's qkv row: one 2-D copy
            rows.view(Nl, C).copy_(k.as_strided((Nl, C), (k.stride(0), 1)))
        else:
            torch.stack((k, v.to(dt)), 1, out=rows)
    with nvtx("exch_p2p"):
        sh.device_barrier()
        kernels.merge_exchange_p2p(pb.peer_rows, pb.peer_out, sh.rank, dt, sh.local * tokens_per_frame,
                                   C, plan, dst_range[0], dst_range[1])
        sh.device_barrier()
    return pb.out[: plan.n_out * row_bytes].view(dt).view(plan.n_out, C)


def merge_exchange(sh: FrameShard, rows: torch.Tensor, plan, tokens_per_frame: int,
                   kernels) -> torch.Tensor:
    """Merged rows of every output slot of `plan` (identical on every rank),
    from this rank's token rows [local_frames * P, C]: merge_local, then one
    all-gather of every rank's merged rows in slot order.  Returns [N_m, C] in
    rows' dtype."""
    own, (unm_cnt, dst_cnt, _, _) = merge_local(sh, rows, plan, tokens_per_frame, kernels)
    nu = unm_cnt[sh.rank]
    with nvtx("exch_gather"):
        unm_all, dst_all = sh.gather_varlen2(own[:nu], own[nu:], unm_cnt, dst_cnt)
        return torch.cat([unm_all, dst_all])


def merge_local(sh: FrameShard, rows: torch.Tensor, plan, tokens_per_frame: int, kernels):
    """This rank's merged output slots of `plan`, from its token rows
    [local_frames * P, C].

    Each output slot belongs to the rank whose frames hold its token (the
    unmerged src token, or the dst token); since ordinals are frame-major, a
    rank's slots are one contiguous range of unmerged slots and one of dst
    slots.  The members of a rank's dst slots that sit in other ranks' frames
    come over one all-to-all; the rank merges its slots with the same kernel
    and summation order as one GPU would (bit-identical results).  Returns
    (its merged rows: its unmerged slots, then its dst slots, in rows' dtype;
    (unmerged slots per rank, dst slots per rank, its first unmerged slot, its
    first dst slot))."""
    with nvtx("exch_index"):
        world, rank = sh.world, sh.rank
        dev = rows.device
        LP = sh.local * tokens_per_frame
        base = rank * LP
        src_pos, dst_pos = plan.src_pos.long(), plan.dst_pos.long()
        seg = plan.seg_start.long()
        unm_owner = torch.div(src_pos[plan.unm_src.long()], LP, rounding_mode="floor")
        dst_owner = torch.div(dst_pos, LP, rounding_mode="floor")
        mem_dst = torch.repeat_interleave(torch.arange(plan.num_dst, device=dev), seg[1:] - seg[:-1],
                                          output_size=plan.seg_src.numel())
        mem_src = plan.seg_src.long()
        mem_owner = dst_owner[mem_dst]
        mem_rank = torch.div(src_pos[mem_src], LP, rounding_mode="floor")
        move = mem_owner != mem_rank
        # one small device-to-host read: slot counts per rank and the row matrix
        # (counted with scatter-adds into fixed-size bins, which need no read)
        def count(idx, bins, weight=None):
            out = torch.zeros(bins, device=dev, dtype=torch.long)
            w = torch.ones_like(idx) if weight is None else weight.long()
            return out.scatter_add_(0, idx, w)
        cnt = torch.cat([count(unm_owner, world), count(dst_owner, world),
                         count(mem_rank * world + mem_owner, world * world, move)]).cpu()
        unm_cnt, dst_cnt = cnt[:world].tolist(), cnt[world:2 * world].tolist()
        mat = cnt[2 * world:].view(world, world)
    with nvtx("exch_a2a"):
        # send: this rank's member rows that other ranks' slots need, by owner rank
        # (a stable sort on the owner, others keyed past the end, then the known
        # count: no further device-to-host read)
        n_send, n_recv = int(mat[rank].sum()), int(mat[:, rank].sum())
        key = torch.where(move & (mem_rank == rank), mem_owner, world)
        send_m = torch.sort(key, stable=True).indices[:n_send]
        send = rows[src_pos[mem_src[send_m]] - base]
        recv = torch.empty((n_recv,) + tuple(rows.shape[1:]), device=dev, dtype=rows.dtype)
        sh.all_to_all(recv, send, mat[:, rank].tolist(), mat[rank].tolist())
    with nvtx("exch_merge"):
        # receive: the members of this rank's slots from elsewhere, by source rank
        key = torch.where(move & (mem_owner == rank), mem_rank, world)
        recv_m = torch.sort(key, stable=True).indices[:n_recv]
        buf = torch.cat([rows, recv]) if recv.shape[0] else rows
        src_map = (src_pos - base).to(torch.int32)
        src_map[mem_src[recv_m]] = torch.arange(LP, LP + recv_m.numel(), device=dev, dtype=torch.int32)
        dst_map = (dst_pos - base).to(torch.int32)
        u0, e0 = sum(unm_cnt[:rank]), sum(dst_cnt[:rank])
        nu, nd = unm_cnt[rank], dst_cnt[rank]
        out = torch.empty((nu + nd,) + tuple(rows.shape[1:]), device=dev, dtype=rows.dtype)
        if nu:
            kernels.merge_kv_rows(buf, src_map, None, plan.unm_src[u0:u0 + nu], None, None, 0, out[:nu])
        if nd:
            kernels.merge_kv_rows(buf, src_map, dst_map[e0:], None, plan.seg_start[e0:], plan.seg_src,
                                  nd, out[nu:])
    return out, (unm_cnt, dst_cnt, u0, e0)

