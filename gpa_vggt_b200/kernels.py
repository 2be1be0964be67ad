"""Torch-facing wrappers of the C ABI: validate tensors, allocate outputs,
launch on the current stream.  One function per entry point of
``include/gpa_b200.h``; the reference-shaped API lives in ``merging/`` and
``layers/`` on top of these.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import call, ptr, stream_of, require_cuda, aligned

BF16 = torch.bfloat16
F32 = torch.float32

# Every pipelined kernel (similarity, attention) writes a nonzero code into a
# device status word when one of its pipeline waits gives up (the kernel then
# drains what it has in flight and returns, its output invalid).
# * By default the launches share one persistent word per device, and
#   check_device_status() reads it at a point that synchronises anyway (the
#   end of the aggregator's forward): a timed-out wait raises there.
# * GPA_CHECK_STATUS=1 gives every launch its own word and reads it right after
#   the launch (synchronises every launch; the tests set it).
CHECK_STATUS = os.environ.get("GPA_CHECK_STATUS", "0") == "1"
_DEVICE_STATUS = {}


# When set to a list, every attention launch appends (start event, end event,
# algorithmic flops, algorithmic bytes, key count) recorded on its stream
# (bench.py's roofline).
ATTN_TIMING = None


class KernelTimeout(RuntimeError):
    """A kernel's pipeline wait gave up (device status word set)."""


def device_status_word(device) -> torch.Tensor:
    """The persistent status word of `device` (int32, zero while all is well)."""
    dev = torch.device(device)
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    w = _DEVICE_STATUS.get(key)
    if w is None:
        w = torch.zeros(1, device=torch.device("cuda", key), dtype=torch.int32)
        _DEVICE_STATUS[key] = w
    return w


def _status_text(v: int) -> str:
    """The device status bits: 1 = a pipeline wait gave up, 2 = an index
    outside its buffer was skipped."""
    parts = []
    if v & 1:
        parts.append("a kernel's pipeline wait gave up")
    if v & 2:
        parts.append("a kernel met an index outside its buffer")
    return "; ".join(parts) or "unknown status"


def check_device_status(device, what: str = "forward") -> None:
    """Read (synchronises) and clear the device's persistent status word;
    raise KernelTimeout if a kernel recorded a wait that gave up or skipped an
    out-of-range index."""
    w = device_status_word(device)
    v = int(w.item())
    if v != 0:
        w.zero_()
        raise KernelTimeout(f"{what}: device status {v} ({_status_text(v)}; "
                            "its output is invalid)")


def _status_word(status, device):
    if status is None:
        if CHECK_STATUS:
            return torch.zeros(1, device=device, dtype=torch.int32), True
        return device_status_word(device), False
    return status, False


def _check_status(status, what):
    v = int(status.item())
    if v != 0:
        raise KernelTimeout(f"{what}: device status {v} ({_status_text(v)})")


def wait_selftest(limit_ns: int, device="cuda") -> None:
    """Run gpa_wait_selftest (a bounded wait on a barrier nothing arrives on)
    with its own status word; raises KernelTimeout as a real timeout would."""
    status = torch.zeros(1, device=device, dtype=torch.int32)
    call("gpa_wait_selftest", ctypes.c_uint64(int(limit_ns)), ptr(status),
         _lib._vp(torch.cuda.current_stream(torch.device(device)).cuda_stream))
    _check_status(status, "gpa_wait_selftest")


def _dt(t: torch.Tensor) -> int:
    if t.dtype == F32:
        return _lib.GPA_DTYPE_F32
    if t.dtype == BF16:
        return _lib.GPA_DTYPE_BF16
    raise TypeError(f"unsupported dtype {t.dtype} (bf16 or fp32)")


def _tma_ok(t: torch.Tensor) -> bool:
    """Innermost dim contiguous, other strides multiples of 8 elements, 16B base."""
    if t.stride(-1) != 1 or not aligned(t):
        return False
    return all(s % 8 == 0 for s, n in zip(t.stride()[:-1], t.shape[:-1]) if n > 1)


def sim_argmax(a: torch.Tensor, b: torch.Tensor, status: Optional[torch.Tensor] = None):
    """node_max [B,M] fp32, node_idx [B,M] int32 of a [B,M,D] vs b [B,N,D] (bf16)."""
    require_cuda(a, b, what="sim_argmax")
    if a.dtype != BF16 or b.dtype != BF16:
        raise TypeError("sim_argmax: a and b must be bf16")
    if not _tma_ok(a):
        a = a.contiguous()
    if not _tma_ok(b):
        b = b.contiguous()
    B, M, D = a.shape
    N = b.shape[1]
    node_max = torch.empty(B, M, device=a.device, dtype=F32)
    node_idx = torch.empty(B, M, device=a.device, dtype=torch.int32)
    status, own = _status_word(status, a.device)
    call("gpa_sim_argmax", ptr(a), ptr(b), B, M, N, D, a.stride(0), a.stride(1), b.stride(0),
         b.stride(1), ptr(node_max), ptr(node_idx), ptr(status), stream_of(a))
    if own:
        _check_status(status, "gpa_sim_argmax")
    return node_max, node_idx


def merge_counts(num_imgs, w, h, sx, sy, num_special, no_rand):
    nd, ns = ctypes.c_int(), ctypes.c_int()
    call("gpa_merge_counts", num_imgs, w, h, sx, sy, num_special, int(bool(no_rand)),
         ctypes.byref(nd), ctypes.byref(ns))
    return nd.value, ns.value


def merge_roles(rand_idx: Optional[torch.Tensor], num_imgs, w, h, sx, sy, num_special, no_rand,
                device):
    """dst_pos [num_dst], src_pos [num_src], slot [N] (int32, device)."""
    nd, ns = merge_counts(num_imgs, w, h, sx, sy, num_special, no_rand)
    N = nd + ns
    dst_pos = torch.empty(nd, device=device, dtype=torch.int32)
    src_pos = torch.empty(max(ns, 1), device=device, dtype=torch.int32)
    slot = torch.empty(N, device=device, dtype=torch.int32)
    if rand_idx is not None:
        require_cuda(rand_idx, what="merge_roles")
        rand_idx = rand_idx.to(torch.int64).contiguous()
    call("gpa_merge_roles", ptr(rand_idx), num_imgs, w, h, sx, sy, num_special,
         int(bool(no_rand)), ptr(dst_pos), ptr(src_pos), ptr(slot),
         _lib._vp(torch.cuda.current_stream(device).cuda_stream))
    return dst_pos, src_pos[:ns], slot


def metric_split(metric: torch.Tensor, src_pos, dst_pos):
    """Row-normalised bf16 a (src rows) and b (dst rows) of metric [N, d]."""
    require_cuda(metric, what="metric_split")
    if metric.stride(-1) != 1 or metric.stride(0) % 8 or not aligned(metric):
        metric = metric.contiguous()
    N, d = metric.shape
    ns, nd = src_pos.numel(), dst_pos.numel()
    a = torch.empty(ns, d, device=metric.device, dtype=BF16)
    b = torch.empty(nd, d, device=metric.device, dtype=BF16)
    call("gpa_metric_split", ptr(metric), _dt(metric), metric.stride(0), d, ptr(src_pos), ns,
         ptr(dst_pos), nd, ptr(a), ptr(b), stream_of(metric))
    return a, b


def proj_norm_split(x: torch.Tensor, proj_t: torch.Tensor, slot: torch.Tensor, num_src: int,
                    num_dst: int, status: Optional[torch.Tensor] = None):
    """bf16 a [num_src, 128] (src rows) and b [num_dst, 128] (dst rows) of
    normalise(bf16(x @ proj)) for x [T, K] bf16 and proj_t = proj^T [128, K]
    bf16, routed by the role slot map [T] of merge_roles (one tcgen05 kernel)."""
    require_cuda(x, proj_t, slot, what="proj_norm_split")
    if x.dtype != BF16 or proj_t.dtype != BF16 or slot.dtype != torch.int32:
        raise TypeError("proj_norm_split: bf16 x and proj_t, int32 slot")
    if x.stride(-1) != 1 or x.stride(0) % 8 or not aligned(x):
        x = x.contiguous()
    proj_t = proj_t.contiguous()
    T, K = x.shape
    if tuple(proj_t.shape) != (128, K) or slot.numel() != T:
        raise ValueError("proj_norm_split: proj_t must be [128, K] and slot [T]")
    a = torch.empty(num_src, 128, device=x.device, dtype=BF16)
    b = torch.empty(num_dst, 128, device=x.device, dtype=BF16)
    status, own = _status_word(status, x.device)
    call("gpa_proj_norm_split", ptr(x), x.stride(0), T, K, ptr(proj_t), ptr(slot.contiguous()),
         ptr(a), ptr(b), ptr(status), stream_of(x))
    if own:
        _check_status(status, "gpa_proj_norm_split")
    return a, b


@dataclass
class MergePlan:
    """Device arrays describing one bipartite merge (B == 1)."""
    num_src: int
    num_dst: int
    r: int
    dst_pos: torch.Tensor     # [num_dst] int32, absolute positions of dst tokens
    src_pos: torch.Tensor     # [num_src] int32, absolute positions of src tokens
    unm_src: torch.Tensor     # [num_src - r] int32, unmerged src ordinals
    seg_start: torch.Tensor   # [num_dst + 1] int32
    seg_src: torch.Tensor     # [r] int32
    counts: torch.Tensor      # [N_m] fp32
    node_max: Optional[torch.Tensor] = None
    node_idx: Optional[torch.Tensor] = None

    @property
    def unm_len(self) -> int:
        return self.num_src - self.r

    @property
    def n_out(self) -> int:
        return self.unm_len + self.num_dst


def merge_plan(node_max, node_idx, r: int, dst_pos, src_pos) -> MergePlan:
    require_cuda(node_max, node_idx, what="merge_plan")
    dev = node_max.device
    ns, nd = src_pos.numel(), dst_pos.numel()
    r = max(0, min(int(r), ns))
    unm = torch.empty(max(ns - r, 1), device=dev, dtype=torch.int32)
    seg_start = torch.empty(nd + 1, device=dev, dtype=torch.int32)
    seg_src = torch.empty(max(r, 1), device=dev, dtype=torch.int32)
    counts = torch.empty(ns - r + nd, device=dev, dtype=F32)
    wsb = _lib.load().gpa_merge_plan_workspace_bytes(ns, nd)
    ws = torch.empty(wsb, device=dev, dtype=torch.uint8)
    nmx = node_max.reshape(-1).contiguous() if ns else node_max
    nix = node_idx.reshape(-1).to(torch.int32).contiguous() if ns else node_idx
    call("gpa_merge_plan", ptr(nmx), ptr(nix), ns, nd, r, ptr(unm), ptr(seg_start), ptr(seg_src),
         ptr(counts), ptr(ws), wsb, stream_of(counts))
    return MergePlan(ns, nd, r, dst_pos, src_pos, unm[: ns - r], seg_start, seg_src[:r], counts,
                     node_max, node_idx)


def merge_kv(t: torch.Tensor, plan: MergePlan, mean: bool = True, out: Optional[torch.Tensor] = None,
             log_counts: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Merge t [H, N, D] (any strides, innermost contiguous) -> [H, N_m, D]."""
    require_cuda(t, what="merge_kv")
    H, N, D = t.shape
    if t.stride(-1) != 1 or t.stride(0) % 8 or t.stride(1) % 8 or not aligned(t):
        t = t.contiguous()
    if out is None:
        out = torch.empty(H, plan.n_out, D, device=t.device, dtype=t.dtype)
    call("gpa_merge_kv_mean", ptr(t), _dt(t), H, N, D, t.stride(0), t.stride(1), ptr(plan.src_pos),
         ptr(plan.dst_pos), ptr(plan.unm_src), plan.unm_len, ptr(plan.seg_start), ptr(plan.seg_src),
         plan.num_dst, int(mean), ptr(log_counts), ptr(out), out.stride(0), out.stride(1),
         stream_of(t))
    return out


def merge_kv_rows(rows: torch.Tensor, src_map: torch.Tensor, dst_map: Optional[torch.Tensor],
                  unm_src: Optional[torch.Tensor], seg_start: Optional[torch.Tensor],
                  seg_src: Optional[torch.Tensor], num_dst: int, out: torch.Tensor,
                  mean: bool = True) -> torch.Tensor:
    """Merge a contiguous range of a plan's slots from a token-major row buffer
    rows [R, C]: the unmerged slots of unm_src (src ordinals), then num_dst dst
    slots whose dst rows are dst_map[0..num_dst) and whose members are
    seg_src[seg_start[j]:seg_start[j+1]] (seg_start already offset to the
    range's first slot).  src_map / dst_map give each ordinal's row in `rows`.
    out [n_unm + num_dst, C] receives the slots in that order (same kernel and
    summation order as merge_kv)."""
    require_cuda(rows, out, what="merge_kv_rows")
    R, C = rows.shape
    if rows.stride(1) != 1 or rows.stride(0) % 8 or out.stride(1) != 1 or out.stride(0) % 8:
        raise ValueError("merge_kv_rows: rows and out must be row-major with 8-element-aligned rows")
    n_unm = 0 if unm_src is None else unm_src.numel()
    if n_unm + num_dst == 0:
        return out
    call("gpa_merge_kv_mean", ptr(rows), _dt(rows), 1, R, C, 0, rows.stride(0), ptr(src_map),
         ptr(dst_map), ptr(unm_src), n_unm, ptr(seg_start), ptr(seg_src), int(num_dst), int(mean),
         None, ptr(out), 0, out.stride(0), stream_of(rows))
    return out


def ipc_export(t: torch.Tensor):
    """(64-byte CUDA IPC handle of t's allocation, t's byte offset in it)."""
    require_cuda(t, what="ipc_export")
    h = ctypes.create_string_buffer(64)
    off = ctypes.c_int64(0)
    call("gpa_ipc_export", ptr(t), h, ctypes.byref(off))
    return h.raw, int(off.value)


def ipc_open(handle: bytes, offset: int) -> int:
    """This process's device address of a peer's exported byte (see ipc_export)."""
    if len(handle) != 64:
        raise ValueError("ipc_open: a 64-byte handle")
    out = ctypes.c_void_p(0)
    call("gpa_ipc_open", ctypes.create_string_buffer(handle, 64), ctypes.c_int64(offset),
         ctypes.byref(out))
    return int(out.value)


def ipc_close(address: int, offset: int) -> None:
    call("gpa_ipc_close", ctypes.c_void_p(address), ctypes.c_int64(offset))


def merge_exchange_p2p(peer_rows: torch.Tensor, peer_out: torch.Tensor, rank: int, dtype: torch.dtype,
                       rows_per_rank: int, row_elems: int, plan: "MergePlan", dst_lo: int,
                       dst_hi: int, status: Optional[torch.Tensor] = None) -> None:
    """Merge this rank's slots of `plan` from every rank's token rows and store
    them into every rank's merged rows (gpa_merge_exchange_p2p).  peer_rows /
    peer_out: int64 device tensors of the world's buffer addresses as this
    process sees them; the rows buffers hold rows_per_rank rows of row_elems
    `dtype` elements, the outputs plan.n_out rows.  The caller orders the
    ranks' launches (a collective on the stream before and after)."""
    require_cuda(peer_rows, peer_out, what="merge_exchange_p2p")
    if peer_rows.dtype != torch.int64 or peer_out.dtype != torch.int64:
        raise TypeError("merge_exchange_p2p: peer address tables are int64 tensors")
    world = peer_rows.numel()
    dt = _lib.GPA_DTYPE_BF16 if dtype == BF16 else (_lib.GPA_DTYPE_F32 if dtype == F32 else None)
    if dt is None:
        raise TypeError("merge_exchange_p2p: rows must be bf16 or fp32")
    status, own = _status_word(status, peer_rows.device)
    call("gpa_merge_exchange_p2p", ptr(peer_rows), ptr(peer_out), world, rank, dt, int(rows_per_rank),
         int(row_elems), ptr(plan.src_pos), ptr(plan.dst_pos), ptr(plan.unm_src), plan.unm_len,
         ptr(plan.seg_start), ptr(plan.seg_src), plan.num_dst, int(dst_lo), int(dst_hi), ptr(status),
         stream_of(peer_rows))
    if own:
        _check_status(status, "gpa_merge_exchange_p2p")


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, bias: Optional[torch.Tensor],
              sm_scale: float, return_lse: bool = False, out: Optional[torch.Tensor] = None,
              status: Optional[torch.Tensor] = None, combine=None,
              lse_out: Optional[torch.Tensor] = None):
    """softmax(q k^T * scale + bias) v for q [B,H,M,64], k/v [B,H,N,64] bf16;
    bias fp32 broadcastable to [B,H,N] (natural-log domain) or None.

    combine=(oa, lse_a): another partition of the same softmax -- its
    normalised output oa [B,H,M,64] bf16 and log2 row sums lse_a [B,H,M] fp32
    -- merged into the result in the kernel's epilogue (exact two-partition
    combine); `out` may be oa itself (in place).  lse_out: where the log2 row
    sums go ([B,H,M] fp32 view, innermost contiguous; implies return_lse)."""
    require_cuda(q, k, v, bias, what="attention")
    for t in (q, k, v):
        if t.dtype != BF16:
            raise TypeError("attention: q, k, v must be bf16")
    if not _tma_ok(q):
        q = q.contiguous()
    if not _tma_ok(k):
        k = k.contiguous()
    if not _tma_ok(v):
        v = v.contiguous()
    B, H, M, D = q.shape
    N = k.shape[2]
    bsb = bsh = 0
    if bias is not None:
        if bias.dtype != F32:
            bias = bias.float()
        bias = bias.reshape(bias.shape[0], bias.shape[1], N) if bias.dim() == 4 else bias
        if bias.stride(-1) != 1:
            bias = bias.contiguous()
        bias = bias.expand(B, H, N)
        bsb, bsh = bias.stride(0), bias.stride(1)
    if out is None:
        out = torch.empty(B, H, M, D, device=q.device, dtype=BF16)
    if lse_out is not None:
        if lse_out.dtype != F32 or tuple(lse_out.shape) != (B, H, M) or lse_out.stride(-1) != 1:
            raise ValueError("attention: lse_out must be an fp32 [B,H,M] view with row stride 1")
        lse, return_lse = lse_out, True
    else:
        lse = torch.empty(B, H, M, device=q.device, dtype=F32) if return_lse else None
    status, own = _status_word(status, q.device)
    timing = ATTN_TIMING
    if timing is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    if combine is None:
        call("gpa_attention_keybias", ptr(q), ptr(k), ptr(v), ptr(bias), B, H, M, N, D,
             q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
             v.stride(0), v.stride(1), v.stride(2), bsb, bsh, float(sm_scale), ptr(out),
             out.stride(0), out.stride(1), out.stride(2), ptr(lse),
             lse.stride(0) if lse is not None else 0, lse.stride(1) if lse is not None else 0,
             ptr(status), stream_of(q))
    else:
        oa, la = combine
        require_cuda(oa, la, what="attention(combine)")
        if (oa.dtype != BF16 or la.dtype != F32 or tuple(oa.shape) != (B, H, M, D)
                or tuple(la.shape) != (B, H, M) or oa.stride(-1) != 1 or la.stride(-1) != 1):
            raise ValueError("attention: combine needs oa [B,H,M,64] bf16 and lse_a [B,H,M] fp32, "
                             "innermost contiguous")
        call("gpa_attention_keybias_combine", ptr(q), ptr(k), ptr(v), ptr(bias), B, H, M, N, D,
             q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
             v.stride(0), v.stride(1), v.stride(2), bsb, bsh, float(sm_scale),
             ptr(oa), oa.stride(0), oa.stride(1), oa.stride(2), ptr(la), la.stride(0), la.stride(1),
             ptr(out), out.stride(0), out.stride(1), out.stride(2), ptr(lse),
             lse.stride(0) if lse is not None else 0, lse.stride(1) if lse is not None else 0,
             ptr(status), stream_of(q))
    if timing is not None:
        e1.record()
        timing.append((e0, e1, 4.0 * B * H * M * N * D, 2.0 * B * H * (2 * M + 2 * N) * D, N))
    if own:
        _check_status(status, "gpa_attention_keybias")
    return (out, lse) if return_lse else out


def frame_pool(k: torch.Tensor, v: torch.Tensor, num_frames: int, ph: int, pw: int,
               num_special: int, kp: int):
    """Pooled k, v [H, S*npool, 64] bf16 and pool_size [H, S*npool] fp32 from
    k, v [H, S*P, 64] bf16."""
    require_cuda(k, v, what="frame_pool")
    H, N, D = k.shape
    if k.stride(-1) != 1 or k.stride(1) % 8 or k.stride(0) % 8 or not aligned(k):
        k = k.contiguous()
    if v.stride() != k.stride() or not aligned(v):
        v = v.contiguous()
        k = k.contiguous()
    npool = (-(-ph // kp)) * (-(-pw // kp))
    pk = torch.empty(H, num_frames * npool, D, device=k.device, dtype=BF16)
    pv = torch.empty_like(pk)
    size = torch.empty(H, num_frames * npool, device=k.device, dtype=F32)
    call("gpa_frame_pool", ptr(k), ptr(v), H, num_frames, ph, pw, num_special, kp, k.stride(0),
         k.stride(1), ptr(pk), ptr(pv), pk.stride(0), pk.stride(1), ptr(size), stream_of(k))
    return pk, pv, size


def lse_combine(oa, la, ob, lb, out=None):
    """Combine two partitions given as [H, S, P, D] (o*) and [H, S, P] (l*) views."""
    require_cuda(oa, la, ob, lb, what="lse_combine")
    H, S, P, D = oa.shape
    if out is None:
        out = torch.empty(H, S, P, D, device=oa.device, dtype=BF16)
    A = _lib.i64array
    call("gpa_lse_combine", H, S, P, D, ptr(oa), A(oa.stride()[:3]), ptr(la), A(la.stride()),
         ptr(ob), A(ob.stride()[:3]), ptr(lb), A(lb.stride()), ptr(out), A(out.stride()[:3]),
         stream_of(oa))
    return out


def layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16 LayerNorm over the last dim (fp32 statistics) -> bf16."""
    require_cuda(x, weight, bias, what="layernorm")
    C = x.shape[-1]
    x2 = x.reshape(-1, C)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or not aligned(x2):
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty(x.shape, device=x.device, dtype=BF16)
    o2 = out.view(-1, C)
    call("gpa_layernorm_bf16", ptr(x2), x2.stride(0), x2.shape[0], C, ptr(weight), ptr(bias),
         _dt(weight), float(eps), ptr(o2), o2.stride(0), stream_of(x))
    return out


def upsample_bilinear_bf16(x: torch.Tensor, size, add: Optional[torch.Tensor] = None,
                           round_first: bool = False) -> torch.Tensor:
    """bf16(bilinear_align_corners(x) [+ add]) for an fp32 or bf16 [N, C, H, W]
    map in channels-last memory, computed in fp32; add is fp32 [1, C, OH, OW]
    (channel stride 1), added after rounding the resize to bf16 when
    round_first.  Returns a bf16 channels-last [N, C, OH, OW] tensor
    (dpt_head.py custom_interpolate, _apply_pos_embed, with the next autocast
    conv's input cast)."""
    require_cuda(x, what="upsample_bilinear_bf16")
    N, C, H, W = x.shape
    OH, OW = int(size[0]), int(size[1])
    if x.dtype not in (torch.float32, BF16) or x.stride(1) != 1:
        raise ValueError("upsample_bilinear_bf16: fp32/bf16 channels-last input required")
    out = torch.empty((N, OH, OW, C), device=x.device, dtype=BF16).permute(0, 3, 1, 2)
    a_sh = a_sw = 0
    if add is not None:
        if add.dtype != torch.float32 or tuple(add.shape[-3:]) != (C, OH, OW) or add.stride(-3) != 1:
            raise ValueError("upsample_bilinear_bf16: add must be fp32 [1, C, OH, OW] with channel stride 1")
        a_sh, a_sw = add.stride(-2), add.stride(-1)
    call("gpa_upsample_bilinear_bf16", ptr(x), _dt(x), N, C, H, W, x.stride(0), x.stride(2), x.stride(3),
         ptr(add), a_sh, a_sw, int(round_first), OH, OW, ptr(out), out.stride(0), out.stride(2),
         out.stride(3), stream_of(x))
    return out


def bias_act(y: torch.Tensor, bias: torch.Tensor, res: Optional[torch.Tensor] = None,
             relu: bool = False) -> torch.Tensor:
    """In place on a channels-last bf16 map y [N, C, H, W]: bf16(y + bias),
    then ReLU, then bf16(. + res) -- each rounded as torch's bf16 ops round."""
    require_cuda(y, bias, res, what="bias_act")
    cl = torch.channels_last
    if (y.dtype != BF16 or y.dim() != 4 or not y.is_contiguous(memory_format=cl)
            or (res is not None and (res.dtype != BF16 or res.shape != y.shape
                                     or not res.is_contiguous(memory_format=cl)))):
        raise ValueError("bias_act: channels-last contiguous bf16 maps of one shape required")
    N, C, H, W = y.shape
    b = bias.to(BF16).contiguous()
    call("gpa_bias_act_bf16", ptr(y), ptr(b), ptr(res), N * H * W, C, int(bool(relu)), ptr(y),
         stream_of(y))
    return y


def gelu(x: torch.Tensor) -> torch.Tensor:
    """Exact GELU of a bf16 tensor, as torch computes it for bf16 -> new tensor."""
    require_cuda(x, what="gelu")
    if x.dtype != BF16:
        raise ValueError("gelu: bf16 input required")
    xc = x.contiguous()
    out = torch.empty_like(xc)
    call("gpa_gelu_bf16", ptr(xc), xc.numel(), ptr(out), stream_of(xc))
    return out


def residual_scale(x: torch.Tensor, y: torch.Tensor, gamma: torch.Tensor,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x + y * gamma over the last dim, all bf16, rounded as torch's bf16 ops
    (vggt/layers/block.py:88,94 with layer_scale.py:21) -> new bf16 tensor."""
    require_cuda(x, y, gamma, what="residual_scale")
    if x.dtype != BF16 or y.dtype != BF16 or gamma.dtype != BF16 or x.shape != y.shape:
        raise ValueError("residual_scale: bf16 x, y of one shape and a bf16 gamma required")
    C = x.shape[-1]
    if gamma.numel() != C:
        raise ValueError("residual_scale: gamma must have the last dim's size")
    x2, y2 = x.reshape(-1, C), y.reshape(-1, C)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or not aligned(x2):
        x2 = x2.contiguous()
    if y2.stride(-1) != 1 or y2.stride(0) % 8 or not aligned(y2):
        y2 = y2.contiguous()
    g = gamma.contiguous()
    if out is None:
        out = torch.empty(x.shape, device=x.device, dtype=BF16)
    o2 = out.view(-1, C)
    call("gpa_residual_scale_bf16", ptr(x2), x2.stride(0), ptr(y2), y2.stride(0), ptr(g), x2.shape[0], C,
         ptr(o2), o2.stride(0), stream_of(x))
    return out


def qk_norm_rope(qkv: torch.Tensor, q_norm, k_norm, positions: Optional[torch.Tensor],
                 cos_table: Optional[torch.Tensor], sin_table: Optional[torch.Tensor]):
    """In place on qkv [T, 3, H, 64] (bf16, contiguous): q, k <- rope(LN(q)), rope(LN(k)).
    Returns the (q, k, v) views [T, H, 64]."""
    require_cuda(qkv, what="qk_norm_rope")
    T, three, H, D = qkv.shape
    if three != 3 or not qkv.is_contiguous() or qkv.dtype != BF16:
        raise ValueError("qk_norm_rope: qkv must be a contiguous bf16 [T, 3, H, D] tensor")
    qw = getattr(q_norm, "weight", None)
    qb = getattr(q_norm, "bias", None)
    kw = getattr(k_norm, "weight", None)
    kb = getattr(k_norm, "bias", None)
    eps = float(getattr(q_norm, "eps", 1e-5))
    pdt = _dt(qw) if qw is not None else _lib.GPA_DTYPE_F32
    pos = None if positions is None else positions.reshape(T, 2).to(torch.int64).contiguous()
    n_pos = 0 if cos_table is None else cos_table.shape[0]
    call("gpa_qk_norm_rope", ptr(qkv), qkv.stride(0), 0, H * D, T, H, D, ptr(qw), ptr(qb), ptr(kw),
         ptr(kb), pdt, eps, ptr(pos), ptr(cos_table), ptr(sin_table), n_pos, ptr(qkv[:, 0]),
         ptr(qkv[:, 1]), qkv.stride(0), stream_of(qkv))
    return qkv[:, 0], qkv[:, 1], qkv[:, 2]
