"""CPU oracle for GPA-VGGT's accelerated attention path -- TEST INFRASTRUCTURE ONLY.

This module restates, in plain torch-on-CPU (float64 where the reference's
contract is "fp32 accumulate"), each step of the reference path so that the
sm_100a kernels can be checked against it.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it;
the product path (``gpa_vggt_b200``) never does.

Pinning: the restatement is checked against golden vectors produced by the
reference itself (``tests/golden/make_golden.py`` imports noheat61/GPA-VGGT,
runs its merge code on CPU and its two Triton kernels under Triton's CPU
interpreter, and stores the outputs in ``tests/golden/*.pt``);
``tests/test_oracle_golden.py`` holds the oracle to them.

Reference files cited below are paths inside noheat61/GPA-VGGT.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch

LOG2E = 1.4426950408889634


# ----------------------------------------------------------------------------
# a1: dst/src split -- merging/merge.py:87-176
# ----------------------------------------------------------------------------
def dst_mask(num_imgs: int, w: int, h: int, sx: int, sy: int, num_special: int,
             rand_idx: Optional[torch.Tensor], no_rand: bool = False) -> torch.Tensor:
    """Boolean [N]: True for dst tokens (merge.py:87-163).

    Frame 0 is all dst; the num_special leading tokens of every frame are dst;
    in frames >= 1 one token per (sy x sx) window is dst, picked by
    rand_idx[f-1, wy, wx] = dy*sx + dx.  The 2-D window pattern of size
    (h//sy*sy) x (w//sx*sx) is written to that many *contiguous* patch
    positions (merge.py:153-163), so the trailing patch tokens are always src.
    With no_rand the whole grid is written with 0 (src) (merge.py:105-118).
    """
    P = w * h + num_special
    N = P * num_imgs
    mask = torch.zeros(N, dtype=torch.bool)
    if num_imgs == 0:
        return mask
    mask[:P] = True
    hsy, wsx = h // sy, w // sx
    eh, ew = hsy * sy, wsx * sx
    for f in range(1, num_imgs):
        base = f * P
        mask[base:base + num_special] = True
        if no_rand:
            continue
        pat = torch.zeros(eh, ew, dtype=torch.bool)
        ri = rand_idx[f - 1]
        for wy in range(hsy):
            for wx in range(wsx):
                k = int(ri[wy, wx])
                dy, dx = k // sx, k % sx
                pat[wy * sy + dy, wx * sx + dx] = True
        mask[base + num_special: base + num_special + eh * ew] = pat.reshape(-1)
    return mask


def split_positions(mask: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """dst_pos, src_pos in ascending position (merge.py:165-170, canonical order)."""
    pos = torch.arange(mask.numel())
    return pos[mask], pos[~mask]


# ----------------------------------------------------------------------------
# a2: random projection + normalise -- merging/merge.py:180-187
# ----------------------------------------------------------------------------
def bf16_round(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(t.dtype)


def project_metric(x: torch.Tensor, proj: torch.Tensor, autocast_bf16: bool = True) -> torch.Tensor:
    """`metric @ proj` (merge.py:185).  Under bf16 autocast (the GPU runs):
    bf16(bf16(x) @ bf16(proj)) with exact accumulation; without autocast (a
    CPU fp32 run): the fp32 product."""
    if not autocast_bf16:
        return x.float() @ proj.float()  # the fp32 CPU product the reference computes
    y = bf16_round(x.double()) @ bf16_round(proj.double())
    return bf16_round(y.float())


def normalize_rows(m: torch.Tensor) -> torch.Tensor:
    """metric / metric.norm(dim=-1) (merge.py:186), then the bf16 cast of
    fused_similarity.py:90-101.  The norm and the quotient are fp32 for a bf16
    metric too: in the reference's GPU run under autocast `metric @ proj` comes
    out bf16 but `norm` is on autocast's fp32 list, so the division promotes to
    fp32 and the matcher rounds its fp32 inputs to bf16."""
    m = m.float()
    return bf16_round(m / m.norm(dim=-1, keepdim=True))


# ----------------------------------------------------------------------------
# a3: similarity + first argmax -- merging/fused_similarity.py:33-112
# ----------------------------------------------------------------------------
def sim_argmax(a: torch.Tensor, b: torch.Tensor, chunk: int = 4096):
    """Exact (float64) scores of bf16 inputs; argmax with the first index on ties
    (tl.argmax within a tile, strict '>' across tiles: fused_similarity.py:70-75).

    Returns node_max (float64), node_idx (int64) and the gap between the best and
    the second-best score of each row (used to identify near-ties).
    """
    a = bf16_round(a.float()).double()
    b = bf16_round(b.float()).double()
    M = a.shape[0]
    node_max = torch.empty(M, dtype=torch.float64)
    node_idx = torch.empty(M, dtype=torch.int64)
    gap = torch.empty(M, dtype=torch.float64)
    for i in range(0, M, chunk):
        s = a[i:i + chunk] @ b.T
        mx, ix = s.max(dim=1)  # torch.max returns the first index of the max
        node_max[i:i + chunk] = mx
        node_idx[i:i + chunk] = ix
        if s.shape[1] > 1:
            top2 = s.topk(2, dim=1).values
            gap[i:i + chunk] = top2[:, 0] - top2[:, 1]
        else:
            gap[i:i + chunk] = math.inf
    return node_max, node_idx, gap


def sim_argmax_bf16_scores(a: torch.Tensor, b: torch.Tensor):
    """The reference's CPU matcher fast_similarity_chunks (merge.py:13-36):
    scores rounded to bf16 before the max."""
    s = bf16_round((bf16_round(a.float()).double() @ bf16_round(b.float()).double().T).float())
    mx, ix = s.max(dim=1)
    return mx, ix


# ----------------------------------------------------------------------------
# a4/a5: edge ranking and counts -- merging/merge.py:189-217
# ----------------------------------------------------------------------------
@dataclass
class Plan:
    merged: torch.Tensor      # bool [num_src]
    unm_src: torch.Tensor     # int64 unmerged src ordinals, ascending
    dst_of_src: torch.Tensor  # int64 [num_src]: dst ordinal (node_idx)
    counts: torch.Tensor      # float [unm_len + num_dst]
    num_dst: int

    @property
    def unm_len(self) -> int:
        return int(self.unm_src.numel())


def merge_plan(node_max: torch.Tensor, node_idx: torch.Tensor, r: int, num_dst: int) -> Plan:
    """Top-r src by node_max (descending; ties to the lower ordinal, i.e. a
    stable sort) are merged into node_idx; counts = ones + scatter_add of the
    merged src (merge.py:199-217)."""
    ns = node_max.numel()
    r = min(ns, r)
    order = sorted(range(ns), key=lambda i: (-float(node_max[i]), i))
    merged = torch.zeros(ns, dtype=torch.bool)
    merged[order[:r]] = True
    unm = torch.nonzero(~merged).reshape(-1)
    counts = torch.ones(unm.numel() + num_dst, dtype=torch.float64)
    for i in torch.nonzero(merged).reshape(-1).tolist():
        counts[unm.numel() + int(node_idx[i])] += 1
    return Plan(merged, unm, node_idx.long(), counts, num_dst)


# ----------------------------------------------------------------------------
# a6: merge.heads scatter-mean -- merging/merge.py:234-250
# ----------------------------------------------------------------------------
def merge_heads(t: torch.Tensor, plan: Plan, dst_pos, src_pos, mode: str = "mean") -> torch.Tensor:
    """t [H, N, D] -> [H, unm_len + num_dst, D] in float64:
    unmerged src rows, then (dst + sum of its merged src) / (1 + count) for
    mode 'mean' (scatter_reduce mean with include_self, merge.py:246-249)."""
    t = t.double()
    H, N, D = t.shape
    out = torch.empty(H, plan.unm_len + plan.num_dst, D, dtype=torch.float64)
    out[:, :plan.unm_len] = t[:, src_pos[plan.unm_src]]
    mid = t[:, dst_pos].clone()
    cnt = torch.ones(plan.num_dst, dtype=torch.float64)
    idx = torch.nonzero(plan.merged).reshape(-1)
    for i in idx.tolist():
        d = int(plan.dst_of_src[i])
        mid[:, d] += t[:, int(src_pos[i])]
        cnt[d] += 1
    if mode == "mean":
        mid = mid / cnt[None, :, None]
    out[:, plan.unm_len:] = mid
    return out


# ----------------------------------------------------------------------------
# a9: attention with a per-key bias -- merging/fused_attention.py:130-180
# ----------------------------------------------------------------------------
def attention_keybias(q, k, v, bias, scale, return_lse: bool = False):
    """softmax(q k^T * scale + bias) v in float64 for q [..., M, D], k/v
    [..., N, D], bias broadcastable to [..., 1, N] or None.  lse is the log2 of
    the softmax denominator in the exp2 domain (fused_attention.py:123-127)."""
    q, k, v = q.double(), k.double(), v.double()
    s = (q @ k.transpose(-1, -2)) * scale
    if bias is not None:
        s = s + bias.double()
    o = torch.softmax(s, dim=-1) @ v
    if not return_lse:
        return o
    lse = torch.logsumexp(s, dim=-1) * LOG2E
    return o, lse


# ----------------------------------------------------------------------------
# a11: content-adaptive pooling -- vggt/layers/attention.py:113-140
# ----------------------------------------------------------------------------
def frame_pool(k5: torch.Tensor, v5: torch.Tensor, ph: int, pw: int, pts: int, kp: int):
    """k5, v5 [H, S, P, D] -> pooled k, v [H, S*npool, D] (float32 means of the
    bf16 inputs, attention.py:135-140) and pool_size [H, S*npool]."""
    H, S, P, D = k5.shape
    nh, nw = -(-ph // kp), -(-pw // kp)
    npool = nh * nw
    x = k5[:, :, pts:, :].reshape(H, S, ph, pw, D).float()
    xf = x.reshape(H, S, ph * pw, D)
    dst = x[:, :, ::kp, ::kp, :].reshape(H, S, npool, D)
    a = xf / xf.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    b = dst / dst.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    assign = torch.einsum("hsid,hsgd->hsig", a.double(), b.double()).argmax(-1)
    size = torch.zeros(H, S, npool, dtype=torch.float32)
    size.scatter_add_(2, assign, torch.ones_like(assign, dtype=torch.float32))
    outs = []
    for t5 in (k5, v5):
        tf = t5[:, :, pts:, :].reshape(H, S, ph * pw, D).float()
        acc = torch.zeros(H, S, npool, D, dtype=torch.float32)
        acc.scatter_add_(2, assign[..., None].expand(H, S, ph * pw, D), tf)
        acc /= size.clamp_min(1.0).unsqueeze(-1)
        outs.append(acc.reshape(H, S * npool, D))
    return outs[0], outs[1], size.reshape(H, S * npool), assign


# ----------------------------------------------------------------------------
# a10/a12: frame attention with the shared cross-frame set -- attention.py:73-206
# ----------------------------------------------------------------------------
def frame_special_attention(q, k, v, S, ph, pw, pts, kp, scale):
    """q, k, v [H, N, D] -> [H, N, D] (float64).  Queries of frame s attend to
    the own frame's patch keys, every frame's special keys and every frame's
    pooled summaries (bias +log size), in one softmax: the replicated-shared
    formula of attention.py:178-206, which is the exact combine of :152-176."""
    H, N, D = q.shape
    P = ph * pw + pts
    k5, v5 = k.reshape(H, S, P, D), v.reshape(H, S, P, D)
    pk, pv, size, _ = frame_pool(k5, v5, ph, pw, pts, kp)
    sp_k = k5[:, :, :pts].reshape(H, S * pts, D)
    sp_v = v5[:, :, :pts].reshape(H, S * pts, D)
    out = torch.empty(H, N, D, dtype=torch.float64)
    shared_bias = torch.cat([torch.zeros(H, S * pts, dtype=torch.float64), size.double().log()], 1)
    for s in range(S):
        kk = torch.cat([k5[:, s, pts:].double(), sp_k.double(), pk.double()], 1)
        vv = torch.cat([v5[:, s, pts:].double(), sp_v.double(), pv.double()], 1)
        bias = torch.cat([torch.zeros(H, ph * pw, dtype=torch.float64), shared_bias], 1)
        out[:, s * P:(s + 1) * P] = attention_keybias(q[:, s * P:(s + 1) * P], kk, vv,
                                                      bias[:, None, :], scale)
    return out


def lse_combine(oa, la, ob, lb):
    """Exact two-partition combine (attention.py:164-176), float64."""
    mx = torch.maximum(la, lb)
    wa, wb = torch.exp2(la - mx), torch.exp2(lb - mx)
    den = wa + wb
    return (oa.double() * (wa / den)[..., None] + ob.double() * (wb / den)[..., None])


# ----------------------------------------------------------------------------
# merged global block core -- vggt/layers/attention.py:233-268
# ----------------------------------------------------------------------------
def merged_attention(x, q, k, v, proj, rand_idx, ratio, w, h, num_special, scale,
                     sx: int = 2, sy: int = 2, bf16_bias: bool = True):
    """The merged-block attention for one sequence: x [N, C] (matching metric),
    q, k, v [H, N, D] -> [H, N, D] float64, plus the intermediate plan."""
    N = x.shape[0]
    P = w * h + num_special
    S = N // P
    mask = dst_mask(S, w, h, sx, sy, num_special, rand_idx)
    dst_pos, src_pos = split_positions(mask)
    metric = project_metric(x, proj)
    mn = normalize_rows(metric)
    a, b = mn[src_pos], mn[dst_pos]
    node_max, node_idx, gap = sim_argmax(a, b)
    r = int(N * ratio)
    plan = merge_plan(node_max, node_idx, r, dst_pos.numel())
    km = merge_heads(k, plan, dst_pos, src_pos)
    vm = merge_heads(v, plan, dst_pos, src_pos)
    bias = plan.counts.log()
    if bf16_bias:
        bias = bf16_round(bias.float()).double()
    o = attention_keybias(q, km, vm, bias[None, None, :], scale)
    return o, dict(dst_pos=dst_pos, src_pos=src_pos, node_max=node_max, node_idx=node_idx,
                   gap=gap, plan=plan, km=km, vm=vm)
