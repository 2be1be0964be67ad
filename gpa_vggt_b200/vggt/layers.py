"""Transformer layers of VGGT around the GPA attention path.

Module and parameter names follow the reference (vggt/layers/*.py) so that one
state_dict loads into either model.  Every head_dim-64 attention runs on the
sm_100a kernels: the GPA global paths (merged, frame + shared set), the plain
global/frame attention and the DINO blocks.  Everything else (linears, norms,
activations) is ordinary torch, run under bf16 autocast as the reference's
evaluation does (eval/bench_e2e.py:90-95).
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from .. import kernels
from ..nvtx import nvtx
from ..merging.merge import (build_plan, draw_dst_choice, fused_metric_ok, projection_basis,
                             projection_basis_t)

BF16 = torch.bfloat16


# ---------------------------------------------------------------------------
# small layers (vggt/layers/mlp.py, layer_scale.py, patch_embed.py)
# ---------------------------------------------------------------------------
class LayerNorm(nn.LayerNorm):
    """nn.LayerNorm whose CUDA bf16 path is the fused kernel (fp32 statistics,
    bf16 result: what a bf16-autocast Linear receives from the reference's fp32
    LayerNorm).  Other inputs (the CPU, fp32, no affine) use torch."""

    def forward(self, x):
        if (x.is_cuda and x.dtype == BF16 and self.weight is not None and self.bias is not None
                and x.shape[-1] % 256 == 0 and x.shape[-1] <= 4096):
            return kernels.layernorm(x, self.weight, self.bias, self.eps)
        return super().forward(x)


class Mlp(nn.Module):
    def __init__(self, in_features, hidden_features=None, out_features=None, act_layer=nn.GELU,
                 drop=0.0, bias=True):
        super().__init__()
        out_features = out_features or in_features
        hidden_features = hidden_features or in_features
        self.fc1 = nn.Linear(in_features, hidden_features, bias=bias)
        self.act = act_layer()
        self.fc2 = nn.Linear(hidden_features, out_features, bias=bias)

    def forward(self, x):
        h = self.fc1(x)
        if (isinstance(self.act, nn.GELU) and self.act.approximate == "none" and h.is_cuda
                and h.dtype == BF16 and h.numel() % 8 == 0):
            h = kernels.gelu(h)   # same fp32 erf expression, one vectorised pass
        else:
            h = self.act(h)
        return self.fc2(h)


class LayerScale(nn.Module):
    def __init__(self, dim, init_values=1e-5):
        super().__init__()
        self.gamma = nn.Parameter(init_values * torch.ones(dim))

    def forward(self, x):
        return x * self.gamma


class PatchEmbed(nn.Module):
    """Conv patchifier: [B, 3, H, W] -> [B, H/p * W/p, C]."""

    def __init__(self, img_size=224, patch_size=16, in_chans=3, embed_dim=768):
        super().__init__()
        self.patch_size = (patch_size, patch_size)
        self.num_patches = (img_size // patch_size) ** 2
        self.proj = nn.Conv2d(in_chans, embed_dim, kernel_size=patch_size, stride=patch_size)
        self.norm = nn.Identity()

    def forward(self, x):
        return self.proj(x).flatten(2).transpose(1, 2)


# ---------------------------------------------------------------------------
# 2D rotary embedding (vggt/layers/rope.py), token-major layout
# ---------------------------------------------------------------------------
class PositionGetter:
    """(y, x) patch coordinates of an h x w grid, [batch, h*w, 2] (rope.py:24-65)."""

    def __init__(self):
        self.cache = {}

    def __call__(self, batch_size, height, width, device):
        key = (height, width, str(device))
        if key not in self.cache:
            ys = torch.arange(height, device=device)
            xs = torch.arange(width, device=device)
            self.cache[key] = torch.cartesian_prod(ys, xs)
        return self.cache[key].view(1, height * width, 2).expand(batch_size, -1, -1).clone()


class RotaryPositionEmbedding2D(nn.Module):
    """First half of each head's features rotates with y, second half with x;
    within a half, the rotate-half convention with base frequency 100
    (rope.py:68-209).  Operates on [B, N, H, D] tokens with [B, N, 2] positions."""

    def __init__(self, frequency: float = 100.0, scaling_factor: float = 1.0):
        super().__init__()
        self.base_frequency = frequency
        self.scaling_factor = scaling_factor
        self.cache = {}

    def tables(self, dim, device, n_pos=1024):
        """fp32 cos/sin tables [n_pos, dim] as the reference computes them for
        fp32 tokens (rope.py:92-123); rows do not depend on n_pos."""
        return self._tables(dim, n_pos, device, torch.float32)

    def _tables(self, dim, n_pos, device, dtype):
        key = (dim, n_pos, str(device), dtype)
        if key not in self.cache:
            inv = 1.0 / (self.base_frequency ** (torch.arange(0, dim, 2, device=device) / dim))
            ang = torch.outer(torch.arange(n_pos, device=device, dtype=inv.dtype), inv).to(dtype)
            ang = torch.cat((ang, ang), dim=-1)
            self.cache[key] = (ang.cos().to(dtype), ang.sin().to(dtype))
        return self.cache[key]

    @staticmethod
    def _rot(t):
        h = t.shape[-1] // 2
        return torch.cat((-t[..., h:], t[..., :h]), dim=-1)

    def forward(self, tokens: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        half = tokens.shape[-1] // 2
        n_pos = int(positions.max()) + 1
        cos, sin = self._tables(half, n_pos, tokens.device, tokens.dtype)
        pos = positions.long()
        out = []
        for i, t in enumerate(tokens.chunk(2, dim=-1)):
            c = F.embedding(pos[..., i], cos)[:, :, None, :]   # [B, N, 1, half]
            s = F.embedding(pos[..., i], sin)[:, :, None, :]
            out.append(t * c + self._rot(t) * s)
        return torch.cat(out, dim=-1)


# ---------------------------------------------------------------------------
# attention (vggt/layers/attention.py)
# ---------------------------------------------------------------------------
class Attention(nn.Module):
    """VGGT attention with the two GPA global paths on the sm_100a kernels.

    Attributes set by the aggregator, as in the reference (attention.py:53-63):
    ``frame_special``, ``num_special``, ``broadcast_pool``, ``merge_grid``,
    ``merge_metric_dim``, ``merge_ratio``, ``patch_width``, ``patch_height``.
    Tests may set ``rng_override = (rand_idx, proj)`` to inject the two random
    draws of the merge (a CPU run draws different numbers than a CUDA run).
    """

    def __init__(self, dim, num_heads=8, qkv_bias=True, proj_bias=True, attn_drop=0.0,
                 proj_drop=0.0, norm_layer=LayerNorm, qk_norm=False, fused_attn=True, rope=None,
                 patch_width=37, patch_height=28, merge_ratio=0.9):
        super().__init__()
        assert dim % num_heads == 0
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.scale = self.head_dim ** -0.5
        self.patch_width = patch_width
        self.patch_height = patch_height
        self.merge_ratio = merge_ratio
        self.frame_special = False
        self.num_special = 5
        self.broadcast_pool = 0
        self.merge_grid = 2
        self.merge_metric_dim = 0
        self.rng_override = None
        self.shard = None            # FrameShard of a global block run across GPUs
        self.qkv = nn.Linear(dim, dim * 3, bias=qkv_bias)
        self.q_norm = norm_layer(self.head_dim) if qk_norm else nn.Identity()
        self.k_norm = norm_layer(self.head_dim) if qk_norm else nn.Identity()
        self.proj = nn.Linear(dim, dim, bias=proj_bias)
        self.rope = rope

    # -- helpers ------------------------------------------------------------
    def _qkv(self, x, pos):
        B, N, C = x.shape
        H, D = self.num_heads, self.head_dim
        qkv = self.qkv(x)
        if (qkv.is_cuda and qkv.dtype == BF16 and D == 64 and isinstance(self.q_norm, nn.LayerNorm)
                and (self.rope is None or pos is not None)):
            # qk-LayerNorm + RoPE + bf16 in one pass, in place on the qkv buffer
            cos = sin = None
            if self.rope is not None:
                cos, sin = self.rope.tables(D // 2, qkv.device)
            q, k, v = kernels.qk_norm_rope(qkv.view(B * N, 3, H, D), self.q_norm, self.k_norm,
                                           None if self.rope is None else pos, cos, sin)
            return q.view(B, N, H, D), k.view(B, N, H, D), v.view(B, N, H, D)
        qkv = qkv.reshape(B, N, 3, H, D)
        q, k, v = qkv.unbind(2)                      # [B, N, H, D] views
        q, k = self.q_norm(q), self.k_norm(k)
        if self.rope is not None:
            q, k = self.rope(q, pos), self.rope(k, pos)
        return q, k, v

    @staticmethod
    def _heads(t):
        """[B, N, H, D] -> [B, H, N, D] view (no copy)."""
        return t.permute(0, 2, 1, 3)

    def forward(self, x: torch.Tensor, pos=None, global_merging=None) -> torch.Tensor:
        B, N, C = x.shape
        q, k, v = self._qkv(x, pos)
        if self.frame_special:
            out = frame_special_attention(q.to(BF16), k.to(BF16), v.to(BF16), self)
        elif global_merging is not None:
            out = merged_attention(x, q, k, v, self)
        else:
            out = torch.empty(B, N, self.num_heads, self.head_dim, device=x.device, dtype=BF16)
            k, v = k.to(BF16), v.to(BF16)
            if self.shard is not None and self.shard.active:   # keys of every frame
                k = self.shard.gather(k[0].contiguous())[None]
                v = self.shard.gather(v[0].contiguous())[None]
            kernels.attention(self._heads(q.to(BF16)), self._heads(k), self._heads(v), None,
                              self.scale, out=self._heads(out))
        return self.proj(out.reshape(B, N, C))


def _merge_draws(attn: Attention, num_imgs: int, C: int, device, dtype):
    """The two random draws of a merge: dst pick per window and projection basis
    (injected by tests, else drawn as the reference draws them)."""
    if attn.rng_override is not None:
        return attn.rng_override
    gen = torch.Generator(device=device)
    gen.manual_seed(33)
    rand_idx = draw_dst_choice(num_imgs, attn.patch_width, attn.patch_height, attn.merge_grid,
                               attn.merge_grid, device, gen)
    proj = projection_basis(C, attn.merge_metric_dim, device, dtype) if attn.merge_metric_dim else None
    return rand_idx, proj


# GPA_OVERLAP_GATHER=1: sharded merged blocks attend to the rank's own merged
# slots while the other ranks' merged rows are all-gathered, then combine the
# two softmax partitions.  Off by default: at S=200 on 4 GPUs it saved 0.8% of
# the forward, while the bf16 rounding of the first partition's output moved
# the pose by 1.7e-2 (rel-L2) from the one-GPU forward, which the default path
# (all merged rows first, one attention launch) reproduces exactly.
OVERLAP_GATHER = os.environ.get("GPA_OVERLAP_GATHER", "0") == "1"
# Sharded merged blocks on CUDA with NCCL exchange their merged K/V through
# peer memory in one kernel (merge_exchange_p2p); GPA_P2P_EXCHANGE=0 keeps the
# NCCL all-to-all + merge + all-gather path (merge_exchange).
P2P_EXCHANGE = os.environ.get("GPA_P2P_EXCHANGE", "1") == "1"


def merged_attention_sharded(x, q, k, v, attn: Attention) -> torch.Tensor:
    """Merged block with the queries sharded by frame (see shard.py): every rank
    builds the same global plan from all-gathered match results, merges the
    output slots of its own frames (merge_exchange) and attends with its own
    queries against all merged keys."""
    from .shard import merge_exchange, merge_exchange_p2p, merge_local
    sh = attn.shard
    B, Nl, C = x.shape
    H, D = attn.num_heads, attn.head_dim
    P = attn.patch_width * attn.patch_height + attn.num_special
    S, N = sh.frames, sh.frames * P
    if Nl != sh.local * P:
        raise ValueError("merged_attention_sharded: local tokens do not match the frame shard")
    dev = x.device
    with nvtx("sharded_metric"):
        a, b, dst_pos, src_pos, ranges = _sharded_metric(x, attn, S, C, P, dev)
    with nvtx("sharded_gather_dst"):
        b_full = sh.gather_varlen(b, [rd[1] - rd[0] for rd, _ in ranges])
    (d0, d1), (s0, s1) = ranges[sh.rank]
    with nvtx("sharded_sim"):
        if s1 > s0:
            nm, ni = kernels.sim_argmax(a[None], b_full[None])
            nm, ni = nm[0], ni[0]
        else:
            nm = torch.empty(0, device=dev)
            ni = torch.empty(0, device=dev, dtype=torch.int32)
    with nvtx("sharded_gather_match"):
        src_counts = [rs[1] - rs[0] for _, rs in ranges]
        nm_full = sh.gather_varlen(nm, src_counts)
        ni_full = sh.gather_varlen(ni, src_counts)
    with nvtx("sharded_plan"):
        plan = kernels.merge_plan(nm_full, ni_full, int(N * attn.merge_ratio), dst_pos, src_pos)
    bias = plan.counts.log().to(BF16).float()
    out = torch.empty(1, Nl, H, D, device=dev, dtype=BF16)
    qh, oh = q.to(BF16).permute(0, 2, 1, 3), out.permute(0, 2, 1, 3)

    def attend(merged, key_bias, **kw):
        m = merged.view(merged.shape[0], 2, H, D)
        with nvtx("sharded_attend"):
            kernels.attention(qh, m[:, 0].to(BF16).permute(1, 0, 2)[None],
                              m[:, 1].to(BF16).permute(1, 0, 2)[None], key_bias[None, None],
                              attn.scale, out=oh, **kw)

    if P2P_EXCHANGE and x.is_cuda and dist.get_backend(sh.group) == "nccl":
        with nvtx("sharded_exchange"):
            merged = merge_exchange_p2p(sh, k[0], v[0], plan, P, (d0, d1), kernels)
        attend(merged, bias)
        return out
    # K and V travel and merge as one [tokens, 2*H*D] row buffer (V widened to
    # K's dtype when they differ: exact, and the merged V is rounded back below)
    kv = torch.stack((k[0], v[0].to(k.dtype)), 1).reshape(Nl, 2 * H * D)
    if not OVERLAP_GATHER:
        with nvtx("sharded_exchange"):
            merged = merge_exchange(sh, kv, plan, P, kernels)
        attend(merged, bias)
        return out
    # The rank's own merged slots are attended while the other ranks' merged
    # rows arrive on the key/value communicator; the second launch attends the
    # rest and combines both softmax partitions by log-sum-exp in its epilogue
    # (attention is invariant to the order and partition of its keys).
    with nvtx("sharded_exchange"):
        own, (unm_cnt, dst_cnt, u0, e0) = merge_local(sh, kv, plan, P, kernels)
        nu, nd, U = unm_cnt[sh.rank], dst_cnt[sh.rank], plan.unm_len
        full, work = sh.gather_varlen2_async(own[:nu], own[nu:], unm_cnt, dst_cnt)
    lse = torch.empty(1, H, Nl, device=dev, dtype=torch.float32)
    attend(own, torch.cat([bias[u0:u0 + nu], bias[U + e0:U + e0 + nd]]), lse_out=lse)
    work.wait()
    ma = max(unm_cnt)
    rows, key_bias = [], []
    uu = ee = 0
    for r in range(sh.world):
        if r != sh.rank:
            rows += [full[r, :unm_cnt[r]], full[r, ma:ma + dst_cnt[r]]]
            key_bias += [bias[uu:uu + unm_cnt[r]], bias[U + ee:U + ee + dst_cnt[r]]]
        uu += unm_cnt[r]
        ee += dst_cnt[r]
    attend(torch.cat(rows), torch.cat(key_bias), combine=(oh, lse))
    return out


def _sharded_metric(x, attn: Attention, S: int, C: int, P: int, dev):
    """This rank's src and dst metric rows of a sharded merged block, the
    roles' token positions and the per-rank ordinal ranges."""
    sh = attn.shard
    pw, ph, ns, g = attn.patch_width, attn.patch_height, attn.num_special, attn.merge_grid
    Nl = x.shape[1]
    rand_idx, proj = _merge_draws(attn, S, C, dev, x.dtype)
    dst_pos, src_pos, slot = kernels.merge_roles(rand_idx, S, pw, ph, g, g, ns, False, dev)
    dpf = ns + (ph // g) * (pw // g)
    ranges = sh.role_ranges(P, dpf)
    (d0, d1), (s0, s1) = ranges[sh.rank]
    base = sh.f0 * P
    metric = x[0]
    if fused_metric_ok(metric, attn.merge_metric_dim):
        # this rank's rows, with the role map renumbered to its own ordinals
        sl = slot[base:base + Nl]
        sl = torch.where(sl >= 0, sl - d0, sl + s0).to(torch.int32)
        proj_t = (projection_basis_t(C, attn.merge_metric_dim, dev) if attn.rng_override is None
                  else proj.to(BF16).t().contiguous())
        a, b = kernels.proj_norm_split(metric, proj_t, sl, s1 - s0, d1 - d0)
    else:
        if attn.merge_metric_dim and attn.merge_metric_dim < C:
            metric = metric @ proj.to(metric.dtype)
        a, b = kernels.metric_split(metric, src_pos[s0:s1] - base, dst_pos[d0:d1] - base)
    return a, b, dst_pos, src_pos, ranges


def merged_attention(x, q, k, v, attn: Attention) -> torch.Tensor:
    """Query-preserving K/V merging (attention.py:233-268): merge K/V into the
    dst tokens matched on the 128-d projected x, then attend with +log(count).
    With B > 1 the dst pattern is drawn once and each batch element is matched,
    merged and attended on its own (merge.py:121-126, attention.py:251-253)."""
    B, N, C = x.shape
    H, D = attn.num_heads, attn.head_dim
    if attn.shard is not None and attn.shard.active:
        if B != 1:
            raise NotImplementedError("merged_attention: frame sharding runs batch size 1")
        return merged_attention_sharded(x, q, k, v, attn)
    r = int(N * attn.merge_ratio)
    if attn.rng_override is not None:
        rand_idx, proj = attn.rng_override
    else:
        gen = torch.Generator(device=x.device)
        gen.manual_seed(33)
        num_imgs = N // (attn.patch_width * attn.patch_height + attn.num_special)
        rand_idx = draw_dst_choice(num_imgs, attn.patch_width, attn.patch_height, attn.merge_grid,
                                   attn.merge_grid, x.device, gen)
        proj = None
    out = torch.empty(B, N, H, D, device=x.device, dtype=BF16)
    for bi in range(B):
        plan = build_plan(x[bi], attn.patch_width, attn.patch_height, attn.merge_grid,
                          attn.merge_grid, r, False, None, attn.merge_metric_dim, attn.num_special,
                          rand_idx=rand_idx, proj=proj)
        # K keeps its dtype through the merge (fp32 after qk-LayerNorm under
        # autocast), then both are bf16 for the attention, as attention_keybias
        # casts them.
        km = kernels.merge_kv(k[bi].transpose(0, 1), plan)          # [H, N_m, D]
        vm = kernels.merge_kv(v[bi].transpose(0, 1), plan)
        bias = plan.counts.log().to(BF16).float()                   # rounded like the reference
        kernels.attention(q[bi:bi + 1].to(BF16).permute(0, 2, 1, 3), km.to(BF16)[None],
                          vm.to(BF16)[None], bias[None, None], attn.scale,
                          out=out[bi:bi + 1].permute(0, 2, 1, 3))
    return out


def frame_special_attention(q, k, v, attn: Attention) -> torch.Tensor:
    """Frame attention plus the shared cross-frame K/V set (attention.py:73-206):
    own-frame keys (with log2 row sums), then every frame's special tokens and
    pooled patch summaries (bias +log size), combined exactly by log-sum-exp.
    q, k, v: [1, N, H, D] bf16 -> [1, N, H, D] bf16."""
    B, N, H, D = q.shape
    if B != 1:   # batch elements are independent sequences of frames
        if attn.shard is not None and attn.shard.active:
            raise NotImplementedError("frame_special_attention: frame sharding runs batch size 1")
        return torch.cat([frame_special_attention(q[bi:bi + 1], k[bi:bi + 1], v[bi:bi + 1], attn)
                          for bi in range(B)], 0)
    pts, pw, ph, kp = attn.num_special, attn.patch_width, attn.patch_height, attn.broadcast_pool
    P = pw * ph + pts
    S = N // P                      # this rank's frames
    sh = attn.shard if (attn.shard is not None and attn.shard.active) else None
    if S * P != N:
        raise ValueError(f"frame_special: token count {N} is not S*(patch_w*patch_h+{pts})")
    if kp <= 0:
        raise NotImplementedError("frame_special_attention: broadcast_pool > 0 only")
    q5, k5, v5 = (t.view(S, P, H, D) for t in (q[0], k[0], v[0]))
    # (a) own-frame patch keys, batch = frames: rows written token-major
    #     [N, H, D] (the layout proj reads), log2 row sums head-major [H, N]
    out = torch.empty(S, P, H, D, device=q.device, dtype=BF16)
    lse_a = torch.empty(H, N, device=q.device, dtype=torch.float32)
    kernels.attention(q5.permute(0, 2, 1, 3), k5[:, pts:].permute(0, 2, 1, 3),
                      v5[:, pts:].permute(0, 2, 1, 3), None, attn.scale,
                      out=out.permute(0, 2, 1, 3), lse_out=lse_a.view(H, S, P).permute(1, 0, 2))
    # (b) shared set: specials of every frame, then the pooled summaries
    kh, vh = k[0].transpose(0, 1), v[0].transpose(0, 1)       # [H, N, D] views
    pk, pv, size = kernels.frame_pool(kh, vh, S, ph, pw, pts, kp)
    spk, spv = k5[:, :pts], v5[:, :pts]                       # [S, pts, H, D]
    St = S
    if sh is not None:                 # the shared set of every frame
        npool = pk.shape[1] // S
        St = sh.frames
        spk, spv = sh.gather(spk.contiguous()), sh.gather(spv.contiguous())
        pk = sh.gather(pk.view(H, S, npool, D).transpose(0, 1).contiguous()).transpose(0, 1)
        pv = sh.gather(pv.view(H, S, npool, D).transpose(0, 1).contiguous()).transpose(0, 1)
        pk, pv = pk.reshape(H, St * npool, D), pv.reshape(H, St * npool, D)
        size = sh.gather(size.view(H, S, npool).transpose(0, 1).contiguous()).transpose(0, 1)
        size = size.reshape(H, St * npool)
    sk = torch.cat([spk.permute(2, 0, 1, 3).reshape(H, St * pts, D), pk], 1)
    sv = torch.cat([spv.permute(2, 0, 1, 3).reshape(H, St * pts, D), pv], 1)
    bias = torch.cat([torch.zeros(H, St * pts, device=q.device), size.log()], 1)
    bias = bias.to(BF16).float()                               # the reference casts it to bf16
    # (c) every query against the shared set, combined exactly with (a) by
    #     log-sum-exp in the kernel's epilogue, in place in `out`
    o_tok = out.view(N, H, D).permute(1, 0, 2)[None]           # [1, H, N, D] view
    kernels.attention(q[0].transpose(0, 1)[None], sk[None], sv[None], bias[None], attn.scale,
                      out=o_tok, combine=(o_tok, lse_a[None]))
    return out.view(1, N, H, D)


class SdpaAttention(Attention):
    """Plain attention through torch SDPA, for the camera head's trunk
    (head_dim 128, S tokens; outside the GPA path)."""

    def forward(self, x, pos=None, global_merging=None):
        B, N, C = x.shape
        q, k, v = self._qkv(x, pos)
        o = F.scaled_dot_product_attention(self._heads(q), self._heads(k), self._heads(v))
        return self.proj(o.transpose(1, 2).reshape(B, N, C))


# ---------------------------------------------------------------------------
# block (vggt/layers/block.py:23-96)
# ---------------------------------------------------------------------------
class Block(nn.Module):
    def __init__(self, dim, num_heads, mlp_ratio=4.0, qkv_bias=True, proj_bias=True, ffn_bias=True,
                 drop=0.0, attn_drop=0.0, init_values=None, drop_path=0.0, act_layer=nn.GELU,
                 norm_layer=LayerNorm, attn_class=Attention, ffn_layer=Mlp, qk_norm=False,
                 fused_attn=True, rope=None, merge_ratio=0.9):
        super().__init__()
        self.norm1 = norm_layer(dim)
        self.attn = attn_class(dim, num_heads=num_heads, qkv_bias=qkv_bias, proj_bias=proj_bias,
                               qk_norm=qk_norm, rope=rope, merge_ratio=merge_ratio)
        self.ls1 = LayerScale(dim, init_values=init_values) if init_values else nn.Identity()
        self.norm2 = norm_layer(dim)
        self.mlp = ffn_layer(in_features=dim, hidden_features=int(dim * mlp_ratio),
                             act_layer=act_layer, bias=ffn_bias)
        self.ls2 = LayerScale(dim, init_values=init_values) if init_values else nn.Identity()

    def forward(self, x, pos=None, global_merging=None):
        x = _residual(x, self.ls1, self.attn(self.norm1(x), pos=pos, global_merging=global_merging))
        return _residual(x, self.ls2, self.mlp(self.norm2(x)))


def _residual(x, ls, y):
    """x + ls(y) (vggt/layers/block.py:88,94).  With a LayerScale on CUDA bf16
    tensors this is one fused pass (same roundings as torch's bf16 ops)."""
    if (isinstance(ls, LayerScale) and x.is_cuda and x.dtype == BF16 and y.dtype == BF16
            and ls.gamma.dtype == BF16 and x.shape == y.shape and x.shape[-1] % 8 == 0):
        return kernels.residual_scale(x, y, ls.gamma)
    return x + ls(y)
