"""Alternating frame/global attention aggregator with the GPA-VGGT schedule
(reference: vggt/models/aggregator.py).

Global blocks 0..early_frame_split-1 run frame attention with the shared
cross-frame K/V set; blocks in [merging, merge_end] run K/V merging (core
blocks at core_merge_ratio); the rest run plain global attention.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .. import kernels
from ..nvtx import nvtx
from .dino import DinoVisionTransformer
from .layers import Block, PositionGetter, RotaryPositionEmbedding2D

_RESNET_MEAN = [0.485, 0.456, 0.406]
_RESNET_STD = [0.229, 0.224, 0.225]


def merge_window(block_num, merging, merge_end, early_frame_split, core_blocks, core_merge_ratio):
    """The merge-window rule of aggregator.py:316-325."""
    if merging is None:
        return False
    return (block_num >= merging and (merge_end < 0 or block_num <= merge_end)
            and block_num >= early_frame_split
            and (block_num not in core_blocks or core_merge_ratio > 0))


def special_tokens(token, B, S, first_frame=0):
    """[1, 2, X, C] -> [B*S, X, C] for frames first_frame.. first_frame+S-1:
    slot 0 for (global) frame 0, slot 1 for the others."""
    if first_frame > 0:
        return token[:, 1:].expand(B, S, *token.shape[2:]).reshape(B * S, *token.shape[2:])
    first = token[:, 0:1].expand(B, 1, *token.shape[2:])
    rest = token[:, 1:].expand(B, S - 1, *token.shape[2:])
    return torch.cat([first, rest], 1).reshape(B * S, *token.shape[2:])


class Aggregator(nn.Module):
    def __init__(self, img_size=518, patch_size=14, embed_dim=1024, depth=24, num_heads=16,
                 mlp_ratio=4.0, num_register_tokens=4, qk_norm=True, rope_freq=100,
                 init_values=0.01, merging=9, merge_end=23, merge_ratio=0.98, early_frame_split=9,
                 broadcast_pool=8, core_blocks=(13, 14, 15, 16), core_merge_ratio=0.2,
                 merge_metric_dim=128):
        super().__init__()
        self.patch_embed = DinoVisionTransformer(img_size=img_size, patch_size=patch_size,
                                                 embed_dim=embed_dim, num_register_tokens=num_register_tokens)
        self.rope = RotaryPositionEmbedding2D(frequency=rope_freq) if rope_freq > 0 else None
        self.position_getter = PositionGetter()
        self.merging, self.merge_end, self.merge_ratio = merging, merge_end, merge_ratio

        def blocks():
            return nn.ModuleList([
                Block(embed_dim, num_heads, mlp_ratio=mlp_ratio, init_values=init_values,
                      qk_norm=qk_norm, rope=self.rope, merge_ratio=merge_ratio) for _ in range(depth)])

        self.frame_blocks = blocks()
        self.global_blocks = blocks()
        self.early_frame_split = early_frame_split
        for i in range(min(early_frame_split, depth)):
            a = self.global_blocks[i].attn
            a.frame_special, a.num_special, a.broadcast_pool = True, 1 + num_register_tokens, broadcast_pool
        self.core_blocks = frozenset(core_blocks)
        self.core_merge_ratio = core_merge_ratio
        for i in self.core_blocks:
            if i < depth:
                self.global_blocks[i].attn.merge_ratio = core_merge_ratio
        for blk in self.global_blocks:
            blk.attn.merge_metric_dim = merge_metric_dim
        self.depth = depth
        self.patch_size = patch_size
        self.camera_token = nn.Parameter(torch.randn(1, 2, 1, embed_dim))
        self.register_token = nn.Parameter(torch.randn(1, 2, num_register_tokens, embed_dim))
        self.patch_start_idx = 1 + num_register_tokens
        self.shard = None
        self.tap_blocks = (4, 11, 17, 23)   # block outputs the DPT head reads (aggregator.py:296)
        self.register_buffer("_resnet_mean", torch.tensor(_RESNET_MEAN).view(1, 1, 3, 1, 1),
                             persistent=False)
        self.register_buffer("_resnet_std", torch.tensor(_RESNET_STD).view(1, 1, 3, 1, 1),
                             persistent=False)

    def set_shard(self, shard):
        """Run the global blocks with their queries sharded by frame (shard.py);
        forward() then receives only this rank's frames."""
        self.shard = shard
        for blk in self.global_blocks:
            blk.attn.shard = shard

    def set_patch_dims(self, pw, ph):
        for m in self.modules():
            if hasattr(m, "patch_width") and hasattr(m, "patch_height"):
                m.patch_width, m.patch_height = pw, ph

    def forward(self, images):
        """images [B, S, 3, H, W] in [0, 1] -> (4 DPT taps [B, S, P, 2C], patch_start_idx)."""
        B, S, _, H, W = images.shape
        dt = self.camera_token.dtype
        x = ((images - self._resnet_mean) / self._resnet_std).to(dt).view(B * S, 3, H, W)
        with nvtx("dino_embed"):
            patch = self.patch_embed(x).to(dt)
        f0 = self.shard.f0 if self.shard is not None else 0
        tokens = torch.cat([special_tokens(self.camera_token, B, S, f0),
                            special_tokens(self.register_token, B, S, f0), patch], 1).to(dt)
        pos = self.position_getter(B * S, H // self.patch_size, W // self.patch_size, images.device) + 1
        pos = torch.cat([torch.zeros(B * S, self.patch_start_idx, 2, device=images.device,
                                     dtype=pos.dtype), pos], 1)
        P, C = tokens.shape[1], tokens.shape[2]
        taps = []
        for b in range(self.depth):
            with nvtx(f"frame_block_{b}"):
                tokens = self.frame_blocks[b](tokens.view(B * S, P, C), pos=pos)
            frame_out = tokens.view(B, S, P, C)
            gm = b if merge_window(b, self.merging, self.merge_end, self.early_frame_split,
                                   self.core_blocks, self.core_merge_ratio) else None
            attn = self.global_blocks[b].attn
            kind = ("frame_shared" if attn.frame_special else
                    ("plain" if gm is None else ("core" if b in self.core_blocks else "merged")))
            with nvtx(f"global_block_{b}_{kind}"):
                tokens = self.global_blocks[b](tokens.view(B, S * P, C), pos=pos.view(B, S * P, 2),
                                               global_merging=gm)
            if b in self.tap_blocks:
                taps.append(torch.cat([frame_out, tokens.view(B, S, P, C)], -1))
        if images.is_cuda:
            # one read of the device's status word per forward: a pipeline wait
            # that gave up in any kernel above raises here (kernels.py)
            kernels.check_device_status(images.device, "aggregator forward")
        return taps, self.patch_start_idx
