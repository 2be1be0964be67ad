"""DINOv2 ViT-L/14 with 4 register tokens, the per-frame patch embedder of the
aggregator (reference: vggt/layers/vision_transformer.py, built by
vggt/models/aggregator.py:192-236).  Parameter names follow the reference; the
blocks' attention runs on the sm_100a kernel (plain attention per frame)."""
from __future__ import annotations

import math
from functools import partial

import torch
import torch.nn as nn
import torch.nn.functional as F

from .layers import Block, LayerNorm, PatchEmbed


class DinoVisionTransformer(nn.Module):
    def __init__(self, img_size=518, patch_size=14, in_chans=3, embed_dim=1024, depth=24,
                 num_heads=16, mlp_ratio=4.0, init_values=1.0, num_register_tokens=4,
                 interpolate_antialias=True, interpolate_offset=0.0):
        super().__init__()
        norm_layer = partial(LayerNorm, eps=1e-6)
        self.embed_dim = embed_dim
        self.patch_size = patch_size
        self.num_register_tokens = num_register_tokens
        self.interpolate_antialias = interpolate_antialias
        self.interpolate_offset = interpolate_offset
        self.patch_embed = PatchEmbed(img_size, patch_size, in_chans, embed_dim)
        n = self.patch_embed.num_patches
        self.cls_token = nn.Parameter(torch.zeros(1, 1, embed_dim))
        self.pos_embed = nn.Parameter(torch.zeros(1, n + 1, embed_dim))
        self.register_tokens = nn.Parameter(torch.zeros(1, num_register_tokens, embed_dim))
        self.mask_token = nn.Parameter(torch.zeros(1, embed_dim))
        self.blocks = nn.ModuleList([
            Block(embed_dim, num_heads, mlp_ratio=mlp_ratio, norm_layer=norm_layer,
                  init_values=init_values) for _ in range(depth)])
        self.norm = norm_layer(embed_dim)
        self.head = nn.Identity()

    def _pos_embed(self, n_patch, w, h):
        """Positional table, resized bicubically when the grid differs
        (vision_transformer.py:213-245)."""
        N = self.pos_embed.shape[1] - 1
        if n_patch == N and w == h:
            return self.pos_embed
        cls_pe, patch_pe = self.pos_embed[:, :1], self.pos_embed[:, 1:]
        M = int(math.sqrt(N))
        w0, h0 = w // self.patch_size, h // self.patch_size
        kw = ({"scale_factor": ((w0 + self.interpolate_offset) / M, (h0 + self.interpolate_offset) / M)}
              if self.interpolate_offset else {"size": (w0, h0)})
        patch_pe = F.interpolate(patch_pe.reshape(1, M, M, -1).permute(0, 3, 1, 2), mode="bicubic",
                                 antialias=self.interpolate_antialias, **kw)
        patch_pe = patch_pe.permute(0, 2, 3, 1).reshape(1, -1, self.embed_dim)
        return torch.cat([cls_pe, patch_pe], 1).to(self.pos_embed.dtype)

    def forward(self, x):
        """[B, 3, H, W] -> normed patch tokens [B, (H/14)*(W/14), C]."""
        B, _, w, h = x.shape
        t = self.patch_embed(x)
        t = torch.cat([self.cls_token.expand(B, -1, -1), t], 1)
        t = t + self._pos_embed(t.shape[1] - 1, w, h)
        t = torch.cat([t[:, :1], self.register_tokens.expand(B, -1, -1), t[:, 1:]], 1)
        for blk in self.blocks:
            t = blk(t)
        return self.norm(t)[:, self.num_register_tokens + 1:]
