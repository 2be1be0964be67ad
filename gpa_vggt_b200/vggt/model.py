"""VGGT with the GPA-VGGT configuration (reference: vggt/models/vggt.py), the
end-to-end caller of the B200 attention path.  Defaults are the paper's GPA
configuration; vanilla VGGT is ``merging=None, early_frame_split=0``."""
from __future__ import annotations

import torch
import torch.nn as nn

from .aggregator import Aggregator
from .heads import CameraHead, DPTHead


class VGGT(nn.Module):
    def __init__(self, img_size=518, patch_size=14, embed_dim=1024, enable_camera=True,
                 enable_depth=True, merging=9, merge_end=23, merge_ratio=0.98, early_frame_split=9,
                 broadcast_pool=8, core_blocks=(13, 14, 15, 16), core_merge_ratio=0.2,
                 merge_metric_dim=128):
        super().__init__()
        self.aggregator = Aggregator(img_size=img_size, patch_size=patch_size, embed_dim=embed_dim,
                                     merging=merging, merge_end=merge_end, merge_ratio=merge_ratio,
                                     early_frame_split=early_frame_split, broadcast_pool=broadcast_pool,
                                     core_blocks=core_blocks, core_merge_ratio=core_merge_ratio,
                                     merge_metric_dim=merge_metric_dim)
        self.camera_head = CameraHead(dim_in=2 * embed_dim) if enable_camera else None
        self.depth_head = DPTHead(dim_in=2 * embed_dim, output_dim=2, activation="exp",
                                  conf_activation="expp1") if enable_depth else None

    def update_patch_dimensions(self, patch_width: int, patch_height: int):
        self.aggregator.set_patch_dims(patch_width, patch_height)

    def set_shard(self, shard):
        """Shard the frames across the ranks of shard.group (see shard.py):
        forward() takes this rank's frames and returns their depth, and the
        camera encoding of every frame."""
        self.aggregator.set_shard(shard)

    def forward(self, images: torch.Tensor):
        if images.dim() == 4:
            images = images[None]
        taps, psi = self.aggregator(images)
        out = {}
        if self.camera_head is not None:
            poses = self.camera_head(taps, shard=self.aggregator.shard)
            out["pose_enc"] = poses[-1]
            out["pose_enc_list"] = poses
        if self.depth_head is not None:
            out["depth"], out["depth_conf"] = self.depth_head(taps, images=images, patch_start_idx=psi)
        return out


def vanilla_config():
    return dict(merging=None, early_frame_split=0)


@torch.no_grad()
def init_weights(model: nn.Module, seed: int = 0) -> nn.Module:
    """Deterministic random weights that depend only on each parameter's name and
    shape (so the same values load into any model with these names): weights of
    linear/conv layers ~ N(0, 1/fan_in), biases ~ N(0, 0.02), norm weights
    1 + N(0, 0.02), layer-scale gammas keep their init value, tokens N(0, 0.02)."""
    for name, p in sorted(model.named_parameters(), key=lambda kv: kv[0]):
        g = torch.Generator().manual_seed((hash_name(name) + seed) % (2 ** 63))
        leaf = name.rsplit(".", 1)[-1]
        if leaf == "gamma":
            continue
        if p.dim() >= 2 and ("weight" in leaf):
            fan_in = p[0].numel()
            v = torch.randn(p.shape, generator=g) / fan_in ** 0.5
        elif leaf == "weight":                         # norm scales
            v = 1 + 0.02 * torch.randn(p.shape, generator=g)
        else:                                          # biases, tokens, embeddings
            v = 0.02 * torch.randn(p.shape, generator=g)
        p.copy_(v.to(p.dtype))
    return model


def hash_name(name: str) -> int:
    """Stable 63-bit FNV-1a hash of a parameter name."""
    h = 0xcbf29ce484222325
    for ch in name.encode():
        h ^= ch
        h = (h * 0x100000001b3) % (1 << 64)
    return h >> 1
