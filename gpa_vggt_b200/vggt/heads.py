"""Camera and depth heads of VGGT (reference: vggt/heads/camera_head.py,
dpt_head.py, head_act.py, utils.py).  These consume the aggregator's tokens;
they are outside the GPA path and run on torch (cuBLAS/cuDNN/SDPA).
Parameter names follow the reference."""
from __future__ import annotations

from typing import List

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import kernels

from .layers import Block, LayerNorm, Mlp, SdpaAttention


# ---------------------------------------------------------------------------
# camera head (camera_head.py)
# ---------------------------------------------------------------------------
class CameraHead(nn.Module):
    def __init__(self, dim_in=2048, trunk_depth=4, num_heads=16, mlp_ratio=4, init_values=0.01):
        super().__init__()
        self.target_dim = 9
        self.trunk = nn.Sequential(*[
            Block(dim_in, num_heads, mlp_ratio=mlp_ratio, init_values=init_values,
                  attn_class=SdpaAttention) for _ in range(trunk_depth)])
        self.token_norm = LayerNorm(dim_in)
        self.trunk_norm = LayerNorm(dim_in)
        self.empty_pose_tokens = nn.Parameter(torch.zeros(1, 1, self.target_dim))
        self.embed_pose = nn.Linear(self.target_dim, dim_in)
        self.poseLN_modulation = nn.Sequential(nn.SiLU(), nn.Linear(dim_in, 3 * dim_in, bias=True))
        self.adaln_norm = nn.LayerNorm(dim_in, elementwise_affine=False, eps=1e-6)
        self.pose_branch = Mlp(dim_in, dim_in // 2, self.target_dim)

    def forward(self, taps: List[torch.Tensor], num_iterations: int = 4, shard=None) -> List[torch.Tensor]:
        cam = taps[-1][:, :, 0]                                   # [B, S, 2C] camera tokens
        if shard is not None and shard.active:                    # every frame's camera token
            cam = shard.gather(cam[0].contiguous())[None]
        pose_tokens = self.token_norm(cam)
        B, S, C = pose_tokens.shape
        pred, out = None, []
        for _ in range(num_iterations):
            inp = self.embed_pose(self.empty_pose_tokens.expand(B, S, -1) if pred is None
                                  else pred.detach())
            shift, scale, gate = self.poseLN_modulation(inp).chunk(3, dim=-1)
            t = gate * (self.adaln_norm(pose_tokens) * (1 + scale) + shift) + pose_tokens
            t = self.trunk(t)
            delta = self.pose_branch(self.trunk_norm(t))
            pred = delta if pred is None else pred + delta
            # activate_pose with trans/quat linear and relu on the field of view
            out.append(torch.cat([pred[..., :7], F.relu(pred[..., 7:])], -1))
        return out


# ---------------------------------------------------------------------------
# DPT depth head (dpt_head.py, utils.py)
# ---------------------------------------------------------------------------
def _uv_grid(w, h, aspect, dtype, device):
    """Normalised (w, h, 2) grid spanning +-(aspect, 1)/diag (utils.py create_uv_grid)."""
    diag = (aspect ** 2 + 1.0) ** 0.5
    sx, sy = aspect / diag, 1.0 / diag
    xs = torch.linspace(-sx * (w - 1) / w, sx * (w - 1) / w, steps=w, dtype=dtype, device=device)
    ys = torch.linspace(-sy * (h - 1) / h, sy * (h - 1) / h, steps=h, dtype=dtype, device=device)
    uu, vv = torch.meshgrid(xs, ys, indexing="xy")
    return torch.stack((uu, vv), dim=-1)


def _sincos(dim, pos, omega_0=100.0):
    omega = torch.arange(dim // 2, dtype=torch.double, device=pos.device) / (dim / 2.0)
    omega = 1.0 / omega_0 ** omega
    out = torch.outer(pos.reshape(-1), omega)
    return torch.cat([out.sin(), out.cos()], 1).float()


def _grid_embed(grid, dim):
    H, W, _ = grid.shape
    flat = grid.reshape(-1, 2)
    return torch.cat([_sincos(dim // 2, flat[:, 0]), _sincos(dim // 2, flat[:, 1])], -1).view(H, W, dim)


def _interp(x, size=None, scale_factor=None, mode="bilinear", align_corners=True):
    """Bilinear resize, chunked along the batch to stay under int32 index limits
    (dpt_head.py custom_interpolate)."""
    if size is None:
        size = (int(x.shape[-2] * scale_factor), int(x.shape[-1] * scale_factor))
    limit = 1610612736
    n = size[0] * size[1] * x.shape[0] * x.shape[1]
    if n > limit:
        parts = torch.chunk(x, (n // limit) + 1, dim=0)
        return torch.cat([F.interpolate(p, size=size, mode=mode, align_corners=align_corners)
                          for p in parts], 0).contiguous()
    return F.interpolate(x, size=size, mode=mode, align_corners=align_corners)


_RESIZE_FP32: dict = {}


def _autocast_resize_in_fp32(device) -> bool:
    """Whether bf16 autocast runs a bilinear resize of a bf16 map in fp32 (and
    returns fp32); probed once per device."""
    key = (device.type, device.index)
    if key not in _RESIZE_FP32:
        with torch.autocast(device.type, dtype=torch.bfloat16):
            y = F.interpolate(torch.zeros(1, 8, 2, 2, device=device, dtype=torch.bfloat16), size=(3, 3),
                              mode="bilinear", align_corners=True)
        _RESIZE_FP32[key] = y.dtype == torch.float32
    return _RESIZE_FP32[key]


def _fused_resize_ok(x) -> bool:
    """The resize feeds an autocast bf16 convolution and the map is channels-last
    on CUDA: the fused resize kernel gives that convolution the same input."""
    return (x.is_cuda and x.dim() == 4 and x.dtype in (torch.bfloat16, torch.float32)
            and torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16
            and x.stride(1) == 1 and x.shape[1] % 8 == 0)


# Convolutions of the head that carry a bias: on CUDA channels-last bf16 maps
# under bf16 autocast, the convolution runs without its bias and one pass adds
# the bias, the ReLU and the residual (kernels.bias_act), rounding as torch's
# separate bf16 ops do; elsewhere the torch ops run.
FUSED_CONV_EPILOGUE = True


def _conv_act(conv, x, relu=False, res=None, transpose=False):
    """conv(x), then ReLU if relu, then + res if res is given (torch semantics)."""
    if (FUSED_CONV_EPILOGUE and conv.bias is not None and x.is_cuda and x.dim() == 4
            and torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16
            and conv.out_channels % 8 == 0 and conv.groups == 1):
        if transpose:
            y = F.conv_transpose2d(x, conv.weight, None, conv.stride, conv.padding,
                                   conv.output_padding, conv.groups, conv.dilation)
        else:
            y = F.conv2d(x, conv.weight, None, conv.stride, conv.padding, conv.dilation, conv.groups)
        cl = torch.channels_last
        if (y.dtype == torch.bfloat16 and y.is_contiguous(memory_format=cl)
                and (res is None or (res.dtype == torch.bfloat16 and res.shape == y.shape
                                     and res.is_contiguous(memory_format=cl)))):
            return kernels.bias_act(y, conv.bias, res, relu)
        y = y + conv.bias.to(y.dtype)[None, :, None, None]   # the bias add torch would do
    else:
        y = conv(x)
    if relu:
        y = F.relu(y)
    return y if res is None else y + res


class ResidualConvUnit(nn.Module):
    """conv2(relu(conv1(relu(x)))) + relu(x): the reference's activation is an
    in-place ReLU applied to the unit's input, so its skip connection carries
    relu(x) (dpt_head.py ResidualConvUnit)."""

    def __init__(self, features):
        super().__init__()
        self.conv1 = nn.Conv2d(features, features, 3, 1, 1, bias=True)
        self.conv2 = nn.Conv2d(features, features, 3, 1, 1, bias=True)

    def forward(self, x):
        x = F.relu(x)
        return _conv_act(self.conv2, _conv_act(self.conv1, x, relu=True), res=x)


class FeatureFusionBlock(nn.Module):
    def __init__(self, features, has_residual=True):
        super().__init__()
        self.out_conv = nn.Conv2d(features, features, 1, 1, 0, bias=True)
        if has_residual:
            self.resConfUnit1 = ResidualConvUnit(features)
        self.has_residual = has_residual
        self.resConfUnit2 = ResidualConvUnit(features)

    def forward(self, *xs, size=None):
        out = xs[0]
        if self.has_residual:
            out = out + self.resConfUnit1(xs[1])
        out = self.resConfUnit2(out)
        if size is None:
            size = (int(out.shape[-2] * 2), int(out.shape[-1] * 2))
        if _fused_resize_ok(out):   # resize + the conv's bf16 input cast, one pass
            out = kernels.upsample_bilinear_bf16(out, size)
        else:
            out = _interp(out, size=size)
        return _conv_act(self.out_conv, out)


class DPTHead(nn.Module):
    def __init__(self, dim_in, patch_size=14, output_dim=2, activation="exp", conf_activation="expp1",
                 features=256, out_channels=(256, 512, 1024, 1024)):
        super().__init__()
        self.patch_size = patch_size
        self.activation, self.conf_activation = activation, conf_activation
        self.norm = LayerNorm(dim_in)
        self.projects = nn.ModuleList([nn.Conv2d(dim_in, oc, 1) for oc in out_channels])
        self.resize_layers = nn.ModuleList([
            nn.ConvTranspose2d(out_channels[0], out_channels[0], 4, 4),
            nn.ConvTranspose2d(out_channels[1], out_channels[1], 2, 2),
            nn.Identity(),
            nn.Conv2d(out_channels[3], out_channels[3], 3, 2, 1)])
        sc = nn.Module()
        for i, oc in enumerate(out_channels):
            setattr(sc, f"layer{i + 1}_rn", nn.Conv2d(oc, features, 3, 1, 1, bias=False))
        sc.stem_transpose = nn.Identity()
        sc.refinenet1 = FeatureFusionBlock(features)
        sc.refinenet2 = FeatureFusionBlock(features)
        sc.refinenet3 = FeatureFusionBlock(features)
        sc.refinenet4 = FeatureFusionBlock(features, has_residual=False)
        sc.output_conv1 = nn.Conv2d(features, features // 2, 3, 1, 1)
        sc.output_conv2 = nn.Sequential(nn.Conv2d(features // 2, 32, 3, 1, 1), nn.ReLU(inplace=True),
                                        nn.Conv2d(32, output_dim, 1, 1, 0))
        self.scratch = sc
        self._pe = {}

    def _pe_map(self, C, h, w, dtype, device, W, H, ratio=0.1):
        """The fp32 positional map [1, C, h, w] (channel stride 1) for a map of
        `dtype` (the uv grid is built in that dtype, as the reference does)."""
        key = (C, h, w, dtype, str(device), W, H)
        pe = self._pe.get(key)
        if pe is None:
            grid = _uv_grid(w, h, W / H, dtype, device)
            pe = (_grid_embed(grid, C) * ratio).permute(2, 0, 1)[None]  # fp32, as the reference
            self._pe[key] = pe
        return pe

    def _pos(self, x, W, H):
        return x + self._pe_map(x.shape[1], x.shape[2], x.shape[3], x.dtype, x.device, W, H)

    def _chunk(self, taps, images, psi, f0, f1):
        imgs = images[:, f0:f1]
        B, S, _, H, W = imgs.shape
        ph, pw = H // self.patch_size, W // self.patch_size
        feats = []
        for i, tap in enumerate(taps):
            x = tap[:, f0:f1, psi:].reshape(B * S, -1, tap.shape[-1])
            x = self.norm(x).permute(0, 2, 1).reshape(B * S, -1, ph, pw)
            x = self._pos(self.projects[i](x), W, H)
            rl = self.resize_layers[i]
            if isinstance(rl, nn.ConvTranspose2d):
                x = _conv_act(rl, x, transpose=True)
            elif isinstance(rl, nn.Conv2d):
                x = _conv_act(rl, x)
            else:
                x = rl(x)
            feats.append(x)
        sc = self.scratch
        l1, l2, l3, l4 = (getattr(sc, f"layer{i + 1}_rn")(f) for i, f in enumerate(feats))
        out = sc.refinenet4(l4, size=l3.shape[2:])
        out = sc.refinenet3(out, l3, size=l2.shape[2:])
        out = sc.refinenet2(out, l2, size=l1.shape[2:])
        out = sc.refinenet1(out, l1)
        out = _conv_act(sc.output_conv1, out)
        size = (ph * self.patch_size, pw * self.patch_size)
        if _fused_resize_ok(out):
            # resize, the fp32 positional add and the conv's bf16 input cast in one
            # pass; the add sees the resize's own dtype under autocast
            fp32 = _autocast_resize_in_fp32(out.device)
            pe = self._pe_map(out.shape[1], size[0], size[1], torch.float32 if fp32 else out.dtype,
                              out.device, W, H)
            up = kernels.upsample_bilinear_bf16(out, size, add=pe, round_first=not fp32)
            oc = sc.output_conv2
            out = oc[2](_conv_act(oc[0], up, relu=True))
        else:
            out = _interp(out, size=size)
            out = sc.output_conv2(self._pos(out, W, H))
        fmap = out.permute(0, 2, 3, 1)
        depth = torch.exp(fmap[..., :-1])          # activation "exp"
        conf = 1 + fmap[..., -1].exp()             # conf_activation "expp1"
        return depth.view(B, S, *depth.shape[1:]), conf.view(B, S, *conf.shape[1:])

    def forward(self, taps, images, patch_start_idx, frames_chunk_size=8):
        S = images.shape[1]
        if not frames_chunk_size or frames_chunk_size >= S:
            return self._chunk(taps, images, patch_start_idx, 0, S)
        ds, cs = [], []
        for f0 in range(0, S, frames_chunk_size):
            d, c = self._chunk(taps, images, patch_start_idx, f0, min(f0 + frames_chunk_size, S))
            ds.append(d)
            cs.append(c)
        return torch.cat(ds, 1), torch.cat(cs, 1)
