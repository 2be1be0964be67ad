"""Bipartite K/V token merging (drop-in for merging/merge.py).

``token_merge_bipartite2d`` keeps the signature and return contract of the
reference's merging/merge.py:39-256.  The device work is done by the sm_100a
kernels: dst/src roles (``gpa_merge_roles``), metric normalise + split
(``gpa_metric_split``), similarity argmax (``gpa_sim_argmax``), the merge plan
(``gpa_merge_plan``) and the scatter-mean (``gpa_merge_kv_mean``).  The two
random draws (the dst pick per window and the projection basis) are made with
the same torch RNG calls on the same device as the reference, so a CUDA run
sees exactly the reference's CUDA draws.

Representation differences (results are the same up to slot order):
  * dst slots are in ascending token position, unmerged src slots in
    ascending src ordinal (the reference orders them by unstable argsorts,
    merge.py:165 and :199); attention over the merged keys is invariant to
    this permutation.
  * at the top-r cut, ties in node_max go to the lower src ordinal.
  * group sums are fp32 in a fixed order (deterministic).
"""
import os
from typing import Callable, Optional

import torch

from .. import kernels

PROJ_SEED = 1234

_proj_cache = {}


def projection_basis(c: int, metric_dim: int, device, dtype) -> torch.Tensor:
    """The fixed Gaussian basis of merge.py:180-184, drawn like the reference."""
    key = (str(device), c, metric_dim, dtype)
    p = _proj_cache.get(key)
    if p is None:
        g = torch.Generator(device=device)
        g.manual_seed(PROJ_SEED)
        p = torch.randn(c, metric_dim, device=device, dtype=torch.float32, generator=g).to(dtype)
        _proj_cache[key] = p
    return p


_proj_t_cache = {}


def projection_basis_t(c: int, metric_dim: int, device) -> torch.Tensor:
    """proj^T [metric_dim, c] in bf16, contiguous (the fused projection kernel's
    K-major operand), drawn as projection_basis draws proj."""
    key = (str(device), c, metric_dim)
    p = _proj_t_cache.get(key)
    if p is None:
        p = projection_basis(c, metric_dim, device, torch.bfloat16).t().contiguous()
        _proj_t_cache[key] = p
    return p


# The one-kernel projection sums the product in its own order, so about one
# metric element in 10^5 rounds to the other bf16 neighbour than the
# reference's cuBLAS product; a src row whose two best dst tokens are closer
# than about 5e-4 can then match the other one.  GPA_FUSED_METRIC=0 keeps
# torch's GEMM for the product (bit-identical matcher inputs).
FUSED_METRIC = os.environ.get("GPA_FUSED_METRIC", "1") == "1"


def fused_metric_ok(metric: torch.Tensor, metric_dim: int) -> bool:
    """Whether the one-kernel projection + normalisation applies: a bf16 metric
    (the autocast run) projected to 128 dims from a width that is a multiple of 64."""
    C = metric.shape[-1]
    return (FUSED_METRIC and metric.dtype == torch.bfloat16 and metric_dim == 128 and C > 128
            and C % 64 == 0)


def draw_dst_choice(num_imgs: int, w: int, h: int, sx: int, sy: int, device,
                    generator: Optional[torch.Generator]) -> Optional[torch.Tensor]:
    """The per-window dst pick of merge.py:121-126 (same RNG call)."""
    if num_imgs <= 1:
        return None
    return torch.randint(sy * sx, size=(num_imgs - 1, h // sy, w // sx), device=device,
                         generator=generator)


def build_plan(metric: torch.Tensor, w: int, h: int, sx: int, sy: int, r: int,
               no_rand: bool = False, generator: Optional[torch.Generator] = None,
               metric_dim: int = 0, num_special: int = 5,
               rand_idx: Optional[torch.Tensor] = None,
               proj: Optional[torch.Tensor] = None) -> kernels.MergePlan:
    """Merge plan for metric [N, C] (one batch element).

    ``rand_idx`` / ``proj`` override the two RNG draws (tests inject the values
    a CPU run drew); by default they are drawn as the reference does.
    """
    N, C = metric.shape
    tokens_per_img = w * h + num_special
    num_imgs = N // tokens_per_img
    assert tokens_per_img * num_imgs == N, (
        f"Token count doesn't match (w*h+{num_special})*num_imgs: N={N} w={w} h={h}")
    dev = metric.device
    if not no_rand and rand_idx is None:
        rand_idx = draw_dst_choice(num_imgs, w, h, sx, sy, dev, generator)
    dst_pos, src_pos, slot = kernels.merge_roles(None if no_rand else rand_idx, num_imgs, w, h,
                                                 sx, sy, num_special, no_rand, dev)
    with torch.no_grad():
        if fused_metric_ok(metric, metric_dim):
            # projection, bf16 rounding, fp32 normalisation and split in one kernel
            proj_t = (projection_basis_t(C, metric_dim, dev) if proj is None
                      else proj.to(torch.bfloat16).t().contiguous())
            a, b = kernels.proj_norm_split(metric, proj_t, slot, src_pos.numel(), dst_pos.numel())
        else:
            if metric_dim and metric_dim < C:
                if proj is None:
                    proj = projection_basis(C, metric_dim, dev, metric.dtype)
                metric = metric @ proj.to(metric.dtype)
            a, b = kernels.metric_split(metric, src_pos, dst_pos)
        if src_pos.numel():
            node_max, node_idx = kernels.sim_argmax(a[None], b[None])
        else:
            node_max = torch.empty(1, 0, device=dev)
            node_idx = torch.empty(1, 0, device=dev, dtype=torch.int32)
        return kernels.merge_plan(node_max[0], node_idx[0], r, dst_pos, src_pos)


def token_merge_bipartite2d(
    metric: torch.Tensor,
    w: int,
    h: int,
    sx: int,
    sy: int,
    r: int,
    no_rand: bool = False,
    generator: Optional[torch.Generator] = None,
    metric_dim: int = 0,
    num_special: int = 5,
) -> Callable:
    """Bipartite token merging over the multi-frame token sequence.

    Same arguments and return contract as the reference (merge.py:39-72):
    returns ``merge(x [B, N, C], mode) -> [B, N_m, C]`` with
    ``merge.heads(t [B, H, N, D], mode)`` and ``merge.size`` ([B, N_m] fp32
    token counts, None for B > 1).
    """
    B, N, _ = metric.shape
    if r <= 0:
        raise ValueError("token_merge_bipartite2d: r must be positive")
    if not metric.is_cuda:
        raise ValueError("token_merge_bipartite2d: CUDA tensors required (no CPU fallback)")
    tokens_per_img = w * h + num_special
    num_imgs = N // tokens_per_img
    assert tokens_per_img * num_imgs == N, (
        f"Token count doesn't match (w*h+{num_special})*num_imgs: N={N} w={w} h={h}")
    # one dst draw for the whole batch (merge.py:121-126 draws once; the
    # matching is then per batch element)
    rand_idx = None if no_rand else draw_dst_choice(num_imgs, w, h, sx, sy, metric.device, generator)
    plans = [build_plan(metric[bi], w, h, sx, sy, r, no_rand, None, metric_dim, num_special,
                        rand_idx=rand_idx) for bi in range(B)]
    n_out = plans[0].n_out

    def merge(x: torch.Tensor, mode: str = "mean") -> torch.Tensor:
        """[B, N, C] -> [B, unm_len + num_dst, C]: unmerged src, then dst."""
        if mode not in ("mean", "sum"):
            raise ValueError(f"merge: unsupported mode {mode!r}")
        C = x.shape[-1]
        pad = (-C) % 8                 # the kernel moves 8-element chunks
        xx = torch.nn.functional.pad(x, (0, pad)) if pad else x
        outs = [kernels.merge_kv(xx[bi][None], plans[bi], mean=(mode == "mean"))[0, :, :C]
                for bi in range(x.shape[0])]
        return torch.stack(outs, 0)

    def merge_heads(t: torch.Tensor, mode: str = "mean") -> torch.Tensor:
        """Merge [B, H, N, D] K/V directly in the attention-kernel layout."""
        n_t, h_t, n_tokens, d_t = t.shape
        if n_t != B or n_tokens != N:
            raise ValueError("merge_heads input does not match the merge mapping")
        if mode not in ("mean", "sum"):
            raise ValueError(f"merge_heads: unsupported mode {mode!r}")
        out = torch.empty(n_t, h_t, n_out, d_t, device=t.device, dtype=t.dtype)
        for bi in range(n_t):
            kernels.merge_kv(t[bi], plans[bi], mean=(mode == "mean"), out=out[bi])
        return out

    merge.size = plans[0].counts[None] if B == 1 else None
    merge.heads = merge_heads
    merge.plans = plans
    return merge
