"""Flash attention with a per-key additive bias (drop-in for
merging/fused_attention.py).

``attention_keybias(q, k, v, bias, sm_scale, return_lse)`` follows the
reference's merging/fused_attention.py:130-180: SDPA(q, k, v, attn_mask=bias)
for a per-key bias [B, H, 1, N] (or None), fp32 q/k/v/bias first cast to the
autocast dtype (bf16 by default), optional log2 softmax denominators
[B, H, M] fp32.  The kernel is ``gpa_attention_keybias`` (tcgen05, head_dim 64).
"""
import torch

from .. import kernels

LOG2E = 1.4426950408889634


def attention_keybias(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      bias, sm_scale: float, return_lse: bool = False):
    """SDPA(q, k, v, attn_mask=bias) where bias is per-key: [B, H, 1, N].

    q [B, H, M, D], k/v [B, H, N, D] (CUDA, bf16; fp32 is cast first as in the
    reference).  Returns [B, H, M, D] bf16, and with return_lse also
    [B, H, M] fp32 log2 softmax denominators.  `bias` may be None.
    """
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("attention_keybias: CUDA tensors required (no CPU fallback)")
    if q.dtype == torch.float32:
        dt = torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else torch.bfloat16
        q, k, v = q.to(dt), k.to(dt), v.to(dt)
        bias = None if bias is None else bias.to(dt)
    if q.dtype == torch.float16:
        raise NotImplementedError("attention_keybias: fp16 inputs are not supported (bf16 only)")
    v = v.to(q.dtype)
    return kernels.attention(q, k, v, bias, sm_scale, return_lse=return_lse)
