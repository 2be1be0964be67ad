"""Fused similarity + row argmax (drop-in for merging/fused_similarity.py).

``fused_similarity_argmax(a, b)`` has the contract of the reference's
merging/fused_similarity.py:81-112: node_max, node_idx = max / first argmax
over j of a_i . b_j, inputs cast to bf16, fp32 accumulation, node_max in a's
dtype and node_idx int64.  The work runs in the tcgen05 kernel
``gpa_sim_argmax``; the [M, N] score matrix is never materialised.
"""
import torch

from .. import kernels


def fused_similarity_argmax(a: torch.Tensor, b: torch.Tensor):
    """node_max, node_idx = (a @ b.transpose(-1,-2)).max(dim=-1), fused.

    a: [B, M, D] src metric, b: [B, N, D] dst metric (CUDA, bf16/fp32; fp16
    is converted to bf16).  Returns node_max [B, M] (a.dtype), node_idx [B, M]
    (int64).
    """
    assert a.is_cuda and b.is_cuda and a.dim() == 3 and b.dim() == 3
    out_dtype = a.dtype
    node_max, node_idx = kernels.sim_argmax(a.to(torch.bfloat16), b.to(torch.bfloat16))
    return node_max.to(out_dtype), node_idx.to(torch.long)
