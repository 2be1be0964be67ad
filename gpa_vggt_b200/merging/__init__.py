"""Drop-in for the reference's ``merging`` package (merge.py,
fused_similarity.py, fused_attention.py), backed by the sm_100a kernels."""
from . import merge  # noqa: F401
from .fused_similarity import fused_similarity_argmax  # noqa: F401
from .fused_attention import attention_keybias  # noqa: F401

__all__ = ["merge", "fused_similarity_argmax", "attention_keybias"]
