"""VGGT with the GPA-VGGT schedule on the B200 attention path (the path's
end-to-end caller; see model.VGGT)."""
from .model import VGGT, init_weights, vanilla_config  # noqa: F401
