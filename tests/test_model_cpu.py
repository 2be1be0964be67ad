"""Model structure (no GPU): the GPA-VGGT caller has the reference's parameter
layout, the GPA block schedule, and deterministic name-keyed weights."""
import torch

from gpa_vggt_b200.vggt import VGGT, init_weights
from gpa_vggt_b200.vggt.aggregator import merge_window


def test_parameter_count_and_schedule():
    with torch.device("meta"):
        m = VGGT()
    n = sum(p.numel() for p in m.parameters())
    assert n == 1_157_941_492            # VGGT-1B with camera + depth heads
    agg = m.aggregator
    early = [i for i, b in enumerate(agg.global_blocks) if b.attn.frame_special]
    assert early == list(range(9))
    merged = [b for b in range(24) if merge_window(b, agg.merging, agg.merge_end, agg.early_frame_split,
                                                   agg.core_blocks, agg.core_merge_ratio)]
    assert merged == list(range(9, 24))
    assert [agg.global_blocks[i].attn.merge_ratio for i in (9, 13, 16, 17)] == [0.98, 0.2, 0.2, 0.98]
    assert all(b.attn.merge_metric_dim == 128 for b in agg.global_blocks)


def test_init_weights_is_name_keyed():
    a = torch.nn.ModuleDict({"x": torch.nn.Linear(4, 3), "y": torch.nn.LayerNorm(3)})
    b = torch.nn.ModuleDict({"y": torch.nn.LayerNorm(3), "x": torch.nn.Linear(4, 3)})
    init_weights(a, 0)
    init_weights(b, 0)
    for k, v in a.state_dict().items():
        assert torch.equal(v, b.state_dict()[k])
