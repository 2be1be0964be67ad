"""The drop-in, literally: the reference's own Attention module
(vggt/layers/attention.py from the unmodified reference in baseline/_ref) runs
with the import shim of INTEGRATION.md, so its `merging` imports resolve to
gpa_vggt_b200.merging, and its output is compared with the same module on its
own path (its Triton kernels) -- same weights (init_weights, seed 0), same
input, same CUDA draws, bf16 autocast.  Each side runs in a fresh process (the
shim must be in place before the reference's module is imported).  Both the
merged global block (global_merging=9) and the early frame + shared-set block
are checked; the bound is rel-L2 < 2e-2."""
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not (REF / "vggt" / "layers" / "attention.py").exists(),
                                 reason="the reference is not installed in baseline/_ref")]

SCRIPT = r'''
import sys, torch
ROOT, REF, SHIM, MODE, OUT = sys.argv[1:6]
sys.path.insert(0, ROOT)
if SHIM == "1":
    import gpa_vggt_b200.merging as m
    sys.modules["merging"] = m
    sys.modules["merging.merge"] = m.merge
    sys.modules["merging.fused_similarity"] = m.fused_similarity
    sys.modules["merging.fused_attention"] = m.fused_attention
sys.path.insert(1, REF)
import vggt.layers.attention as A                        # the reference's module
from vggt.layers.rope import RotaryPositionEmbedding2D, PositionGetter
from gpa_vggt_b200.vggt.model import init_weights
if SHIM == "1":
    assert A.token_merge_bipartite2d.__module__ == "gpa_vggt_b200.merging.merge"
    assert A.attention_keybias.__module__ == "gpa_vggt_b200.merging.fused_attention"
else:
    assert A.token_merge_bipartite2d.__module__ == "merging.merge"
S, P = 4, 37 * 37 + 5
attn = A.Attention(1024, num_heads=16, qk_norm=True, rope=RotaryPositionEmbedding2D(frequency=100),
                   patch_width=37, patch_height=37, merge_ratio=0.98)
attn.merge_metric_dim = 128
if MODE == "frame":
    attn.frame_special, attn.num_special, attn.broadcast_pool = True, 5, 8
init_weights(attn, seed=0)
attn = attn.eval().cuda().to(torch.bfloat16)
x = torch.randn(1, S * P, 1024, generator=torch.Generator().manual_seed(0)).cuda().bfloat16()
pos = PositionGetter()(S, 37, 37, device="cuda") + 1
pos = torch.cat([torch.zeros(S, 5, 2, dtype=pos.dtype, device="cuda"), pos], 1).reshape(1, S * P, 2)
with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
    out = attn(x, pos=pos, global_merging=None if MODE == "frame" else 9)
torch.save(out.float().cpu(), OUT)
'''


def _run(shim, mode, out):
    r = subprocess.run([sys.executable, "-c", SCRIPT, str(ROOT), str(REF), "1" if shim else "0", mode,
                        str(out)], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    return torch.load(out)


@pytest.mark.parametrize("mode", ["merged", "frame"])
def test_reference_attention_module_runs_on_the_dropin(tmp_path, mode):
    ours = _run(True, mode, tmp_path / "ours.pt")
    theirs = _run(False, mode, tmp_path / "theirs.pt")
    err = float((ours.double() - theirs.double()).norm() / theirs.double().norm())
    print(f"{mode}: the reference's Attention on the drop-in vs on its own path: rel-L2 {err:.2e}")
    assert err < 2e-2
