"""The one-kernel matching metric (gpa_proj_norm_split, merging/merge.py:180-187):
bf16(x @ proj) -> fp32 norm and quotient -> bf16, routed to the src / dst rows.

* Against the unfused path (torch's bf16 GEMM, then gpa_metric_split) and the
  oracle (float64 accumulation of the bf16 operands, rounded to bf16, then the
  fp32 normalisation): within two bf16 ulps plus 1e-5 (a product that rounds
  to the other bf16 neighbour moves its element by one ulp before the
  division rounds again; fp32 sums carry an absolute error that dominates
  near-zero elements), and exact on more than 99% of the elements.
* Row counts that are not a multiple of the 128-row tile, and the S=200 size.
"""
import pytest
import torch

from oracle import gpa_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from gpa_vggt_b200 import build, _lib
    build.build()
    _lib.load()


def _case(S, seed):
    from gpa_vggt_b200 import kernels
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    N = S * (37 * 37 + 5)
    x = torch.randn(N, 1024, device=DEV, generator=g).bfloat16()
    proj = torch.randn(1024, 128, device=DEV, generator=g).bfloat16()
    g.manual_seed(33)
    rand = torch.randint(4, (S - 1, 18, 18), device=DEV, generator=g)
    dst, src, slot = kernels.merge_roles(rand, S, 37, 37, 2, 2, 5, False, DEV)
    return x, proj, dst, src, slot


def _check(got, want, what):
    got, want = got.float(), want.float()
    d = (got - want).abs()
    bad = d > want.abs() * 2 ** -6 + 1e-5          # two ulps, also across a binade edge
    frac = float((d > 0).float().mean())
    print(f"{what}: {frac:.2e} of the elements differ, max |d| {float(d.max()):.2e}")
    assert int(bad.sum()) == 0
    assert frac < 1e-2


@pytest.mark.parametrize("S", [4, 200])
def test_fused_metric_matches_unfused_path(S):
    from gpa_vggt_b200 import kernels
    x, proj, dst, src, slot = _case(S, S)
    a, b = kernels.proj_norm_split(x, proj.t().contiguous(), slot, src.numel(), dst.numel())
    a0, b0 = kernels.metric_split(x @ proj, src, dst)
    for got, want, what in ((a, a0, f"S={S} src"), (b, b0, f"S={S} dst")):
        _check(got, want, what)


def test_fused_metric_matches_oracle():
    from gpa_vggt_b200 import kernels
    x, proj, dst, src, slot = _case(4, 7)
    a, b = kernels.proj_norm_split(x, proj.t().contiguous(), slot, src.numel(), dst.numel())
    ref = O.normalize_rows(O.project_metric(x.cpu(), proj.cpu()))
    for got, pos, what in ((a, src, "oracle src"), (b, dst, "oracle dst")):
        _check(got.cpu(), ref[pos.cpu().long()], what)


def test_merge_plan_through_fused_metric_matches_unfused():
    """build_plan with a bf16 metric takes the fused kernel; its plan equals the
    unfused path's except on rows whose exact top-2 gap is below 1e-3 (a
    rounding flip in the metric moves such a row's argmax)."""
    from gpa_vggt_b200 import kernels
    from gpa_vggt_b200.merging import merge as M
    x, proj, dst, src, slot = _case(10, 3)
    g = torch.Generator(device=DEV)
    g.manual_seed(33)
    rand = M.draw_dst_choice(10, 37, 37, 2, 2, DEV, g)
    plan = M.build_plan(x, 37, 37, 2, 2, int(x.shape[0] * 0.98), rand_idx=rand, proj=proj,
                        metric_dim=128)
    a0, b0 = kernels.metric_split(x @ proj, plan.src_pos, plan.dst_pos)
    nm0, ni0 = kernels.sim_argmax(a0[None], b0[None])
    diff = (plan.node_idx.long() != ni0[0].long()).nonzero().reshape(-1)
    if diff.numel():
        s = a0[diff].double() @ b0.double().T
        t = s.topk(2, dim=1).values
        assert float((t[:, 0] - t[:, 1]).max()) < 1e-3
    assert diff.numel() <= 0.01 * plan.num_src
