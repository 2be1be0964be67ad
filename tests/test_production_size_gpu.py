"""Parity at the production size: one merged block at S = 200 frames
(274,800 tokens; 207,955 src and 66,845 dst at 37x37 patches).  The oracle
cannot run the whole block in seconds, so each kernel is checked on a sample of
rows against the oracle, and the rest through size-independent properties:

* similarity argmax: 4,096 sampled src rows against all 66,845 dst rows --
  indices bit-exact except rows whose exact top-2 gap is below 1e-6, node_max
  within 1e-5 (oracle, float64 on the CPU);
* merge plan, in full: counts = 1 + the number of src matched to each dst; at
  ratio 0.2 the merged set is the top r of node_max with ties to the lower src
  ordinal (a stable sort); group members ascending;
* scatter-mean, in full: K (fp32) within 1e-6 relative and V (bf16) within one
  bf16 ulp of a float64 index_add mean;
* biased attention at the merged shape (274,800 queries x 66,845 keys x 16
  heads): 256 sampled query rows against the float64 oracle, rel-L2 < 1e-2.
"""
import pytest
import torch

from oracle import gpa_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
S, P_TOK = 200, 37 * 37 + 5
N = S * P_TOK


@pytest.fixture(scope="module")
def block():
    """Roles, metric, match and plans of one S=200 merged block (bf16 metric,
    as the projected norm1 output under autocast)."""
    from gpa_vggt_b200 import build, _lib, kernels
    from gpa_vggt_b200.merging.merge import draw_dst_choice, projection_basis
    build.build()
    _lib.load()
    g = torch.Generator(device=DEV)
    g.manual_seed(200)
    x = torch.randn(N, 1024, device=DEV, generator=g).bfloat16()
    g.manual_seed(33)
    rand_idx = draw_dst_choice(S, 37, 37, 2, 2, DEV, g)
    dst_pos, src_pos, _ = kernels.merge_roles(rand_idx, S, 37, 37, 2, 2, 5, False, DEV)
    metric = x @ projection_basis(1024, 128, DEV, torch.bfloat16)
    a, b = kernels.metric_split(metric, src_pos, dst_pos)
    nm, ni = kernels.sim_argmax(a[None], b[None])
    return dict(dst_pos=dst_pos, src_pos=src_pos, a=a, b=b, nm=nm[0], ni=ni[0])


def test_sizes_are_the_s200_split(block):
    assert block["src_pos"].numel() == 207955 and block["dst_pos"].numel() == 66845


def test_similarity_sampled_rows_match_oracle(block):
    g = torch.Generator().manual_seed(0)
    rows = torch.randperm(block["a"].shape[0], generator=g)[:4096].sort().values
    rm, ri, gap = O.sim_argmax(block["a"][rows.to(DEV)].cpu(), block["b"].cpu())
    ni, nm = block["ni"].cpu()[rows].long(), block["nm"].cpu()[rows]
    bad = (ni != ri) & (gap >= 1e-6)
    print(f"S=200 similarity: {int((ni != ri).sum())} of 4096 sampled rows differ, "
          f"{int(bad.sum())} outside near-ties")
    assert int(bad.sum()) == 0
    assert float((nm.double() - rm).abs().max()) < 1e-5


@pytest.mark.parametrize("ratio", [0.98, 0.2])
def test_plan_properties_in_full(block, ratio):
    from gpa_vggt_b200 import kernels
    ns, nd = block["src_pos"].numel(), block["dst_pos"].numel()
    r = min(int(N * ratio), ns)
    plan = kernels.merge_plan(block["nm"], block["ni"], r, block["dst_pos"], block["src_pos"])
    order = torch.sort(-block["nm"], stable=True).indices       # descending, ties to lower ordinal
    merged = torch.zeros(ns, dtype=torch.bool, device=DEV)
    merged[order[:r]] = True
    unm = (~merged).nonzero().reshape(-1)
    assert torch.equal(plan.unm_src.long(), unm)
    ni = block["ni"].long()
    cnt = torch.bincount(ni[merged], minlength=nd).float() + 1
    assert torch.equal(plan.counts[plan.unm_len:], cnt)
    assert bool((plan.counts[:plan.unm_len] == 1).all())
    mi = merged.nonzero().reshape(-1)
    want = mi[torch.sort(ni[mi], stable=True).indices]
    assert torch.equal(plan.seg_src.long(), want)
    block[f"plan_{ratio}"] = plan


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_scatter_mean_in_full(block, dtype):
    from gpa_vggt_b200 import kernels
    plan = block.get("plan_0.2")
    if plan is None:
        plan = kernels.merge_plan(block["nm"], block["ni"], int(N * 0.2), block["dst_pos"],
                                  block["src_pos"])
    g = torch.Generator(device=DEV)
    g.manual_seed(9)
    t = torch.randn(16, N, 64, device=DEV, generator=g).to(dtype)
    out = kernels.merge_kv(t, plan)
    td = t.double()
    src_pos, dst_pos = plan.src_pos.long(), plan.dst_pos.long()
    want = torch.empty(16, plan.n_out, 64, device=DEV, dtype=torch.float64)
    want[:, :plan.unm_len] = td[:, src_pos[plan.unm_src.long()]]
    acc = td[:, dst_pos].clone()
    seg = plan.seg_start.long()
    dst_of = torch.repeat_interleave(torch.arange(plan.num_dst, device=DEV), seg[1:] - seg[:-1])
    acc.index_add_(1, dst_of, td[:, src_pos[plan.seg_src.long()]])
    want[:, plan.unm_len:] = acc / plan.counts[plan.unm_len:].double()[None, :, None]
    d = (out.double() - want).abs()
    if dtype == torch.float32:     # fp32 sums of up to a few dozen N(0,1) rows
        assert bool((d <= 1e-6 * want.abs() + 2e-6).all())
    else:
        assert bool((d <= want.abs() * 2 ** -8 + 1e-30).all())


def test_attention_sampled_rows_at_merged_shape(block):
    from gpa_vggt_b200 import kernels
    plan = kernels.merge_plan(block["nm"], block["ni"], int(N * 0.98), block["dst_pos"],
                              block["src_pos"])
    nk = plan.n_out
    assert nk == 66845
    g = torch.Generator(device=DEV)
    g.manual_seed(10)
    q = torch.randn(1, 16, N, 64, device=DEV, generator=g).bfloat16()
    k = torch.randn(1, 16, nk, 64, device=DEV, generator=g).bfloat16()
    v = torch.randn(1, 16, nk, 64, device=DEV, generator=g).bfloat16()
    bias = plan.counts.log().bfloat16().float()
    o = kernels.attention(q, k, v, bias[None, None], 64 ** -0.5)
    rows = torch.randperm(N, generator=torch.Generator().manual_seed(1))[:256].sort().values
    errs = []
    for h in range(16):
        ref = O.attention_keybias(q[0, h, rows.to(DEV)].cpu(), k[0, h].cpu(), v[0, h].cpu(),
                                  bias.cpu()[None, :], 64 ** -0.5)
        errs.append(((o[0, h, rows.to(DEV)].cpu().double() - ref).norm() / ref.norm()).item())
    print(f"S=200 merged-shape attention, 256 rows x 16 heads: max rel-L2 {max(errs):.2e}")
    assert max(errs) < 1e-2
