"""Parity of the sm_100a kernels with the CPU oracle, on identical inputs.

Integer/index work is compared bit-exactly (similarity argmax: except rows whose
exact top-2 gap is below 1e-6, accumulation-order near-ties).  Floating point:
merged K/V within fp32 rounding (fp32) or 1 bf16 ulp (bf16); attention output
rel-L2 < 1e-2 and max |err| < 3e-2 against the float64 oracle (bf16 P and
output), LSE within 2e-3.
"""
import pytest
import torch

from oracle import gpa_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


def rel_l2(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from gpa_vggt_b200 import build, _lib
    build.build()
    _lib.load()
    torch.manual_seed(0)


def _unit_rows(n, d, gen):
    x = torch.randn(n, d, generator=gen)
    return (x / x.norm(dim=1, keepdim=True)).bfloat16()


# ---------------------------------------------------------------- similarity
@pytest.mark.parametrize("m,n,d,batch", [(1000, 777, 128, 1), (513, 300, 64, 2), (260, 1025, 256, 1),
                                         (300, 129, 192, 1), (5, 3, 128, 1)])
def test_sim_argmax_matches_oracle(m, n, d, batch):
    from gpa_vggt_b200 import kernels
    g = torch.Generator().manual_seed(m * 7 + n)
    a = torch.stack([_unit_rows(m, d, g) for _ in range(batch)])
    b = torch.stack([_unit_rows(n, d, g) for _ in range(batch)])
    nm, ni = kernels.sim_argmax(a.to(DEV), b.to(DEV))
    torch.cuda.synchronize()
    for bi in range(batch):
        rm, ri, gap = O.sim_argmax(a[bi], b[bi])
        bad = (ni[bi].cpu().long() != ri) & (gap >= 1e-6)
        assert int(bad.sum()) == 0, f"{int(bad.sum())} argmax mismatches outside near-ties"
        assert float((nm[bi].cpu().double() - rm).abs().max()) < 1e-5


def test_sim_argmax_ties_take_first_index():
    from gpa_vggt_b200 import kernels
    g = torch.Generator().manual_seed(1)
    b = _unit_rows(600, 128, g)
    b[300] = b[17]           # exact duplicate dst rows: the lower index wins
    b[590] = b[17]
    a = b[[17, 300, 590, 5]].clone()
    nm, ni = kernels.sim_argmax(a[None].to(DEV), b[None].to(DEV))
    assert ni[0].tolist()[:3] == [17, 17, 17]


# ---------------------------------------------------------------- roles
@pytest.mark.parametrize("S,w,h,ns", [(4, 37, 37, 5), (10, 37, 37, 5), (3, 9, 9, 5), (1, 8, 8, 5),
                                      (5, 10, 7, 3)])
def test_merge_roles_match_oracle(S, w, h, ns):
    from gpa_vggt_b200 import kernels
    g = torch.Generator().manual_seed(S)
    rand = torch.randint(4, size=(max(S - 1, 0), h // 2, w // 2), generator=g)
    mask = O.dst_mask(S, w, h, 2, 2, ns, rand)
    dst, src = O.split_positions(mask)
    dpos, spos, slot = kernels.merge_roles(rand.to(DEV) if S > 1 else None, S, w, h, 2, 2, ns,
                                           False, DEV)
    assert dpos.cpu().long().tolist() == dst.tolist()
    assert spos.cpu().long().tolist() == src.tolist()
    sl = slot.cpu().long()
    assert sl[dst].tolist() == list(range(dst.numel()))
    assert (-sl[src] - 1).tolist() == list(range(src.numel()))


def test_merge_roles_no_rand():
    from gpa_vggt_b200 import kernels
    mask = O.dst_mask(4, 9, 9, 2, 2, 5, None, no_rand=True)
    dst, src = O.split_positions(mask)
    dpos, spos, _ = kernels.merge_roles(None, 4, 9, 9, 2, 2, 5, True, DEV)
    assert dpos.cpu().long().tolist() == dst.tolist()
    assert spos.cpu().long().tolist() == src.tolist()


# ---------------------------------------------------------------- metric split
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_metric_split_matches_oracle(dtype):
    from gpa_vggt_b200 import kernels
    g = torch.Generator().manual_seed(2)
    metric = torch.randn(2000, 128, generator=g).to(dtype)
    perm = torch.randperm(2000, generator=g)
    src, dst = perm[:1500].sort().values, perm[1500:].sort().values
    a, b = kernels.metric_split(metric.to(DEV), src.int().to(DEV), dst.int().to(DEV))
    ref = O.normalize_rows(metric)
    for got, pos in ((a, src), (b, dst)):
        d = (got.cpu().float() - ref[pos]).abs()
        ulp = ref[pos].abs() * 2 ** -7 + 1e-30
        assert bool((d <= ulp).all())                    # at most one bf16 ulp
        assert float((d > 0).float().mean()) < 1e-3       # and almost always exact


# ---------------------------------------------------------------- merge plan
@pytest.mark.parametrize("ns,nd,ratio,hub", [(3000, 1200, 1.0, 10), (3000, 1200, 0.5, 10),
                                             (3000, 1200, 0.01, 10), (50000, 9000, 0.3, 10),
                                             (10, 4, 0.0, 10), (1000, 1, 0.7, 10),
                                             (207955, 66845, 1.0, 2), (207955, 66845, 0.3, 2)])
def test_merge_plan_matches_oracle(ns, nd, ratio, hub):
    """Every group's members in ascending src ordinal, also for a hub group
    holding 1/hub of all src (half of the S=200 src rows in the last cases)."""
    from gpa_vggt_b200 import kernels
    g = torch.Generator().manual_seed(ns + nd)
    node_max = (torch.randint(0, 50, (ns,), generator=g).float() / 50)  # many ties
    node_idx = torch.randint(0, nd, (ns,), generator=g)
    node_idx[: ns // hub] = min(3, nd - 1)                                # a hub group
    r = int(ns * ratio)
    dst_pos = torch.arange(nd, dtype=torch.int32)
    src_pos = torch.arange(nd, nd + ns, dtype=torch.int32)
    plan = kernels.merge_plan(node_max.to(DEV), node_idx.int().to(DEV), r, dst_pos.to(DEV),
                              src_pos.to(DEV))
    ref = O.merge_plan(node_max.double(), node_idx, r, nd)
    assert plan.unm_src.cpu().long().tolist() == ref.unm_src.tolist()
    assert plan.counts.cpu().double().tolist() == ref.counts.tolist()
    merged = torch.nonzero(ref.merged).reshape(-1)
    order = torch.sort(node_idx[merged], stable=True).indices
    assert plan.seg_src.cpu().long().tolist() == merged[order].tolist()
    starts = torch.zeros(nd + 1, dtype=torch.long)
    starts[1:] = torch.cumsum(torch.bincount(node_idx[merged], minlength=nd), 0)
    assert plan.seg_start.cpu().long().tolist() == starts.tolist()


# ---------------------------------------------------------------- scatter-mean
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("ratio,hub", [(1.0, False), (0.3, False), (1.0, True)])
def test_merge_kv_matches_oracle(dtype, ratio, hub):
    """hub: one dst receives 300 members (staged in several row batches)."""
    from gpa_vggt_b200 import kernels
    g = torch.Generator().manual_seed(5)
    S, w, h, ns_, H, D = 4, 37, 37, 5, 16, 64
    P = w * h + ns_
    N = S * P
    rand = torch.randint(4, size=(S - 1, h // 2, w // 2), generator=g)
    mask = O.dst_mask(S, w, h, 2, 2, ns_, rand)
    dst, src = O.split_positions(mask)
    node_max = torch.rand(src.numel(), generator=g)
    node_idx = torch.randint(0, dst.numel(), (src.numel(),), generator=g)
    if hub:
        node_idx[::10] = 7
    r = int(N * ratio)
    t = torch.randn(H, N, D, generator=g).to(dtype)
    plan = kernels.merge_plan(node_max.to(DEV), node_idx.int().to(DEV), r, dst.int().to(DEV),
                              src.int().to(DEV))
    got = kernels.merge_kv(t.to(DEV), plan).cpu()
    ref_plan = O.merge_plan(node_max.double(), node_idx, r, dst.numel())
    ref = O.merge_heads(t, ref_plan, dst, src)
    if dtype == torch.float32:
        torch.testing.assert_close(got.double(), ref, atol=1e-6, rtol=1e-6)
    else:
        d = (got.double() - ref).abs()
        assert bool((d <= ref.abs() * 2 ** -8 + 1e-6).all())
    # token-major [N, H, D] input/output layout through strides
    tm = t.transpose(0, 1).contiguous().to(DEV)
    out = torch.empty(plan.n_out, H, D, device=DEV, dtype=dtype)
    kernels.merge_kv(tm.transpose(0, 1), plan, out=out.transpose(0, 1))
    assert torch.equal(out.transpose(0, 1).cpu(), got)


# ---------------------------------------------------------------- attention
ATTN_CASES = [
    # B, H, M, N, bias, lse
    (1, 2, 300, 200, True, True),
    (1, 4, 1000, 777, True, False),
    (2, 3, 129, 128, False, True),
    (1, 1, 256, 4000, True, True),
    (1, 16, 2048, 1500, True, False),
    (1, 2, 17, 5, True, True),
    # short keys: persistent CTAs, each walking two or three work items
    (40, 4, 260, 520, True, True),
]


@pytest.mark.parametrize("B,H,M,N,with_bias,lse", ATTN_CASES)
def test_attention_matches_oracle(B, H, M, N, with_bias, lse):
    from gpa_vggt_b200 import kernels
    g = torch.Generator().manual_seed(M + N)
    q = torch.randn(B, H, M, 64, generator=g).bfloat16()
    k = torch.randn(B, H, N, 64, generator=g).bfloat16()
    v = torch.randn(B, H, N, 64, generator=g).bfloat16()
    bias = (1 + torch.poisson(torch.ones(B, H, N), generator=g)).log() if with_bias else None
    scale = 64 ** -0.5
    res = kernels.attention(q.to(DEV), k.to(DEV), v.to(DEV), None if bias is None else bias.to(DEV),
                            scale, return_lse=lse)
    o = res[0] if lse else res
    ro = O.attention_keybias(q, k, v, None if bias is None else bias[:, :, None, :], scale,
                             return_lse=lse)
    ref = ro[0] if lse else ro
    assert rel_l2(o, ref) < 1e-2
    assert float((o.cpu().double() - ref).abs().max()) < 3e-2
    if lse:
        assert float((res[1].cpu().double() - ro[1]).abs().max()) < 2e-3


def test_attention_strided_views_and_large_logits():
    """q/k/v as views into a [N, 3, H, D] qkv buffer; logits up to ~60 (lazy
    rescaling must stay exact)."""
    from gpa_vggt_b200 import kernels
    g = torch.Generator().manual_seed(9)
    N, H = 700, 4
    qkv = (torch.randn(N, 3, H, 64, generator=g) * 3).bfloat16()
    q = qkv[:, 0].permute(1, 0, 2)[None]
    k = qkv[:, 1].permute(1, 0, 2)[None]
    v = qkv[:, 2].permute(1, 0, 2)[None]
    qkv_d = qkv.to(DEV)
    o = kernels.attention(qkv_d[:, 0].permute(1, 0, 2)[None], qkv_d[:, 1].permute(1, 0, 2)[None],
                          qkv_d[:, 2].permute(1, 0, 2)[None], None, 64 ** -0.5)
    ref = O.attention_keybias(q, k, v, None, 64 ** -0.5)
    assert rel_l2(o, ref) < 1e-2


@pytest.mark.parametrize("ramp", [2.0, 40.0, 120.0])
def test_attention_running_max_moves_along_keys(ramp):
    """A bias that rises along the keys moves the row max on many key tiles
    (ramp 120: about 15 log2 units per 128-key tile, past the lazy-rescale
    threshold every tile); in head 1 the first 200 keys have -inf bias, so
    the max jumps from the masked value on the second tile.  Tiles whose
    exponentials were taken against a stale max must be redone, and O
    rescaled, without changing the result."""
    from gpa_vggt_b200 import kernels
    g = torch.Generator().manual_seed(int(ramp))
    B, H, M, N = 1, 2, 300, 1500
    q = torch.randn(B, H, M, 64, generator=g).bfloat16()
    k = torch.randn(B, H, N, 64, generator=g).bfloat16()
    v = torch.randn(B, H, N, 64, generator=g).bfloat16()
    bias = torch.linspace(0.0, ramp, N).expand(B, H, N).clone()
    bias[:, 1, :200] = float("-inf")
    scale = 64 ** -0.5
    o, lse = kernels.attention(q.to(DEV), k.to(DEV), v.to(DEV), bias.to(DEV), scale, return_lse=True)
    ro, rlse = O.attention_keybias(q, k, v, bias[:, :, None, :], scale, return_lse=True)
    assert torch.isfinite(o.float()).all()
    assert rel_l2(o, ro) < 1e-2
    assert float((lse.cpu().double() - rlse).abs().max()) < 2e-3


def test_attention_matches_reference_golden(golden):
    """Against the reference Triton kernel's own output (interpreter run)."""
    from gpa_vggt_b200.merging.fused_attention import attention_keybias
    gd = golden("attn_small.pt")
    o, lse = attention_keybias(gd["q"].to(DEV), gd["k"].to(DEV), gd["v"].to(DEV),
                               gd["bias"].to(DEV), gd["scale"], return_lse=True)
    assert rel_l2(o, gd["o_bias"]) < 1e-2
    assert float((lse.cpu() - gd["lse_bias"]).abs().max()) < 2e-3


# ---------------------------------------------------------------- frame pool / combine
def test_frame_pool_matches_oracle():
    from gpa_vggt_b200 import kernels
    g = torch.Generator().manual_seed(11)
    H, S, ph, pw, ns, kp = 4, 3, 37, 37, 5, 8
    P = ph * pw + ns
    k = torch.randn(H, S * P, 64, generator=g).bfloat16()
    v = torch.randn(H, S * P, 64, generator=g).bfloat16()
    pk, pv, size = kernels.frame_pool(k.to(DEV), v.to(DEV), S, ph, pw, ns, kp)
    rk, rv, rsize, _ = O.frame_pool(k.reshape(H, S, P, 64), v.reshape(H, S, P, 64), ph, pw, ns, kp)
    assert torch.equal(size.cpu(), rsize)
    torch.testing.assert_close(pk.cpu().float(), rk.bfloat16().float(), atol=0, rtol=0)
    torch.testing.assert_close(pv.cpu().float(), rv.bfloat16().float(), atol=0, rtol=0)


def test_frame_pool_matches_reference_golden(golden):
    from gpa_vggt_b200 import kernels
    gd = golden("frame_small.pt")
    H, N, D = gd["k"].shape
    pk, pv, size = kernels.frame_pool(gd["k"].bfloat16().to(DEV), gd["v"].bfloat16().to(DEV),
                                      gd["S"], gd["h"], gd["w"], gd["num_special"], gd["kp"])
    torch.testing.assert_close(pk.cpu().float(), gd["pooled_k"].bfloat16().float(), atol=0, rtol=0)
    torch.testing.assert_close(size.cpu().log(), gd["pooled_log_size"], atol=1e-6, rtol=0)


def test_lse_combine_matches_oracle():
    from gpa_vggt_b200 import kernels
    g = torch.Generator().manual_seed(12)
    H, S, P = 3, 4, 50
    oa = torch.randn(S, H, P, 64, generator=g).bfloat16()      # frame-major like q_f
    ob = torch.randn(H, S * P, 64, generator=g).bfloat16()
    la = torch.randn(S, H, P, generator=g) * 4
    lb = torch.randn(H, S * P, generator=g) * 4
    got = kernels.lse_combine(oa.to(DEV).permute(1, 0, 2, 3), la.to(DEV).permute(1, 0, 2),
                              ob.to(DEV).reshape(H, S, P, 64), lb.to(DEV).reshape(H, S, P))
    ref = O.lse_combine(oa.permute(1, 0, 2, 3), la.permute(1, 0, 2).double(),
                        ob.reshape(H, S, P, 64), lb.reshape(H, S, P).double())
    assert float((got.cpu().double() - ref).abs().max()) < 2e-2
    assert rel_l2(got, ref) < 5e-3


# ---------------------------------------------------------------- no fallback
def test_cpu_tensors_raise():
    from gpa_vggt_b200 import kernels
    with pytest.raises(ValueError):
        kernels.attention(torch.zeros(1, 1, 4, 64, dtype=torch.bfloat16),
                          torch.zeros(1, 1, 4, 64, dtype=torch.bfloat16),
                          torch.zeros(1, 1, 4, 64, dtype=torch.bfloat16), None, 0.125)
