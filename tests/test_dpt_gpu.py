"""DPT head resize kernel (gpa_upsample_bilinear_bf16) against the torch ops it
replaces (same inputs): F.interpolate(bilinear, align_corners=True) in fp32,
the optional fp32 positional add, and the bf16 cast of the next autocast
convolution's input.  Bound: at most one bf16 ulp, and almost always exact
(torch's and this kernel's fp32 weight arithmetic may round differently in the
last bit)."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _build():
    from gpa_vggt_b200 import build
    build.build()


def _ulp_ok(got, ref, scale, frac=1e-2):
    """|got - ref| <= one bf16 ulp of the larger magnitude plus 2^-20 * scale
    (the inputs' magnitude): the two fp32 weight computations may differ in the
    last bit, which can move a value across a bf16 rounding boundary, and where
    the interpolation cancels to near zero an absolute fp32 difference of a few
    ulps of the inputs is large next to the result.  Almost always exact."""
    g, r = got.float(), ref.float()
    d = (g - r).abs()
    e = torch.frexp(torch.maximum(g.abs(), r.abs())).exponent
    bound = torch.ldexp(torch.ones_like(d), e - 8) + 2.0 ** -20 * float(scale)
    assert bool((d <= bound).all()), float((d / bound).max())
    assert float((d > 0).float().mean()) < frac


def _channels_last(n, c, h, w, dtype, gen):
    return torch.randn(n, c, h, w, device="cuda", generator=gen).to(dtype).contiguous(
        memory_format=torch.channels_last)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape,size", [((2, 64, 30, 30), (61, 61)), ((3, 256, 37, 37), (74, 74)),
                                        ((1, 128, 74, 74), (518, 518)), ((2, 16, 1, 5), (1, 9))])
def test_resize_matches_interpolate(dtype, shape, size):
    from gpa_vggt_b200 import kernels
    g = torch.Generator(device="cuda").manual_seed(shape[1] + size[0])
    x = _channels_last(*shape, dtype, g)
    got = kernels.upsample_bilinear_bf16(x, size)
    ref = F.interpolate(x.float(), size=size, mode="bilinear", align_corners=True).bfloat16()
    assert got.shape == ref.shape and got.stride(1) == 1
    _ulp_ok(got, ref, x.float().abs().max())


@pytest.mark.parametrize("round_first", [False, True])
def test_resize_with_positional_add(round_first):
    from gpa_vggt_b200 import kernels
    g = torch.Generator(device="cuda").manual_seed(7)
    x = _channels_last(2, 128, 40, 40, torch.bfloat16, g)
    size = (81, 79)
    pe = torch.randn(size[0], size[1], 128, device="cuda", generator=g).permute(2, 0, 1)[None]
    got = kernels.upsample_bilinear_bf16(x, size, add=pe, round_first=round_first)
    r = F.interpolate(x.float(), size=size, mode="bilinear", align_corners=True)
    if round_first:
        r = r.bfloat16().float()
    _ulp_ok(got, (r + pe).bfloat16(), x.float().abs().max() + pe.abs().max())


def test_dpt_fusion_block_matches_unfused_path():
    """A refinement block under bf16 autocast: the fused resize path equals the
    torch resize path feeding the same convolution (up to the resize's last-bit
    rounding)."""
    from gpa_vggt_b200.vggt import heads
    g = torch.Generator(device="cuda").manual_seed(3)
    blk = heads.FeatureFusionBlock(64).cuda().bfloat16().to(memory_format=torch.channels_last)
    x0 = _channels_last(2, 64, 20, 20, torch.bfloat16, g)
    x1 = _channels_last(2, 64, 20, 20, torch.bfloat16, g)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        fused = blk(x0, x1, size=(37, 37))
        assert heads._fused_resize_ok(blk.resConfUnit2(x0 + blk.resConfUnit1(x1)))
        orig = heads._fused_resize_ok
        heads._fused_resize_ok = lambda t: False
        try:
            plain = blk(x0, x1, size=(37, 37))
        finally:
            heads._fused_resize_ok = orig
    rel = float((fused.float() - plain.float()).norm() / plain.float().norm())
    assert rel < 2e-3


@pytest.mark.parametrize("what", ["rcu", "fusion", "head"])
def test_fused_conv_epilogue_matches_torch_ops(what):
    """Convolutions without their bias, then one pass for bias + ReLU +
    residual (gpa_bias_act_bf16), against the module's own torch ops: the
    roundings are torch's (a bf16 bias add after the convolution, a bf16
    residual add), so the outputs are equal."""
    from gpa_vggt_b200.vggt import heads, init_weights
    g = torch.Generator(device="cuda").manual_seed(11)
    if what == "rcu":
        mod = heads.ResidualConvUnit(64)
        args = (_channels_last(2, 64, 24, 24, torch.bfloat16, g),)
        kw = {}
    elif what == "fusion":
        mod = heads.FeatureFusionBlock(64)
        args = (_channels_last(2, 64, 20, 20, torch.bfloat16, g), _channels_last(2, 64, 20, 20, torch.bfloat16, g))
        kw = {"size": (37, 37)}
    else:
        mod = heads.DPTHead(dim_in=256, features=64, out_channels=(32, 64, 128, 128))
        taps = [torch.randn(1, 2, 5 + 16 * 16, 256, device="cuda", generator=g).bfloat16() for _ in range(4)]
        args = (taps,)
        kw = {"images": torch.rand(1, 2, 3, 224, 224, device="cuda", generator=g), "patch_start_idx": 5}
    init_weights(mod, seed=4)
    mod = mod.cuda().bfloat16().to(memory_format=torch.channels_last)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        fused = mod(*args, **kw)
        heads.FUSED_CONV_EPILOGUE = False
        try:
            plain = mod(*args, **kw)
        finally:
            heads.FUSED_CONV_EPILOGUE = True
    outs = fused if isinstance(fused, tuple) else (fused,)
    refs = plain if isinstance(plain, tuple) else (plain,)
    for a, b in zip(outs, refs):
        d = (a.float() - b.float()).abs()
        print(f"{what}: max |d| {float(d.max()):.3e}, {float((d > 0).float().mean()):.2e} of elements differ")
        assert torch.equal(a, b)
