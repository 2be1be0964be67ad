"""Fused normalisation kernels against the torch ops they replace (same inputs):
bf16 LayerNorm vs F.layer_norm in fp32 rounded to bf16; qk-LayerNorm + 2D RoPE
vs the reference-shaped torch path (LayerNorm then RotaryPositionEmbedding2D in
fp32).  Bound: at most one bf16 ulp, and almost always exact."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _build():
    from gpa_vggt_b200 import build
    build.build()


def _ulp_ok(got, ref, frac=2e-2):
    d = (got.float() - ref.float()).abs()
    ulp = ref.float().abs() * 2 ** -7 + 1e-6
    assert bool((d <= ulp).all()), float((d / ulp).max())
    assert float((d > 0).float().mean()) < frac


@pytest.mark.parametrize("rows,cols,pdt", [(3000, 1024, torch.bfloat16), (257, 2048, torch.float32),
                                           (5, 256, torch.bfloat16)])
def test_layernorm_matches_torch(rows, cols, pdt):
    from gpa_vggt_b200 import kernels
    g = torch.Generator(device="cuda").manual_seed(rows)
    x = (torch.randn(rows, cols, device="cuda", generator=g) * 3 + 1).bfloat16()
    w = (1 + 0.1 * torch.randn(cols, device="cuda", generator=g)).to(pdt)
    b = (0.1 * torch.randn(cols, device="cuda", generator=g)).to(pdt)
    got = kernels.layernorm(x, w, b, 1e-6)
    ref = F.layer_norm(x.float(), (cols,), w.float(), b.float(), 1e-6).bfloat16()
    _ulp_ok(got, ref)


@pytest.mark.parametrize("with_rope", [True, False])
def test_qk_norm_rope_matches_torch_path(with_rope):
    from gpa_vggt_b200 import kernels
    from gpa_vggt_b200.vggt.layers import RotaryPositionEmbedding2D, PositionGetter
    g = torch.Generator(device="cuda").manual_seed(3)
    S, P, H = 3, 37 * 37 + 5, 16
    T = S * P
    qkv = torch.randn(T, 3, H, 64, device="cuda", generator=g).bfloat16()
    qn = torch.nn.LayerNorm(64).cuda()
    kn = torch.nn.LayerNorm(64).cuda()
    with torch.no_grad():
        for m in (qn, kn):
            m.weight.copy_(1 + 0.1 * torch.randn(64, device="cuda", generator=g))
            m.bias.copy_(0.1 * torch.randn(64, device="cuda", generator=g))
    qn, kn = qn.bfloat16(), kn.bfloat16()
    rope = RotaryPositionEmbedding2D(100)
    pos = PositionGetter()(S, 37, 37, "cuda") + 1
    pos = torch.cat([torch.zeros(S, 5, 2, device="cuda", dtype=pos.dtype), pos], 1).reshape(1, T, 2)
    # torch path: fp32 LayerNorm (autocast semantics) then rope in fp32
    qr = F.layer_norm(qkv[:, 0].float(), (64,), qn.weight.float(), qn.bias.float(), 1e-5)[None]
    kr = F.layer_norm(qkv[:, 1].float(), (64,), kn.weight.float(), kn.bias.float(), 1e-5)[None]
    if with_rope:
        qr, kr = rope(qr, pos), rope(kr, pos)
    v_before = qkv[:, 2].clone()
    cos, sin = rope.tables(32, "cuda")
    q, k, v = kernels.qk_norm_rope(qkv, qn, kn, pos if with_rope else None,
                                   cos if with_rope else None, sin if with_rope else None)
    _ulp_ok(q, qr[0].bfloat16())
    _ulp_ok(k, kr[0].bfloat16())
    assert torch.equal(v, v_before)


@pytest.mark.parametrize("shape", [(200, 1374, 1024), (1, 3001, 1024), (7, 64)])
def test_residual_scale_bitexact_with_torch(shape):
    """x + y * gamma (LayerScale residual) equals torch's two bf16 ops bit for
    bit, including a strided y (a column slice of a wider buffer)."""
    from gpa_vggt_b200 import kernels
    g = torch.Generator(device="cuda").manual_seed(shape[-1] + shape[0])
    x = (torch.randn(*shape, device="cuda", generator=g) * 4).bfloat16()
    y = (torch.randn(*shape, device="cuda", generator=g) * 50).bfloat16()
    gamma = (0.01 * torch.randn(shape[-1], device="cuda", generator=g)).bfloat16()
    assert torch.equal(kernels.residual_scale(x, y, gamma), x + y * gamma)
    wide = torch.randn(*shape[:-1], shape[-1] + 16, device="cuda", generator=g).bfloat16()
    ys = wide[..., 8:8 + shape[-1]]
    assert torch.equal(kernels.residual_scale(x, ys, gamma), x + ys * gamma)


def test_block_residual_uses_fused_kernel_and_matches():
    """Block.forward's residual path with LayerScale on CUDA bf16 gives the
    unfused expression's result exactly."""
    from gpa_vggt_b200.vggt.layers import LayerScale, _residual
    g = torch.Generator(device="cuda").manual_seed(3)
    ls = LayerScale(1024, init_values=0.01).cuda().bfloat16()
    x = torch.randn(2, 300, 1024, device="cuda", generator=g).bfloat16()
    y = torch.randn(2, 300, 1024, device="cuda", generator=g).bfloat16()
    assert torch.equal(_residual(x, ls, y), x + ls(y))


def test_gelu_matches_torch():
    """Exact-erf GELU of bf16 values equals torch's bf16 F.gelu (same fp32
    expression); at most a last-bit difference on a tiny fraction."""
    from gpa_vggt_b200 import kernels
    g = torch.Generator(device="cuda").manual_seed(4)
    x = (torch.randn(3001, 4096, device="cuda", generator=g) * 3).bfloat16()
    got, ref = kernels.gelu(x), F.gelu(x)
    _ulp_ok(got, ref, frac=1e-3)


def test_mlp_uses_fused_gelu_and_matches():
    from gpa_vggt_b200.vggt.layers import Mlp
    g = torch.Generator(device="cuda").manual_seed(5)
    mlp = Mlp(256, 1024).cuda().bfloat16()
    x = torch.randn(4, 77, 256, device="cuda", generator=g).bfloat16()
    with torch.no_grad():
        got = mlp(x)
        ref = mlp.fc2(F.gelu(mlp.fc1(x)))
    rel = float((got.float() - ref.float()).norm() / ref.float().norm())
    assert rel < 1e-3, rel
