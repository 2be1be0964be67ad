"""Generate the golden vectors in tests/golden/ from the reference itself.

Run in a container that has the reference checkout (noheat61/GPA-VGGT); the
path is required:

    GPA_REF=/path/to/GPA-VGGT python tests/golden/make_golden.py [what]

what: (none) the small kernel/merge/attention/frame/block fixtures;
      config1 (one merged block at BASELINE config 1: S=4, 37x37, dim 1024);
      model [S] / model_bf16 [S] (full forward, GPA; S=2 by default);
      vanilla [S] / vanilla_bf16 [S] (full forward, vanilla global attention).

What it runs, all on CPU:
  * merging/merge.py: token_merge_bipartite2d, with its matcher replaced by the
    reference's own Triton kernel _sim_argmax_kernel (merging/fused_similarity.py)
    executed by Triton's CPU interpreter, so the indices follow the GPU
    contract (fp32 accumulation, first index); the stock bf16-score CPU matcher
    (fast_similarity_chunks) is recorded too.
  * merging/fused_attention.py: _attn_keybias_kernel under the interpreter.
    numpy has no bf16, so the inputs are fp32 tensors holding bf16 values (the
    kernel's P stays fp32 there instead of bf16).
  * vggt/layers/attention.py: Attention._frame_special_attention (CPU path)
    and Attention.forward with global merging (CPU path: SDPA with the bias).

Outputs are small .pt files; nothing here runs at test time.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import torch  # noqa: E402

REF = os.environ.get("GPA_REF")
if not REF:
    sys.exit("make_golden.py: set GPA_REF to the reference checkout (noheat61/GPA-VGGT)")
OUT = Path(__file__).resolve().parent
sys.path.insert(0, REF)

import merging.merge as ref_merge  # noqa: E402
import merging.fused_similarity as ref_fs  # noqa: E402
import merging.fused_attention as ref_fa  # noqa: E402
from vggt.layers.attention import Attention  # noqa: E402
from vggt.layers.rope import RotaryPositionEmbedding2D, PositionGetter  # noqa: E402
import vggt.layers.attention as ref_attn_mod  # noqa: E402


def bf16v(t):
    return t.to(torch.bfloat16).float()


def interp_sim_argmax(a, b):
    """merging/fused_similarity.py:_sim_argmax_kernel under the interpreter."""
    a = bf16v(a).contiguous()
    b = bf16v(b).contiguous()
    B, M, D = a.shape
    N = b.shape[1]
    node_max = torch.empty(B, M, dtype=torch.float32)
    node_idx = torch.empty(B, M, dtype=torch.int32)
    BM = 64
    ref_fs._sim_argmax_kernel.fn[((M + BM - 1) // BM, B)](
        a, b, node_max, node_idx, M, N, D,
        a.stride(0), a.stride(1), a.stride(2), b.stride(0), b.stride(1), b.stride(2),
        node_max.stride(0), node_max.stride(1), node_idx.stride(0), node_idx.stride(1),
        BLOCK_M=BM, BLOCK_N=128, BLOCK_K=64)
    return node_max, node_idx.long()


def interp_attention(q, k, v, bias, scale, return_lse=True):
    """merging/fused_attention.py:_attn_keybias_kernel under the interpreter,
    prepared exactly as attention_keybias does (clamped K/V, padded log2 bias)."""
    B, H, M, D = q.shape
    N = k.shape[2]
    BH = B * H
    PAD = ref_fa._PAD
    Npad = (N + PAD - 1) // PAD * PAD
    qc = bf16v(q).reshape(BH, M, D).contiguous()
    kp = bf16v(k).reshape(BH, N, D).contiguous()
    vp = bf16v(v).reshape(BH, N, D).contiguous()
    bp = torch.full((BH, Npad), -1e9, dtype=torch.float32)
    bp[:, :N] = 0.0 if bias is None else bias.reshape(BH, N).float() * ref_fa.LOG2E
    o = torch.empty_like(qc)
    lse = torch.empty(BH, M, dtype=torch.float32)
    BM, BN = 64, 64
    ref_fa._attn_keybias_kernel.fn[((M + BM - 1) // BM, BH)](
        qc, kp, vp, bp, o, lse, M, N, Npad,
        qc.stride(0), qc.stride(1), kp.stride(0), kp.stride(1), vp.stride(0), vp.stride(1),
        bp.stride(0), o.stride(0), o.stride(1), lse.stride(0), scale * ref_fa.LOG2E,
        HEAD_DIM=D, BLOCK_M=BM, BLOCK_N=BN, RETURN_LSE=return_lse)
    return o.reshape(B, H, M, D), lse.reshape(B, H, M)


def closure_vars(fn):
    return {n: c.cell_contents for n, c in zip(fn.__code__.co_freevars, fn.__closure__)}


def run_merge(x, w, h, r, metric_dim, num_special, patched=True):
    captured = {}
    stock = ref_merge.fast_similarity_chunks

    def matcher(a, bT, chunk):
        nm, ni = interp_sim_argmax(a, bT.transpose(-1, -2))
        captured["node_max"], captured["node_idx"] = nm.clone(), ni.clone()
        return nm.to(a.dtype), ni

    def stock_capture(a, bT, chunk):
        nm, ni = stock(a, bT, chunk)
        captured["node_max"], captured["node_idx"] = nm.clone(), ni.clone()
        return nm, ni

    ref_merge.fast_similarity_chunks = matcher if patched else stock_capture
    sorts = []
    argsort = torch.Tensor.argsort

    def capture_argsort(self, *a, **k):
        out = argsort(self, *a, **k)
        sorts.append(out.clone())
        return out

    torch.Tensor.argsort = capture_argsort
    try:
        g = torch.Generator().manual_seed(33)
        m = ref_merge.token_merge_bipartite2d(x, w, h, 2, 2, r, False, g, metric_dim=metric_dim,
                                              num_special=num_special)
    finally:
        ref_merge.fast_similarity_chunks = stock
        torch.Tensor.argsort = argsort
    cv = closure_vars(m)
    num_dst = cv["num_dst"]
    captured["a_idx"] = sorts[0].reshape(-1)[num_dst:].clone()  # merge.py:165,168
    return m, cv, captured


def gen_merge():
    torch.manual_seed(0)
    S, w, h, ns, C, H, D = 4, 9, 9, 5, 256, 4, 64
    P = w * h + ns
    N = S * P
    x = torch.randn(1, N, C)
    k = torch.randn(1, H, N, D)
    v = bf16v(torch.randn(1, H, N, D))
    g = torch.Generator().manual_seed(33)
    rand_idx = torch.randint(4, size=(S - 1, h // 2, w // 2), generator=g)
    gp = torch.Generator().manual_seed(ref_merge.PROJ_SEED)
    proj = torch.randn(C, 128, dtype=torch.float32, generator=gp)
    cases = {}
    for name, ratio in (("r098", 0.98), ("r020", 0.2)):
        r = int(N * ratio)
        m, cv, cap = run_merge(x, w, h, r, 128, ns)
        cases[name] = dict(
            r=r,
            a_idx=cap["a_idx"],
            b_idx=cv["b_idx"].reshape(-1).clone(),
            unm_abs_idx=cv["unm_abs_idx"].reshape(-1).clone(),
            src_abs_idx=cv["src_abs_idx"].reshape(-1).clone(),
            dst_idx=cv["dst_idx"].reshape(-1).clone(),
            node_max=cap["node_max"].reshape(-1), node_idx=cap["node_idx"].reshape(-1),
            size=m.size.reshape(-1).clone(),
            k_merged=m.heads(k, "mean")[0].clone(),
            v_merged=m.heads(v, "mean")[0].clone(),
        )
        m2, cv2, cap2 = run_merge(x, w, h, r, 128, ns, patched=False)
        cases[name]["stock_a_idx"] = cap2["a_idx"]
        cases[name]["stock_b_idx"] = cv2["b_idx"].reshape(-1).clone()
        cases[name]["stock_node_max"] = cap2["node_max"].reshape(-1)
        cases[name]["stock_node_idx"] = cap2["node_idx"].reshape(-1)
    torch.save(dict(S=S, w=w, h=h, num_special=ns, C=C, x=x[0], k=k[0], v=v[0],
                    rand_idx=rand_idx, proj=proj, cases=cases), OUT / "merge_small.pt")


def gen_attention():
    torch.manual_seed(1)
    B, H, M, N, D = 1, 2, 300, 200, 64
    q = bf16v(torch.randn(B, H, M, D))
    k = bf16v(torch.randn(B, H, N, D))
    v = bf16v(torch.randn(B, H, N, D))
    cnt = 1 + torch.poisson(torch.ones(N))
    bias = bf16v(cnt.log()).reshape(1, 1, 1, N).expand(B, H, 1, N).contiguous()
    scale = D ** -0.5
    o_b, lse_b = interp_attention(q, k, v, bias, scale)
    o_n, lse_n = interp_attention(q, k, v, None, scale)
    sdpa = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=bias)
    torch.save(dict(q=q, k=k, v=v, bias=bias, scale=scale, o_bias=o_b, lse_bias=lse_b,
                    o_nobias=o_n, lse_nobias=lse_n, sdpa_bias=sdpa), OUT / "attn_small.pt")


def gen_frame():
    torch.manual_seed(2)
    S, w, h, ns, H, D, kp = 3, 9, 9, 5, 2, 64, 4
    P = w * h + ns
    N = S * P
    C = H * D
    attn = Attention(C, num_heads=H, qk_norm=True, patch_width=w, patch_height=h)
    attn.frame_special = True
    attn.num_special = ns
    attn.broadcast_pool = kp
    attn.eval()
    q = bf16v(torch.randn(1, H, N, D))
    k = bf16v(torch.randn(1, H, N, D))
    v = bf16v(torch.randn(1, H, N, D))
    cap = {}
    sdpa = torch.nn.functional.scaled_dot_product_attention

    def capture(qq, kk, vv, attn_mask=None, **kw):
        cap["k_f"], cap["v_f"], cap["mask"] = kk.clone(), vv.clone(), attn_mask.clone()
        return sdpa(qq, kk, vv, attn_mask=attn_mask, **kw)

    ref_attn_mod.F.scaled_dot_product_attention = capture
    try:
        out = attn._frame_special_attention(q, k, v, 1, N, C)
    finally:
        ref_attn_mod.F.scaled_dot_product_attention = sdpa
    npool = (-(-h // kp)) * (-(-w // kp))
    # frame 0's key list: own patches, S*ns specials, S*npool pooled summaries
    pooled_k = cap["k_f"][0, :, w * h + S * ns:].clone()
    pooled_v = cap["v_f"][0, :, w * h + S * ns:].clone()
    pooled_bias = cap["mask"][0, :, 0, w * h + S * ns:].clone()
    torch.save(dict(S=S, w=w, h=h, num_special=ns, kp=kp, q=q[0], k=k[0], v=v[0],
                    out=out[0].reshape(N, H, D).transpose(0, 1).clone(),
                    pooled_k=pooled_k, pooled_v=pooled_v, pooled_log_size=pooled_bias,
                    npool=npool), OUT / "frame_small.pt")


def gen_block():
    torch.manual_seed(3)
    S, w, h, ns, H, D = 4, 9, 9, 5, 4, 64
    C = H * D
    P = w * h + ns
    N = S * P
    rope = RotaryPositionEmbedding2D(frequency=100)
    attn = Attention(C, num_heads=H, qk_norm=True, rope=rope, patch_width=w, patch_height=h,
                     merge_ratio=0.98)
    attn.merge_metric_dim = 128
    attn.eval()
    x = torch.randn(1, N, C)
    pg = PositionGetter()
    pos = pg(S, h, w, device="cpu") + 1
    pos = torch.cat([torch.zeros(S, ns, 2, dtype=pos.dtype), pos], 1).reshape(1, N, 2)
    stock = ref_merge.fast_similarity_chunks

    def matcher(a, bT, chunk):
        nm, ni = interp_sim_argmax(a, bT.transpose(-1, -2))
        return nm.to(a.dtype), ni

    ref_merge.fast_similarity_chunks = matcher
    try:
        with torch.no_grad():
            out_merged = attn(x, pos=pos, global_merging=9)
            out_plain = attn(x, pos=pos, global_merging=None)
    finally:
        ref_merge.fast_similarity_chunks = stock
    g = torch.Generator().manual_seed(33)
    rand_idx = torch.randint(4, size=(S - 1, h // 2, w // 2), generator=g)
    gp = torch.Generator().manual_seed(ref_merge.PROJ_SEED)
    proj = torch.randn(C, 128, dtype=torch.float32, generator=gp)
    torch.save(dict(S=S, w=w, h=h, num_special=ns, heads=H, x=x[0], pos=pos[0],
                    state=attn.state_dict(), rand_idx=rand_idx, proj=proj,
                    out_merged=out_merged[0], out_plain=out_plain[0]), OUT / "block_small.pt")


def _ref_model(vanilla, bf16):
    sys.path.insert(0, str(OUT.parents[1]))
    from gpa_vggt_b200.vggt.model import init_weights
    from vggt.models.vggt import VGGT as RefVGGT
    torch.manual_seed(0)
    model = RefVGGT(merging=None, early_frame_split=0) if vanilla else RefVGGT()
    init_weights(model, seed=0)
    model = model.eval()
    if bf16:
        model = model.to(torch.bfloat16)
    model.update_patch_dimensions(37, 37)
    return model


def _store(out, S, depth_stride):
    """pose encoding in full; depth and confidence every depth_stride-th pixel
    in each direction (fp16), which keeps the S=10 fixture near 1 MB."""
    st = depth_stride
    return dict(pose_enc=out["pose_enc"].float().clone(),
                depth=out["depth"].float()[:, :, ::st, ::st].half().clone(),
                depth_conf=out["depth_conf"].float()[:, :, ::st, ::st].half().clone(),
                depth_stride=st)


def gen_model(S=2, vanilla=False, bf16=False):
    """Full VGGT forward on CPU with the weights of
    gpa_vggt_b200.vggt.init_weights(seed=0) (a function of parameter names and
    shapes only, so the GPU test rebuilds the same weights) on
    torch.rand(1, S, 3, 518, 518) frames (CPU generator seed 0).  GPA
    configuration, or vanilla global attention (merging=None,
    early_frame_split=0).  fp32, or with bf16 the model in bf16 under CPU
    autocast: the reference's own bf16 drift, which sets the GPU test's
    tolerance.  The matcher is the reference's Triton kernel under the
    interpreter (the GPU contract)."""
    model = _ref_model(vanilla, bf16)
    images = torch.rand(1, S, 3, 518, 518, generator=torch.Generator().manual_seed(0))
    stock = ref_merge.fast_similarity_chunks

    def matcher(a, bT, chunk):
        nm, ni = interp_sim_argmax(a.float(), bT.transpose(-1, -2).float())
        return nm.to(a.dtype), ni

    ref_merge.fast_similarity_chunks = matcher
    try:
        with torch.no_grad():
            if bf16:
                with torch.autocast("cpu", dtype=torch.bfloat16):
                    out = model(images.to(torch.bfloat16))
            else:
                out = model(images)
    finally:
        ref_merge.fast_similarity_chunks = stock
    g = torch.Generator().manual_seed(33)
    rand_idx = torch.randint(4, size=(S - 1, 18, 18), generator=g)
    gp = torch.Generator().manual_seed(ref_merge.PROJ_SEED)
    proj = torch.randn(1024, 128, dtype=torch.float32, generator=gp)
    rec = dict(S=S, image_seed=0, weight_seed=0, vanilla=vanilla, rand_idx=rand_idx, proj=proj)
    rec.update(_store(out, S, 1 if S <= 2 else 2))
    name = f"{'vanilla' if vanilla else 'model'}_s{S}{'_bf16' if bf16 else ''}.pt"
    torch.save(rec, OUT / name)
    print(name, (OUT / name).stat().st_size)


def gen_config1():
    """One GPA merged global block at BASELINE config 1: S=4 frames of
    1 + 4 + 37x37 tokens (N=5,496), dim 1024, 16 heads x 64, x ~ N(0,1) from a
    CPU generator seeded 0; the reference's Attention (qk-LayerNorm, 2-D RoPE
    at frequency 100) with init_weights(seed=0), merge ratio 0.98, metric dim
    128; its forward(x, pos, global_merging=9) on CPU in fp32, the matcher
    being the reference's Triton kernel under the interpreter.  Stored: the
    metric the matcher saw (bf16 values), the match, the merge map keyed by
    absolute position, and every 8th row of the block output (fp16), also of
    the same forward in bf16 under CPU autocast (the reference's bf16 drift)."""
    sys.path.insert(0, str(OUT.parents[1]))
    from gpa_vggt_b200.vggt.model import init_weights
    S, w, h, ns, C, H = 4, 37, 37, 5, 1024, 16
    P = w * h + ns
    N = S * P
    attn = Attention(C, num_heads=H, qk_norm=True, rope=RotaryPositionEmbedding2D(frequency=100),
                     patch_width=w, patch_height=h, merge_ratio=0.98)
    attn.merge_metric_dim = 128
    init_weights(attn, seed=0)
    attn.eval()
    x = torch.randn(1, N, C, generator=torch.Generator().manual_seed(0))
    pos = PositionGetter()(S, h, w, device="cpu") + 1
    pos = torch.cat([torch.zeros(S, ns, 2, dtype=pos.dtype), pos], 1).reshape(1, N, 2)
    cap = {}
    stock = ref_merge.fast_similarity_chunks

    def matcher(a, bT, chunk):
        cap["a"], cap["b"] = bf16v(a).clone(), bf16v(bT.transpose(-1, -2)).clone()
        nm, ni = interp_sim_argmax(a, bT.transpose(-1, -2))
        cap["node_max"], cap["node_idx"] = nm.clone(), ni.clone()
        return nm.to(a.dtype), ni

    ref_merge.fast_similarity_chunks = matcher
    sorts = []
    argsort = torch.Tensor.argsort

    def capture_argsort(self, *a, **k):
        out = argsort(self, *a, **k)
        sorts.append(out.clone())
        return out

    torch.Tensor.argsort = capture_argsort
    try:
        with torch.no_grad():
            out = attn(x, pos=pos, global_merging=9)
    finally:
        ref_merge.fast_similarity_chunks = stock
        torch.Tensor.argsort = argsort
    num_dst = cap["b"].shape[1]
    a_idx = sorts[0].reshape(-1)[num_dst:]          # src positions in the matcher's row order
    b_idx = sorts[0].reshape(-1)[:num_dst]          # dst positions in its column order
    dst_of_src = torch.full((N,), -1, dtype=torch.long)
    dst_of_src[a_idx] = b_idx[cap["node_idx"].reshape(-1)]
    g = torch.Generator().manual_seed(33)
    rand_idx = torch.randint(4, size=(S - 1, h // 2, w // 2), generator=g)
    gp = torch.Generator().manual_seed(ref_merge.PROJ_SEED)
    proj = torch.randn(C, 128, dtype=torch.float32, generator=gp)
    # the reference's own bf16 drift at this block: the same forward with the
    # module in bf16 under CPU autocast (sets the GPU test's tolerance)
    ref_merge.fast_similarity_chunks = lambda a_, bT_, c_: tuple(
        t.to(a_.dtype) if i == 0 else t
        for i, t in enumerate(interp_sim_argmax(a_.float(), bT_.transpose(-1, -2).float())))
    try:
        attn16 = attn.to(torch.bfloat16)
        with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16):
            out16 = attn16(x.to(torch.bfloat16), pos=pos, global_merging=9).float()
    finally:
        ref_merge.fast_similarity_chunks = stock
    rows = torch.arange(0, N, 8)
    torch.save(dict(S=S, w=w, h=h, num_special=ns, heads=H, x_seed=0, weight_seed=0, ratio=0.98,
                    rand_idx=rand_idx, proj=proj,
                    a=cap["a"][0].bfloat16(), b=cap["b"][0].bfloat16(),
                    a_pos=a_idx.int(), b_pos=b_idx.int(),
                    node_max=cap["node_max"].reshape(-1), node_idx=cap["node_idx"].reshape(-1).int(),
                    dst_of_src=dst_of_src.int(), rows=rows, out_rows=out[0, rows].half().clone(),
                    out_rows_bf16=out16[0, rows].half().clone()),
               OUT / "config1_block.pt")
    print("config1_block.pt", (OUT / "config1_block.pt").stat().st_size)


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else ""
    n = int(sys.argv[2]) if len(sys.argv) > 2 else 2
    if what == "config1":
        gen_config1()
    elif what in ("model", "model_bf16", "vanilla", "vanilla_bf16"):
        gen_model(n, vanilla=what.startswith("vanilla"), bf16=what.endswith("bf16"))
    else:
        gen_merge()
        gen_attention()
        gen_frame()
        gen_block()
        for f in sorted(OUT.glob("*.pt")):
            print(f.name, f.stat().st_size)
