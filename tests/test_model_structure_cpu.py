"""The model's wiring, checked on the CPU: the GPA-VGGT caller is run in fp32
with every kernel entry point replaced by the CPU oracle (the checker), and
compared with the reference's own fp32 forward (tests/golden/model_s2.pt).  With
the arithmetic taken out of the picture, any layout, stride, RoPE, schedule or
head mistake shows up as a large error; the bound is fp32-level."""
from types import SimpleNamespace

import pytest
import torch

from oracle import gpa_oracle as O


def _oracle_kernels(monkeypatch, rand_idx, proj):
    from gpa_vggt_b200 import kernels
    from gpa_vggt_b200.vggt import layers

    from cpu_kernels import attention   # noqa: E402 (tests/ is on sys.path under pytest)

    def build_plan(metric, w, h, sx, sy, r, no_rand=False, generator=None, metric_dim=0,
                   num_special=5, rand_idx=None, proj=None):
        N = metric.shape[0]
        S = N // (w * h + num_special)
        mask = O.dst_mask(S, w, h, sx, sy, num_special, rand_idx)
        dst, src = O.split_positions(mask)
        m = O.normalize_rows(O.project_metric(metric.float(), proj.float(), autocast_bf16=False))
        nm, ni, _ = O.sim_argmax(m[src], m[dst])
        plan = O.merge_plan(nm, ni, r, dst.numel())
        return SimpleNamespace(oracle=plan, dst=dst, src=src, counts=plan.counts.float())

    def merge_kv(t, plan, mean=True, out=None, log_counts=None):
        res = O.merge_heads(t, plan.oracle, plan.dst, plan.src).to(t.dtype)
        if out is not None:
            out.copy_(res)
            return out
        return res

    def frame_pool(k, v, S, ph, pw, pts, kp):
        H, N, D = k.shape
        P = ph * pw + pts
        pk, pv, size, _ = O.frame_pool(k.reshape(H, S, P, D), v.reshape(H, S, P, D), ph, pw, pts, kp)
        return pk.to(k.dtype), pv.to(k.dtype), size

    def lse_combine(oa, la, ob, lb, out=None):
        res = O.lse_combine(oa, la.double(), ob, lb.double()).to(oa.dtype)
        out.copy_(res)
        return out

    monkeypatch.setattr(kernels, "attention", attention)
    monkeypatch.setattr(kernels, "merge_kv", merge_kv)
    monkeypatch.setattr(kernels, "frame_pool", frame_pool)
    monkeypatch.setattr(kernels, "lse_combine", lse_combine)
    monkeypatch.setattr(layers, "build_plan", build_plan)
    monkeypatch.setattr(layers, "BF16", torch.float32)   # keep the whole run in fp32


def test_model_wiring_matches_reference_fp32(monkeypatch, golden):
    from gpa_vggt_b200.vggt import VGGT, init_weights
    g = golden("model_s2.pt")
    _oracle_kernels(monkeypatch, g["rand_idx"], g["proj"])
    m = VGGT()
    init_weights(m, seed=0)
    m.eval()
    m.update_patch_dimensions(37, 37)
    for blk in m.aggregator.global_blocks:
        blk.attn.rng_override = (g["rand_idx"], g["proj"])
    images = torch.rand(1, g["S"], 3, 518, 518, generator=torch.Generator().manual_seed(g["image_seed"]))
    with torch.no_grad():
        out = m(images)

    def rel(a, b):
        return float((a.double() - b.double()).norm() / b.double().norm())
    e = (rel(out["pose_enc"], g["pose_enc"]), rel(out["depth"], g["depth"].float()),
         rel(out["depth_conf"], g["depth_conf"].float()))
    print("rel-L2 pose/depth/conf", e)
    assert e[0] < 1e-3
    assert e[1] < 2e-3 and e[2] < 2e-3   # depth and conf are stored in fp16
