"""Runs of the reference itself, for measurement -- TEST/BENCH INFRASTRUCTURE.

Nothing in the product (gpa_vggt_b200/) imports this module.  The unmodified
reference, noheat61/GPA-VGGT, is installed offline into baseline/_ref
(git-ignored; the tree carries it to the GPU box).  This module imports it
from there only, and times it in two ways.

* Its CPU path on the host cores.  This is bench.py's reference arm and its
  cpu_baseline leg.
  - direct: the whole forward (aggregator, camera head, DPT head) in fp32 at
    an S that a CPU runs: the S=10 forward of BASELINE config 2.  The merged
    block of config 1 is timed by `block_ms`.
  - composed: at S=200 the reference's CPU merged attention would hold a
    [16, 274,800, 66,845] fp32 score matrix (1.2 TB).  So its own pieces are
    timed on bounded samples and composed by the block schedule: 24 DINO,
    24 frame and 24 global blocks (9 frame + shared set, 11 merged at 0.98,
    4 core at 0.2), then the camera and DPT heads.  The result is an
    extrapolation and is labelled as one.
* Its GPU path on one B200 (`python -m oracle.reference_runs gpu ...`): its
  two Triton kernels at the S=200 shapes, and its bf16 forward timed as
  eval/bench_e2e.py:49-98 times it.

Where baseline/_ref is missing, the CPU timings use this directory's port of
the reference instead (kind "port").
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

import torch
import torch.nn.functional as F

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"
P_TOK = 37 * 37 + 5
SCHEDULE = "24 DINO + 24 frame + 9 frame+shared + 11 merged@0.98 + 4 core@0.2 blocks, camera + DPT heads"


def have_reference() -> bool:
    return (REF / "merging" / "merge.py").exists() and (REF / "vggt" / "models" / "vggt.py").exists()


def _ref():
    """The reference's modules, from baseline/_ref."""
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import merging.merge as merge                                   # noqa: E402
    from vggt.models.vggt import VGGT                               # noqa: E402
    from vggt.layers.block import Block                             # noqa: E402
    from vggt.layers.rope import PositionGetter, RotaryPositionEmbedding2D   # noqa: E402
    from vggt.heads.dpt_head import DPTHead                         # noqa: E402
    from vggt.heads.camera_head import CameraHead                   # noqa: E402
    return dict(merge=merge, VGGT=VGGT, Block=Block, PositionGetter=PositionGetter,
                RoPE=RotaryPositionEmbedding2D, DPTHead=DPTHead, CameraHead=CameraHead)


def _init(module, seed=0):
    sys.path.insert(0, str(ROOT))
    from gpa_vggt_b200.vggt.model import init_weights
    return init_weights(module, seed=seed)


def merged_len(S: int, ratio: float) -> int:
    nd = P_TOK + (S - 1) * 329
    ns = S * P_TOK - nd
    r = int(S * P_TOK * ratio)
    return nd if r >= ns else ns - r + nd


def _med(fn, reps=3):
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts)


def threads() -> int:
    return torch.get_num_threads()


# ----------------------------------------------------------------------------
# CPU: direct runs
# ----------------------------------------------------------------------------
def build_cpu_model(vanilla=False):
    R = _ref()
    model = R["VGGT"](merging=None, early_frame_split=0) if vanilla else R["VGGT"]()
    _init(model, 0)
    model.eval()
    model.update_patch_dimensions(37, 37)
    return model


def forward_ms(model, S: int) -> float:
    """One fp32 forward of the reference on the CPU (aggregator + camera +
    DPT heads, eval/bench_e2e.py:90-95)."""
    images = torch.rand(1, S, 3, 518, 518, generator=torch.Generator().manual_seed(0))
    t0 = time.perf_counter()
    with torch.no_grad():
        toks, psi = model.aggregator(images)
        model.camera_head(toks)
        model.depth_head(toks, images=images, patch_start_idx=psi)
    return (time.perf_counter() - t0) * 1e3


def block_ms(S: int = 4, ratio: float = 0.98, vanilla=False) -> float:
    """One global block of the reference at S frames on the CPU (config 1:
    S=4, merged at 0.98): Block.forward(x, pos, global_merging)."""
    R = _ref()
    rope = R["RoPE"](frequency=100)
    blk = R["Block"](1024, 16, mlp_ratio=4.0, init_values=0.01, qk_norm=True, rope=rope,
                     merge_ratio=ratio)
    blk.attn.merge_metric_dim = 128
    blk.attn.patch_width = blk.attn.patch_height = 37
    _init(blk, 0)
    blk.eval()
    N = S * P_TOK
    x = torch.randn(1, N, 1024, generator=torch.Generator().manual_seed(0))
    pos = _positions(R, S)
    t0 = time.perf_counter()
    with torch.no_grad():
        blk(x, pos=pos, global_merging=None if vanilla else 9)
    return (time.perf_counter() - t0) * 1e3


def _positions(R, S):
    pos = R["PositionGetter"]()(S, 37, 37, device="cpu") + 1
    pos = torch.cat([torch.zeros(S, 5, 2, dtype=pos.dtype), pos], 1)
    return pos.reshape(1, S * P_TOK, 2)


# ----------------------------------------------------------------------------
# CPU: the reference's pieces on bounded samples, composed
# ----------------------------------------------------------------------------
class Composer:
    """Per-piece seconds of one reference forward at S frames, each timed on a
    bounded sample with the reference's own modules and calls."""

    def __init__(self, S: int, vanilla: bool = False):
        self.S, self.vanilla = S, vanilla
        self.R = _ref()
        R = self.R
        g = torch.Generator().manual_seed(0)
        self.g = g
        rope = R["RoPE"](frequency=100)
        self.block = _init(R["Block"](1024, 16, mlp_ratio=4.0, init_values=0.01, qk_norm=True,
                                      rope=rope), 0).eval()
        # the frame-local pieces run on a batch of up to 4 frames (the forward
        # runs frame blocks batched over its frames; one frame's GEMMs are less
        # efficient per token on some hosts) and are divided per frame
        self.nf = min(S, 4)
        self.x1 = torch.randn(self.nf, P_TOK, 1024, generator=g)
        self.pos1 = _positions(R, 1).expand(self.nf, P_TOK, 2).contiguous()
        self.qf = torch.randn(self.nf, 16, P_TOK, 64, generator=g)
        self.q1 = self.qf[:1]
        N = S * P_TOK
        self.N = N
        nd = P_TOK + (S - 1) * 329
        self.nd, self.ns = nd, N - nd
        self.x = torch.randn(1, N, 1024, generator=g)
        self.k = torch.randn(1, 16, N, 64, generator=g)                   # fp32 after qk-LN
        self.v = torch.randn(1, 16, N, 64, generator=g)
        self.dpt = _init(R["DPTHead"](dim_in=2048, output_dim=2, activation="exp",
                                      conf_activation="expp1"), 0).eval()
        self.cam = _init(R["CameraHead"](dim_in=2048), 0).eval()
        self.warm = False

    def parts(self, reps: int = 3) -> dict:
        """Seconds per piece: the median of `reps` runs of each piece (the
        first call of a Composer runs every piece once untimed: TorchScript
        compiles the reference's matcher on its first call, and first
        allocations are slow)."""
        if not self.warm:
            self.warm = True
            self.parts(reps=1)
        R, S, N = self.R, self.S, self.N
        p = {}
        self.reps = reps
        with torch.no_grad():
            # a frame's tokens through one block (frame, DINO and the linears,
            # norms and MLP of a global block), and its own-frame attention
            p["block_per_frame"] = _med(lambda: self.block(self.x1, pos=self.pos1), reps) / self.nf
            p["frame_sdpa_per_frame"] = _med(
                lambda: F.scaled_dot_product_attention(self.qf, self.qf, self.qf), reps) / self.nf
            if self.vanilla:
                rq = 128
                q = self.q1[:, :, :rq]
                kk = self.k.to(torch.float32)
                p["global_attn_per_block"] = _med(lambda: F.scaled_dot_product_attention(q, kk, kk), reps) * N / rq
            else:
                # early blocks, CPU path: own patches + every frame's shared set in
                # one SDPA with the +log size bias (attention.py:178-206), per frame
                kk = torch.randn(1, 16, 1369 + 30 * S, 64, generator=self.g)
                mask = torch.zeros(1, 16, 1, 1369 + 30 * S)
                p["early_attn_per_frame"] = _med(
                    lambda: F.scaled_dot_product_attention(self.q1, kk, kk, attn_mask=mask), reps)
                p.update(self._merged())
            # heads: DPT on one frame (8-frame chunks, dpt_head.py:150-213), camera on S frames
            taps = [torch.randn(1, 1, P_TOK, 2048, generator=self.g)] * 24
            img1 = torch.rand(1, 1, 3, 518, 518, generator=self.g)
            p["dpt_per_frame"] = _med(lambda: self.dpt(taps, images=img1, patch_start_idx=5), reps)
            cam_taps = [torch.randn(1, S, P_TOK, 2048, generator=self.g)] * 24
            p["camera"] = _med(lambda: self.cam(cam_taps), reps)
        return p

    def _merged(self) -> dict:
        """The merged blocks' pieces: token_merge_bipartite2d without its
        matcher (roles, projection, argsorts, gathers) at full size; the
        reference's CPU matcher fast_similarity_chunks on a row sample; the
        merge.heads scatter-means of K (fp32) and V at full size; SDPA with
        the log(count) mask (attention.py:270-276) on a query sample."""
        R, S, N = self.R, self.S, self.N
        merge = R["merge"]
        p = {}
        stock = merge.fast_similarity_chunks
        captured = {}

        def stub(a, bT, chunk):
            captured["a"], captured["bT"] = a, bT
            return a[..., 0].clone(), torch.zeros(a.shape[:-1], dtype=torch.long)
        merge.fast_similarity_chunks = stub
        try:
            g = torch.Generator().manual_seed(33)
            t0 = time.perf_counter()
            m = merge.token_merge_bipartite2d(self.x, 37, 37, 2, 2, int(N * 0.98), False, g,
                                              metric_dim=128, num_special=5)
            p["merge_no_matcher"] = time.perf_counter() - t0
        finally:
            merge.fast_similarity_chunks = stock
        reps = self.reps
        rs = min(1000, self.ns)
        a, bT = captured["a"][:, :rs].contiguous(), captured["bT"]
        p["matcher"] = _med(lambda: stock(a, bT, rs), reps) * self.ns / rs
        p["merge_heads_kv"] = _med(lambda: (m.heads(self.k), m.heads(self.v)), reps)
        rq = 128
        q = self.q1[:, :, :rq]
        for name, ratio in (("attn_0.98", 0.98), ("attn_0.2", 0.2)):
            nm = merged_len(S, ratio)
            kk, vv = self.k[:, :, :nm], self.v[:, :, :nm]
            bias = torch.rand(1, 16, 1, nm, generator=self.g)
            p[name] = _med(lambda: F.scaled_dot_product_attention(q, kk, vv, attn_mask=bias), reps) * N / rq
        return p

    def compose_ms(self, p: dict) -> float:
        S = self.S
        t = 48 * S * p["block_per_frame"]                                   # DINO + frame blocks
        t += 24 * S * max(p["block_per_frame"] - p["frame_sdpa_per_frame"], 0.0)   # global linears
        if self.vanilla:
            t += 24 * p["global_attn_per_block"]
        else:
            t += 9 * S * p["early_attn_per_frame"]
            merged = p["merge_no_matcher"] + p["matcher"] + p["merge_heads_kv"]
            t += 11 * (merged + p["attn_0.98"]) + 4 * (merged + p["attn_0.2"])
        t += S * p["dpt_per_frame"] + p["camera"]
        return t * 1e3


def composed_sample_note(S, vanilla):
    return (f"{'vanilla' if vanilla else 'GPA'} VGGT forward at S={S} composed from the reference's own "
            f"CPU pieces (baseline/_ref, fp32, all host threads): a block and the own-frame SDPA "
            f"on a batch of up to 4 frames, the early blocks' SDPA with the shared set per frame, "
            f"token_merge_bipartite2d without its matcher at full size, fast_similarity_chunks on "
            f"1,000 src rows, merge.heads of K and V at full size, the masked SDPA on 128 query "
            f"rows, the DPT head on one frame, the camera head on S frames; scaled by rows/frames "
            f"and composed by the schedule ({SCHEDULE}): an extrapolation")


# ----------------------------------------------------------------------------
# CPU without baseline/_ref: the port (gpa_oracle.py) composed the same way
# ----------------------------------------------------------------------------
def port_forward_ms(S: int, vanilla: bool = False) -> float:
    """The forward at S composed from this directory's port of the reference's
    CPU path (torch CPU fp32): the same pieces as Composer, with the port's
    functions where the reference's are not at hand."""
    from oracle import gpa_oracle as O
    g = torch.Generator().manual_seed(0)
    N = S * P_TOK
    R = 1024
    xr = torch.randn(R, 1024, generator=g)
    w = [torch.randn(o, i, generator=g) * 0.02 for o, i in ((3072, 1024), (1024, 1024), (4096, 1024), (1024, 4096))]

    def lin():
        F.linear(xr, w[0]); F.linear(xr, w[1]); h = F.linear(xr, w[2]); F.linear(h, w[3])
    t_lin = _med(lin, 1) * N / R
    qf = torch.randn(1, 16, P_TOK, 64, generator=g)
    t_frame = _med(lambda: F.scaled_dot_product_attention(qf, qf, qf), 1) * S
    t = 72 * t_lin + 48 * t_frame
    q = torch.randn(1, 16, 64, 64, generator=g)
    if vanilla:
        k = torch.randn(1, 16, N, 64, generator=g)
        return (t + 24 * _med(lambda: F.scaled_dot_product_attention(q, k, k), 1) * N / 64) * 1e3
    ksh = torch.randn(1, 16, 1369 + 30 * S, 64, generator=g)
    t += 9 * S * _med(lambda: F.scaled_dot_product_attention(qf, ksh, ksh), 1)
    x = torch.randn(N, 1024, generator=g)
    t0 = time.perf_counter()
    rand = torch.randint(4, (S - 1, 18, 18), generator=g)
    d, s_ = O.split_positions(O.dst_mask(S, 37, 37, 2, 2, 5, rand))
    mn = O.normalize_rows(x @ torch.randn(1024, 128, generator=g))
    t_match = time.perf_counter() - t0
    sub = min(1000, s_.numel())
    t_sim = _med(lambda: (mn[s_[:sub]] @ mn[d].T).max(dim=1), 1) * s_.numel() / sub
    kv = torch.randn(N, 1024, generator=g)
    idx = torch.randint(0, d.numel(), (s_.numel(),), generator=g)

    def merge():
        for _ in range(2):
            mid = kv[d].clone()
            mid.index_add_(0, idx, kv[s_])
    t_merge = _med(merge, 1)
    for n_blk, ratio in ((11, 0.98), (4, 0.2)):
        kk = torch.randn(1, 16, merged_len(S, ratio), 64, generator=g)
        t_att = _med(lambda: F.scaled_dot_product_attention(q, kk, kk), 1) * N / 64
        t += n_blk * (t_match + t_sim + t_merge + t_att)
    return t * 1e3


def port_sample_note(S, vanilla):
    return (f"{'vanilla' if vanilla else 'GPA'} VGGT forward at S={S} composed from this repo's port "
            f"of the reference's CPU path (oracle/, torch CPU fp32): linears on 1,024 rows, one "
            f"frame's attention, matching at full size, similarity on 1,000 src rows, K/V merge at "
            f"full size, attention on 64 query rows; heads excluded; an extrapolation")


# ----------------------------------------------------------------------------
# GPU: the reference's Triton kernels and bf16 forward on one B200
# ----------------------------------------------------------------------------
def _cuda_ms(fn, warmup=2, iters=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def gpu_kernels(out_lines):
    """The reference's Triton kernels and this library's kernels on the same
    inputs at the S=200 shapes, CUDA events, one B200."""
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import merging.fused_attention as rfa                         # noqa: E402
    import merging.fused_similarity as rfs                        # noqa: E402
    sys.path.insert(0, str(ROOT))
    from gpa_vggt_b200 import kernels
    dev = "cuda"
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    M, Nd = 207955, 66845
    a = torch.randn(1, M, 128, device=dev, generator=g)
    b = torch.randn(1, Nd, 128, device=dev, generator=g)
    a = (a / a.norm(dim=-1, keepdim=True)).bfloat16()
    b = (b / b.norm(dim=-1, keepdim=True)).bfloat16()
    flops = 2.0 * M * Nd * 128
    t_ref = _cuda_ms(lambda: rfs.fused_similarity_argmax(a, b))
    t_ours = _cuda_ms(lambda: kernels.sim_argmax(a, b))
    out_lines.append(dict(kernel="similarity argmax", shape=f"{M} x {Nd} x 128", ref_ms=t_ref,
                          ours_ms=t_ours, ref_tflops=flops / t_ref / 1e9,
                          ours_tflops=flops / t_ours / 1e9, speedup=t_ref / t_ours))
    for Mq, Nk, label in ((274800, 66845, "merged block"), (274800, 219840, "core block")):
        q = torch.randn(1, 16, Mq, 64, device=dev, generator=g).bfloat16()
        k = torch.randn(1, 16, Nk, 64, device=dev, generator=g).bfloat16()
        v = torch.randn(1, 16, Nk, 64, device=dev, generator=g).bfloat16()
        cnt = 1 + torch.poisson(torch.ones(Nk, device=dev), generator=g)
        bias = cnt.log().bfloat16().reshape(1, 1, 1, Nk).expand(1, 16, 1, Nk).contiguous()
        flops = 4.0 * Mq * Nk * 64 * 16
        t_ref = _cuda_ms(lambda: rfa.attention_keybias(q, k, v, bias, 0.125), 1, 2)
        t_ours = _cuda_ms(lambda: kernels.attention(q, k, v, bias.float()[:, :, 0], 0.125), 1, 2)
        out_lines.append(dict(kernel=f"biased attention ({label})", shape=f"{Mq} x {Nk} x 16 x 64",
                              ref_ms=t_ref, ours_ms=t_ours, ref_tflops=flops / t_ref / 1e9,
                              ours_tflops=flops / t_ours / 1e9, speedup=t_ref / t_ours))
        del q, k, v


def gpu_forward(S, vanilla, warmup=2, iters=3):
    """The reference's bf16 forward on one B200 (random init), timed as
    eval/bench_e2e.py:49-98 times it: wall clock around synchronise, mean
    over iters after warmup."""
    R = _ref()
    torch.manual_seed(0)
    model = R["VGGT"](merging=None, early_frame_split=0) if vanilla else R["VGGT"]()
    _init(model, 0)
    model = model.eval().cuda().to(torch.bfloat16)
    model.update_patch_dimensions(37, 37)
    images = torch.rand(1, S, 3, 518, 518, device="cuda", dtype=torch.bfloat16,
                        generator=torch.Generator(device="cuda").manual_seed(0))

    def e2e():
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            toks, psi = model.aggregator(images)
            pose = model.camera_head(toks)
            depth, conf = model.depth_head(toks, images=images, patch_start_idx=psi)
        return pose, depth, conf
    for _ in range(warmup):
        e2e()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(iters):
        e2e()
    torch.cuda.synchronize()
    return (time.perf_counter() - t0) / iters * 1e3


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("cpu", help="the reference on the host cores")
    c.add_argument("--frames", type=int, default=200)
    c.add_argument("--vanilla", action="store_true")
    c.add_argument("--direct", action="store_true", help="time the whole forward (small S only)")
    c.add_argument("--block", action="store_true", help="time one merged global block (config 1)")
    c.add_argument("--reps", type=int, default=3)
    gk = sub.add_parser("gpu", help="the reference's GPU path on one B200")
    gk.add_argument("what", choices=["kernels", "forward"])
    gk.add_argument("--frames", type=int, default=200)
    gk.add_argument("--vanilla", action="store_true")
    a = ap.parse_args(argv)
    if not have_reference():
        print(json.dumps({"unavailable": "the reference is not installed in baseline/_ref"}))
        return 0
    if a.cmd == "cpu":
        if a.block:
            ms = [block_ms(a.frames, vanilla=a.vanilla) for _ in range(a.reps)]
            print(json.dumps({"what": f"reference global block S={a.frames}", "ms": ms,
                              "median_ms": statistics.median(ms), "threads": threads()}))
        elif a.direct:
            model = build_cpu_model(a.vanilla)
            ms = [forward_ms(model, a.frames) for _ in range(a.reps)]
            print(json.dumps({"what": f"reference forward S={a.frames}", "ms": ms,
                              "median_ms": statistics.median(ms), "threads": threads()}))
        else:
            comp = Composer(a.frames, a.vanilla)
            vals = []
            for _ in range(a.reps):
                parts = comp.parts()
                vals.append(comp.compose_ms(parts))
            print(json.dumps({"what": f"reference forward S={a.frames} composed", "ms": vals,
                              "median_ms": statistics.median(vals), "parts_s": parts,
                              "threads": threads()}))
        return 0
    if a.what == "kernels":
        lines = []
        gpu_kernels(lines)
        for ln in lines:
            print(json.dumps(ln), flush=True)
    else:
        ms = gpu_forward(a.frames, a.vanilla)
        print(json.dumps({"what": f"reference GPU forward S={a.frames}"
                          + (" vanilla" if a.vanilla else ""), "ms": ms,
                          "frames_per_s": a.frames / (ms / 1e3)}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
