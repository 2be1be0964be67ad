"""Benchmark: GPA-VGGT forward on B200 (the reference's bench_e2e workload).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--frames S] [--workload forward|merged_block] [--vanilla]

Workload "forward" (default): the full GPA-VGGT forward -- DINO patch embed,
24 alternating frame/global blocks with the GPA schedule (9 frame+shared-set
blocks, 11 merged blocks at ratio 0.98, 4 core blocks at 0.2), camera head and
DPT depth head -- on S = 200 synthetic 518x518 frames (torch.rand, seed 0),
random-init VGGT-1B weights (gpa_vggt_b200.vggt.init_weights, seed 0), model
in bf16 under bf16 autocast, as eval/bench_e2e.py:90-95 of the reference.
Every head_dim-64 attention (global, frame and DINO blocks) runs on the
sm_100a kernels.  Inputs resident in HBM; the activations are far larger than
L2, so no flush is needed between steps.

Workload "merged_block": one merged global block's attention core at S frames
(roles, projection, similarity argmax, plan, K/V scatter-mean, biased
attention).

With N > 1 (torchrun, one process per GPU, NCCL) the forward's S frames are
sharded by query frame (gpa_vggt_b200/vggt/shard.py): each rank runs S/N
frames end to end and the global blocks all-gather what their keys need
(strong scaling; the time is the max over ranks).  The merged_block workload
runs one replica per rank (weak scaling).  --impl reference times the
reference's CPU path (the oracle port in oracle/, torch on all host cores) on
a bounded sample and extrapolates it to the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

P_TOK = 37 * 37 + 5  # tokens per frame
ATTN_TRAFFIC_RATIO = 350.9 / 341.0  # measured DRAM bytes / algorithmic bytes of attn_kernel
METRIC = "GPA-VGGT fwd latency (ms) & frames/s at S=200, 1/2/4/8 B200; % roofline"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--frames", type=int, default=200)
    ap.add_argument("--ratio", type=float, default=0.98)
    ap.add_argument("--workload", default="forward", choices=["forward", "merged_block"])
    ap.add_argument("--vanilla", action="store_true", help="no merging, no frame+shared set")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm=d["hbm_gbs"], bf16=d["bf16_tflops"], bf16_sus=d["bf16_tflops_sustained"],
                    src="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sus=1400.0, src="fallback")


class Clocks:
    """nvidia-smi samples (200 ms) of one GPU while the timed region runs."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons, power = [], 0.0, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx = max(mx, float(f[1]))
                power.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "power_w_max": max(power) if power else None, "samples": len(sm)}


# ----------------------------------------------------------------------------
# workloads
# ----------------------------------------------------------------------------
def build_model(dev, vanilla=False):
    import torch
    from gpa_vggt_b200.vggt import VGGT, init_weights, vanilla_config
    m = VGGT(**(vanilla_config() if vanilla else {}))
    init_weights(m, seed=0)
    m = m.eval().to(dev).to(torch.bfloat16)
    m.update_patch_dimensions(37, 37)
    return m


def forward(model, images):
    import torch
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        taps, psi = model.aggregator(images)
        pose = model.camera_head(taps, shard=model.aggregator.shard)[-1]
        depth, conf = model.depth_head(taps, images=images, patch_start_idx=psi)
    return pose, depth, conf


def make_block_inputs(S, dev, seed=0):
    import torch
    g = torch.Generator(device="cpu").manual_seed(seed)
    N = S * P_TOK
    x = torch.randn(N, 1024, generator=g).bfloat16()
    qkv = torch.randn(N, 3, 16, 64, generator=g).bfloat16()
    return x.to(dev), qkv.to(dev)


def merged_block(x, qkv, ratio, out=None):
    """One merged block's attention core (attention.py:233-268) on device
    tensors: x [N, 1024] (matching metric), qkv [N, 3, 16, 64] -> [N, 16, 64]."""
    import torch
    from gpa_vggt_b200 import kernels
    from gpa_vggt_b200.merging.merge import build_plan
    N = x.shape[0]
    gen = torch.Generator(device=x.device)
    gen.manual_seed(33)
    plan = build_plan(x, 37, 37, 2, 2, int(N * ratio), False, gen, 128, 5)
    km = torch.empty(plan.n_out, 16, 64, device=x.device, dtype=torch.bfloat16)
    vm = torch.empty_like(km)
    logc = torch.empty(plan.n_out, device=x.device, dtype=torch.float32)
    kernels.merge_kv(qkv[:, 1].transpose(0, 1), plan, out=km.transpose(0, 1), log_counts=logc)
    kernels.merge_kv(qkv[:, 2].transpose(0, 1), plan, out=vm.transpose(0, 1))
    if out is None:
        out = torch.empty(N, 16, 64, device=x.device, dtype=torch.bfloat16)
    kernels.attention(qkv[:, 0].transpose(0, 1)[None], km.transpose(0, 1)[None],
                      vm.transpose(0, 1)[None], logc[None, None], 64 ** -0.5,
                      out=out.transpose(0, 1)[None])
    return out, plan


# ----------------------------------------------------------------------------
# CPU baseline: the reference path on the host cores, composed from samples
# ----------------------------------------------------------------------------
def _t(fn, reps=1):
    t0 = time.perf_counter()
    for _ in range(reps):
        fn()
    return (time.perf_counter() - t0) / reps


def merged_len(S, ratio):
    nd = P_TOK + (S - 1) * 329
    ns = S * P_TOK - nd
    r = int(S * P_TOK * ratio)
    return nd if r >= ns else ns - r + nd


def cpu_block_parts(S):
    """Seconds on the host cores (torch CPU fp32, all threads) for the pieces of
    one GPA forward at S frames, each measured on a bounded sample and scaled by
    the fraction of rows / frames it covers."""
    import torch
    import torch.nn.functional as F
    from oracle import gpa_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    N = S * P_TOK
    parts = {}
    # linear layers of one block (qkv, proj, fc1, fc2) on 1024 rows
    R = 1024
    xr = torch.randn(R, 1024, generator=g)
    w = [torch.randn(o, i, generator=g) * 0.02 for o, i in ((3072, 1024), (1024, 1024), (4096, 1024), (1024, 4096))]
    def lin():
        F.linear(xr, w[0]); F.linear(xr, w[1]); h = F.linear(xr, w[2]); F.linear(h, w[3])
    parts["linear_per_block"] = _t(lin, 2) * N / R
    # per-frame attention (frame blocks, DINO blocks, own-frame part of early blocks)
    qf = torch.randn(1, 16, P_TOK, 64, generator=g)
    parts["frame_attn_per_block"] = _t(lambda: F.scaled_dot_product_attention(qf, qf, qf), 2) * S
    # shared-set attention of an early block on a query sample
    qs = 2048
    q = torch.randn(1, 16, qs, 64, generator=g)
    ksh = torch.randn(1, 16, 30 * S, 64, generator=g)
    parts["shared_attn_per_block"] = _t(lambda: F.scaled_dot_product_attention(q, ksh, ksh,
                                        attn_mask=torch.zeros(1, 1, 1, 30 * S)), 1) * N / qs
    # merged-block matching (roles, projection, normalise) at full size, similarity on a sample
    x = torch.randn(N, 1024, generator=g)
    def match():
        rand = torch.randint(4, (S - 1, 18, 18), generator=g)
        mask = O.dst_mask(S, 37, 37, 2, 2, 5, rand)
        d, s_ = O.split_positions(mask)
        mn = O.normalize_rows(x @ torch.randn(1024, 128, generator=g))
        return mn, d, s_
    t0 = time.perf_counter()
    mn, dst, src = match()
    t_match = time.perf_counter() - t0
    sub = max(256, src.numel() // 256)
    t_sim = _t(lambda: (mn[src[:sub]] @ mn[dst].T).max(dim=1)) * src.numel() / sub
    kv = torch.randn(N, 1024, generator=g)
    idx = torch.randint(0, dst.numel(), (src.numel(),), generator=g)
    def merge():
        for _ in range(2):
            mid = kv[dst].clone()
            mid.index_add_(0, idx, kv[src])
    t_merge = _t(merge)
    for name, ratio in (("merged_0.98", 0.98), ("merged_0.2", 0.2)):
        nm_ = merged_len(S, ratio)
        qq = torch.randn(1, 16, 512, 64, generator=g)
        kk = torch.randn(1, 16, nm_, 64, generator=g)
        b = torch.rand(1, 1, 1, nm_, generator=g)
        t_att = _t(lambda: F.scaled_dot_product_attention(qq, kk, kk, attn_mask=b)) * N / 512
        parts[f"{name}_per_block"] = t_match + t_sim + t_merge + t_att
    return parts


def cpu_forward_ms(S, vanilla=False):
    p = cpu_block_parts(S)
    lin = p["linear_per_block"] * 72                      # 24 DINO + 24 frame + 24 global
    frame = p["frame_attn_per_block"] * (24 + 24)         # DINO + frame blocks
    if vanilla:
        glob = merged_ms = 0.0
        import torch
        import torch.nn.functional as F
        N = S * P_TOK
        q = torch.randn(1, 16, 512, 64)
        k = torch.randn(1, 16, N, 64)
        glob = _t(lambda: F.scaled_dot_product_attention(q, k, k)) * N / 512 * 24
    else:
        glob = (9 * (p["frame_attn_per_block"] + p["shared_attn_per_block"])
                + 11 * p["merged_0.98_per_block"] + 4 * p["merged_0.2_per_block"])
    total = lin + frame + glob
    sample = (f"GPA forward at S={S} composed from sampled components on the host cores "
              f"(torch CPU fp32): linears on 1024 rows, per-frame attention on 1 frame, "
              f"global/merged attention on 512-2048 query rows, similarity on 1/256 of the src "
              f"rows, matching and K/V merge at full size; scaled by rows/frames and the block "
              f"schedule (24 DINO + 24 frame + 9 early + 11 merged + 4 core); heads excluded")
    return total * 1e3, sample


# ----------------------------------------------------------------------------
def main():
    args = parse()
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    S = args.frames
    fwd = args.workload == "forward"
    if fwd:
        workload = f"gpa_vggt_forward_S{S}" + ("_vanilla" if args.vanilla else "")
        config = {"workload": workload, "model": "VGGT-1B (random init, seed 0)", "frames": S,
                  "image": "518x518", "tokens_per_global_block": S * P_TOK,
                  "schedule": "vanilla" if args.vanilla else
                  "9 frame+shared, 11 merged@0.98, 4 core@0.2 (blocks 9-23)",
                  "global_batch": 1, "seq_len": S * P_TOK,
                  "l2": "activations > L2 (no flush needed)"}
        metric = METRIC
    else:
        config = {"workload": f"gpa_merged_block_S{S}", "frames": S, "tokens": S * P_TOK,
                  "merge_ratio": args.ratio, "heads": 16, "head_dim": 64,
                  "l2": "inputs > L2 (no flush needed)"}
        metric = f"GPA merged global block latency (ms) at S={S}"
    if world == 1:
        config["parallelism"] = "single GPU"
    elif fwd:
        config["parallelism"] = f"query-frame shards x{world} (NCCL all-gather of keys per global block)"
    else:
        config["parallelism"] = f"replicas x{world}"
    base = {"metric": metric, "unit": "ms", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": False,
            "scaling": "strong" if (fwd and world > 1) else "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (torch.rand frames / seeded N(0,1) tokens, random-init weights)",
            "config": config}

    if args.impl == "reference":
        if rank != 0:
            return
        vals, sample = [], ""
        for _ in range(max(1, args.warmup) + args.steps):
            if fwd:
                ms, sample = cpu_forward_ms(S, args.vanilla)
            else:
                p = cpu_block_parts(S)
                ms = p["merged_0.98_per_block"] * 1e3
                sample = f"one merged block at S={S}, composed from sampled components"
            vals.append(ms)
        ms = statistics.mean(vals[-args.steps:])
        line = dict(base, impl="reference", value=ms, ms_per_step=ms,
                    cpu_baseline={"value": ms, "unit": "ms", "cores": os.cpu_count(), "kind": "port",
                                  "sample": sample},
                    e2e={"value": ms, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
        if fwd:
            line["frames_per_s"] = S / (ms / 1e3)
        print(json.dumps(line), flush=True)
        return

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    from gpa_vggt_b200 import _lib, kernels
    _lib.load()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    if fwd:
        model = build_model(dev, args.vanilla)
        g = torch.Generator(device="cpu").manual_seed(0)
        images = torch.rand(1, S, 3, 518, 518, generator=g).to(torch.bfloat16)
        S_local = S
        if world > 1:
            from gpa_vggt_b200.vggt.shard import FrameShard
            shard = FrameShard(S)
            model.set_shard(shard)
            images = images[:, shard.f0:shard.f1]
            S_local = shard.local
        images = images.contiguous().to(dev)
        step = lambda: forward(model, images)  # noqa: E731
    else:
        x, qkv = make_block_inputs(S, dev, seed=rank)
        out = torch.empty(S * P_TOK, 16, 64, device=dev, dtype=torch.bfloat16)
        step = lambda: merged_block(x, qkv, args.ratio, out=out)  # noqa: E731

    for _ in range(args.warmup):
        step()
    barrier()
    kernels.ATTN_TIMING = []
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    l0 = _lib.launch_count()
    with Clocks(local) as clk:
        # the timed steps form the CUDA profiler range (ncu --profile-from-start off
        # captures exactly these launches; a no-op without a profiler)
        torch.cuda.profiler.start()
        start.record()
        for _ in range(args.steps):
            step()
        stop.record()
        barrier()
        torch.cuda.profiler.stop()
    launches = _lib.launch_count() - l0
    timing, kernels.ATTN_TIMING = kernels.ATTN_TIMING, None
    ms = start.elapsed_time(stop) / args.steps
    attn_ms = sum(rec[0].elapsed_time(rec[1]) for rec in timing) / args.steps
    attn_flops = sum(rec[2] for rec in timing) / args.steps
    attn_bytes = sum(rec[3] for rec in timing) / args.steps
    n_attn = len(timing) // args.steps
    if world > 1:
        t = torch.tensor([ms, attn_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, attn_ms = t.tolist()

    # end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        if fwd:
            h_img = images.cpu().pin_memory()
            h_pose = torch.empty(1, S, 9, dtype=torch.float32).pin_memory()
            h_depth = torch.empty(1, S_local, 518, 518, 1, dtype=torch.float32).pin_memory()
            h_conf = torch.empty(1, S_local, 518, 518, dtype=torch.float32).pin_memory()

            def e2e_step():
                d_img = h_img.to(dev, non_blocking=True)
                pose, depth, conf = forward(model, d_img)
                h_pose.copy_(pose, non_blocking=True)
                h_depth.copy_(depth, non_blocking=True)
                h_conf.copy_(conf, non_blocking=True)

            h2d = h_img.numel() * h_img.element_size()
            d2h = sum(t.numel() * t.element_size() for t in (h_pose, h_depth, h_conf))
        else:
            from gpa_vggt_b200.merging.merge import token_merge_bipartite2d
            from gpa_vggt_b200.merging.fused_attention import attention_keybias
            hx, hq = x.cpu().pin_memory(), qkv.cpu().pin_memory()
            N = S * P_TOK
            hout = torch.empty(N, 1024, dtype=torch.bfloat16).pin_memory()

            def e2e_step():
                dx, dq = hx.to(dev, non_blocking=True), hq.to(dev, non_blocking=True)
                gen = torch.Generator(device=dev)
                gen.manual_seed(33)
                m = token_merge_bipartite2d(dx[None], 37, 37, 2, 2, int(N * args.ratio), False, gen,
                                            metric_dim=128, num_special=5)
                o = attention_keybias(dq[:, 0].transpose(0, 1)[None],
                                      m.heads(dq[:, 1].transpose(0, 1)[None]),
                                      m.heads(dq[:, 2].transpose(0, 1)[None]),
                                      m.size.log().reshape(1, 1, 1, -1), 64 ** -0.5)
                hout.copy_(o[0].transpose(0, 1).reshape(N, 1024), non_blocking=True)

            h2d = (hx.numel() + hq.numel()) * 2
            d2h = hout.numel() * 2
        e2e_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            e2e_step()
        e1.record()
        barrier()
        e_ms = e0.elapsed_time(e1) / args.steps
        if world > 1:
            t = torch.tensor([e_ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e_ms = t.item()
        e2e = {"value": e_ms, "unit": "ms", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
        if fwd:
            e2e["frames_per_s"] = S / (e_ms / 1e3)   # the job covers S frames at any N

    pk = peaks()
    achieved = attn_flops / (attn_ms * 1e-3) / 1e12
    roof = {"kernel": "attn_kernel (gpa_attention_keybias), all launches of a step",
            "bound": "tensor", "achieved": achieved, "peak": pk["bf16_sus"], "unit": "TFLOP/s",
            "frac": achieved / pk["bf16_sus"], "peak_kind": f"{pk['src']} sustained bf16 (long step)",
            "frac_of_burst": achieved / pk["bf16"], "flops_per_step": attn_flops,
            "launches_per_step": n_attn, "ms_per_step": attn_ms,
            "share_of_step": attn_ms / ms,
            # DRAM bytes per step: the algorithmic q/k/v/o bytes of this step's launches
            # times the measured ratio dram__bytes_read+write / algorithmic = 1.03 of
            # the ncu capture in profiles/attn_kernel_q16384_k66845.md (K/V read once)
            "traffic": ATTN_TRAFFIC_RATIO * attn_bytes, "traffic_unit": "bytes per step",
            "algorithmic_bytes_per_step": attn_bytes}
    line = dict(base, value=ms, ms_per_step=ms, gpu_launches=launches, roofline=roof, e2e=e2e,
                clocks=clk.summary())
    if fwd:
        line["frames_per_s"] = S / (ms / 1e3)
        line["gpu_memory_peak_gib"] = torch.cuda.max_memory_allocated(dev) / 2 ** 30
    if world == 1 and not args.no_cpu:   # the CPU baseline is an N=1 figure
        if fwd:
            cms, sample = cpu_forward_ms(S, args.vanilla)
        else:
            cms, sample = cpu_block_parts(S)["merged_0.98_per_block"] * 1e3, f"merged block at S={S}"
        line["cpu_baseline"] = {"value": cms, "unit": "ms", "cores": os.cpu_count(), "kind": "port",
                                "sample": sample}
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
