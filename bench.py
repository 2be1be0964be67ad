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
reference's own CPU path on all host cores (oracle/reference_runs.py, with the
unmodified reference from baseline/_ref; the port in oracle/ where it is
missing): the whole fp32 forward at S <= 10, and at S=200 its pieces on
bounded samples composed by the block schedule (an extrapolation, labelled).
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
# Measured DRAM bytes (ncu dram__bytes_read.sum + dram__bytes_write.sum of one
# launch) over the algorithmic q/k/v/o bytes of attn_kernel, S=200, 16 heads:
# 274,800 x 66,845 keys: 1.384 GB / 1.400 GB; 274,800 x 219,840 keys:
# 4.847 GB / 2.026 GB (a head's 56 MB of K/V no longer stays in L2 between the
# waves of its query tiles).  Launches up to 66,845 keys use the first ratio.
ATTN_TRAFFIC_RATIO_SMALL = 1.384 / 1.400
ATTN_TRAFFIC_RATIO_LARGE = 4.847 / 2.026


def attn_traffic(nbytes, n_keys):
    return nbytes * (ATTN_TRAFFIC_RATIO_LARGE if n_keys > 100_000 else ATTN_TRAFFIC_RATIO_SMALL)
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
    from gpa_vggt_b200.nvtx import nvtx
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        taps, psi = model.aggregator(images)
        with nvtx("camera_head"):
            pose = model.camera_head(taps, shard=model.aggregator.shard)[-1]
        with nvtx("depth_head"):
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
# CPU baseline: the reference's own CPU path on the host cores
# ----------------------------------------------------------------------------
def cpu_reference(S, vanilla=False, reps=3):
    """(ms per forward, kind, sample note, extrapolated) of the reference's CPU
    forward at S frames (oracle/reference_runs.py): the reference's own modules
    from baseline/_ref when installed (kind "reference"), else the port.  At
    S <= 10 the whole forward runs; above, its pieces are timed on bounded
    samples and composed by the block schedule."""
    import torch
    from oracle import reference_runs as RR
    torch.set_num_threads(os.cpu_count() or 1)
    if not RR.have_reference():
        return RR.port_forward_ms(S, vanilla), "port", RR.port_sample_note(S, vanilla), True
    if S <= 10:
        model = RR.build_cpu_model(vanilla)
        RR.forward_ms(model, S)            # warm-up
        ms = statistics.median(RR.forward_ms(model, S) for _ in range(reps))
        return ms, "reference", (f"the reference's whole fp32 forward at S={S} (baseline/_ref, "
                                 f"aggregator + camera + DPT heads)"), False
    comp = RR.Composer(S, vanilla)
    ms = statistics.median(comp.compose_ms(comp.parts(reps=2)) for _ in range(reps))
    return ms, "reference", RR.composed_sample_note(S, vanilla), True


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
        # the reference's CPU path on the host cores (rank 0 only); a step is
        # one run of the reference's forward at S <= 10, else one bounded sample
        # of every piece of the S=200 forward, composed into its time
        if rank != 0:
            return
        import torch
        from oracle import reference_runs as RR
        torch.set_num_threads(os.cpu_count() or 1)
        if not fwd:
            print(json.dumps(dict(base, impl="reference", unavailable=(
                "the merged_block workload has no reference arm; use --workload forward"))), flush=True)
            return
        have = RR.have_reference()
        kind = "reference" if have else "port"
        direct = have and S <= 10
        if direct:
            model = RR.build_cpu_model(args.vanilla)
            one = lambda: RR.forward_ms(model, S)  # noqa: E731
            sample = f"the reference's whole fp32 forward at S={S} (baseline/_ref)"
        elif have:
            comp = RR.Composer(S, args.vanilla)
            one = lambda: comp.compose_ms(comp.parts(reps=2))  # noqa: E731
            sample = RR.composed_sample_note(S, args.vanilla)
        else:
            one = lambda: RR.port_forward_ms(S, args.vanilla)  # noqa: E731
            sample = RR.port_sample_note(S, args.vanilla)
        for _ in range(args.warmup):
            one()
        vals, walls = [], []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            vals.append(one())
            walls.append((time.perf_counter() - t0) * 1e3)
        ms = statistics.median(vals)
        step_ms = statistics.mean(walls)
        spread = (max(vals) - min(vals)) / ms if ms else 0.0
        cores = torch.get_num_threads()
        line = dict(base, impl="reference", value=ms, ms_per_step=step_ms, dtype="fp32",
                    extrapolated=not direct,
                    step=("one whole forward" if direct else
                          "one bounded sample of every piece of the forward, timed and composed "
                          "into value (ms_per_step is the sample's own wall time)"),
                    steps_values_ms={"median": ms, "min": min(vals), "max": max(vals),
                                     "spread": spread},
                    cpu_baseline={"value": ms, "unit": "ms", "cores": cores, "kind": kind,
                                  "sample": sample},
                    e2e={"value": ms, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
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
    from gpa_vggt_b200 import nvtx as _nv
    if _nv.TIMING:
        _nv.block_times(reset=True)   # drop the warm-up steps' ranges
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
    if _nv.TIMING:   # per-range device ms of the timed steps, grouped by kind
        bt = _nv.block_times()
        kinds = {}
        for name, v in bt.items():
            k = ("global_" + name.split("_", 3)[-1]) if name.startswith("global_block") else (
                "frame_block" if name.startswith("frame_block") else name)
            kinds[k] = kinds.get(k, 0.0) + v / args.steps
        print(json.dumps({"rank": rank, "block_ms_per_step": kinds}), file=sys.stderr, flush=True)
    timing, kernels.ATTN_TIMING = kernels.ATTN_TIMING, None
    ms = start.elapsed_time(stop) / args.steps
    attn_ms = sum(rec[0].elapsed_time(rec[1]) for rec in timing) / args.steps
    attn_flops = sum(rec[2] for rec in timing) / args.steps
    attn_bytes = sum(rec[3] for rec in timing) / args.steps
    attn_traffic_bytes = sum(attn_traffic(rec[3], rec[4]) for rec in timing) / args.steps
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
    roof = {"kernel": "attention kernels (gpa_attention_keybias: attn_kernel, and attn_persistent_kernel "
                      "for short key sequences), all launches of a step",
            "bound": "tensor", "achieved": achieved, "peak": pk["bf16_sus"], "unit": "TFLOP/s",
            "frac": achieved / pk["bf16_sus"], "peak_kind": f"{pk['src']} sustained bf16 (long step)",
            "frac_of_burst": achieved / pk["bf16"], "flops_per_step": attn_flops,
            "launches_per_step": n_attn, "ms_per_step": attn_ms,
            "share_of_step": attn_ms / ms,
            # DRAM bytes per step: each launch's algorithmic q/k/v/o bytes times the
            # ncu-measured DRAM/algorithmic ratio of its shape (attn_traffic)
            "traffic": attn_traffic_bytes, "traffic_unit": "bytes per step",
            "algorithmic_bytes_per_step": attn_bytes}
    line = dict(base, value=ms, ms_per_step=ms, gpu_launches=launches, roofline=roof, e2e=e2e,
                clocks=clk.summary())
    if fwd:
        line["frames_per_s"] = S / (ms / 1e3)
        line["gpu_memory_peak_gib"] = torch.cuda.max_memory_allocated(dev) / 2 ** 30
    if world == 1 and not args.no_cpu and fwd:   # the CPU baseline is an N=1 figure
        cms, kind, sample, extra = cpu_reference(S, args.vanilla)
        line["cpu_baseline"] = {"value": cms, "unit": "ms", "cores": torch.get_num_threads(),
                                "kind": kind, "sample": sample, "extrapolated": extra}
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
