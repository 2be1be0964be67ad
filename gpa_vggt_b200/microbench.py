"""Kernel microbenchmarks (one JSON line per case), each against its roofline.

    python -m gpa_vggt_b200.microbench attn  --lq 274800 --lk 66845 [--heads 16] [--no-bias] [--batch 1]
    python -m gpa_vggt_b200.microbench sim   --m 131072 --n 131072 [--d 128]
    python -m gpa_vggt_b200.microbench merge --frames 200 [--ratio 0.98]
    python -m gpa_vggt_b200.microbench pool  --frames 200
    python -m gpa_vggt_b200.microbench sweep            # the three kernel sweeps

Inputs are seeded N(0,1) (bias = log(1 + Poisson(1)) per key).  Times are
CUDA-event averages over --iters launches after --warmup launches on the
current stream; inputs are larger than L2 for the full-size cases.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

from . import kernels, _lib

ROOT = Path(__file__).resolve().parents[1]
P_TOK = 37 * 37 + 5


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


LAST_CLOCKS: dict = {}


def _sm_clock_sampler(stop, out):
    """Median SM clock (MHz) of the current GPU while `stop` is unset (NVML)."""
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(torch.cuda.current_device())
        vals = []
        while not stop.is_set():
            vals.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
            stop.wait(0.005)
        if vals:
            vals.sort()
            out["sm_mhz"] = vals[len(vals) // 2]
            out["samples"] = len(vals)
    except Exception as e:  # no NVML: report the reason, timing is unaffected
        out["error"] = str(e)[:80]


def timed(fn, iters, warmup):
    import threading
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    stop, clk = threading.Event(), {}
    th = threading.Thread(target=_sm_clock_sampler, args=(stop, clk), daemon=True)
    th.start()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    stop.set()
    th.join()
    LAST_CLOCKS.clear()
    LAST_CLOCKS.update(clk)
    return a.elapsed_time(b) / iters


def merged_len(S, ratio=0.98):
    nd = P_TOK + (S - 1) * 329
    ns = S * P_TOK - nd
    r = int(S * P_TOK * ratio)
    return nd if r >= ns else ns - r + nd


def bench_attn(lq, lk, heads=16, bias=True, iters=5, warmup=2, seed=0, batch=1):
    """batch > 1: independent sequences (e.g. the frame attention, one per frame)."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(batch, heads, lq, 64, device=dev, generator=g).bfloat16()
    k = torch.randn(batch, heads, lk, 64, device=dev, generator=g).bfloat16()
    v = torch.randn(batch, heads, lk, 64, device=dev, generator=g).bfloat16()
    b = ((1 + torch.poisson(torch.ones(batch, 1, lk, device=dev), generator=g)).log().expand(batch, heads, lk)
         if bias else None)
    out = torch.empty_like(q)
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    ms = timed(lambda: kernels.attention(q, k, v, b, 0.125, out=out, status=status), iters, warmup)
    flops = 4.0 * batch * lq * lk * 64 * heads
    _, peak, src = peaks()
    tf = flops / ms / 1e9
    return {"kernel": "attention", "batch": batch, "lq": lq, "lk": lk, "heads": heads, "bias": bias, "ms": ms,
            "tflops": tf, "peak_tflops": peak, "frac": tf / peak, "peak_src": src,
            "status": int(status.item()), "clocks": dict(LAST_CLOCKS)}


def bench_sim(m, n, d=128, iters=5, warmup=2, seed=0):
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    a = torch.randn(1, m, d, device=dev, generator=g)
    a = (a / a.norm(dim=-1, keepdim=True)).bfloat16()
    b = torch.randn(1, n, d, device=dev, generator=g)
    b = (b / b.norm(dim=-1, keepdim=True)).bfloat16()
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    ms = timed(lambda: kernels.sim_argmax(a, b, status=status), iters, warmup)
    flops = 2.0 * m * n * d
    _, peak, src = peaks()
    tf = flops / ms / 1e9
    return {"kernel": "sim_argmax", "m": m, "n": n, "d": d, "ms": ms, "tflops": tf,
            "peak_tflops": peak, "frac": tf / peak, "peak_src": src, "status": int(status.item())}


def bench_merge(frames, ratio=0.98, iters=5, warmup=2, seed=0):
    """K and V scatter-mean at the S-frame split (real roles, random matches)."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    S = frames
    N = S * P_TOK
    rand = torch.randint(4, (S - 1, 18, 18), device=dev, generator=g)
    dst, src, _ = kernels.merge_roles(rand, S, 37, 37, 2, 2, 5, False, dev)
    nm = torch.rand(src.numel(), device=dev, generator=g)
    ni = torch.randint(0, dst.numel(), (src.numel(),), device=dev, generator=g).int()
    plan = kernels.merge_plan(nm, ni, int(N * ratio), dst, src)
    kv = torch.randn(N, 2, 16, 64, device=dev, generator=g).bfloat16()
    out = torch.empty(plan.n_out, 2, 16, 64, device=dev, dtype=torch.bfloat16)

    def run():
        kernels.merge_kv(kv[:, 0].transpose(0, 1), plan, out=out[:, 0].transpose(0, 1))
        kernels.merge_kv(kv[:, 1].transpose(0, 1), plan, out=out[:, 1].transpose(0, 1))

    ms = timed(run, iters, warmup)
    plan_ms = timed(lambda: kernels.merge_plan(nm, ni, int(N * ratio), dst, src), iters, warmup)
    nbytes = 2 * N * 1024 * 2 + 2 * plan.n_out * 1024 * 2 + N * 8
    hbm, _, src_ = peaks()
    gbs = nbytes / ms / 1e6
    return {"kernel": "merge_kv (K+V)", "frames": S, "n_out": plan.n_out, "ms": ms,
            "plan_ms": plan_ms, "bytes": nbytes, "gbs": gbs, "peak_gbs": hbm, "frac": gbs / hbm,
            "peak_src": src_}


def bench_pool(frames, iters=5, warmup=2, seed=0):
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    N = frames * P_TOK
    k = torch.randn(16, N, 64, device=dev, generator=g).bfloat16()
    v = torch.randn(16, N, 64, device=dev, generator=g).bfloat16()
    ms = timed(lambda: kernels.frame_pool(k, v, frames, 37, 37, 5, 8), iters, warmup)
    nbytes = 2 * 16 * frames * 1369 * 64 * 2
    hbm, _, src = peaks()
    return {"kernel": "frame_pool", "frames": frames, "ms": ms, "gbs": nbytes / ms / 1e6,
            "frac": nbytes / ms / 1e6 / hbm, "peak_src": src}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("what", choices=["attn", "sim", "merge", "pool", "sweep"])
    ap.add_argument("--lq", type=int, default=200 * P_TOK)
    ap.add_argument("--lk", type=int, default=merged_len(200))
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--no-bias", action="store_true")
    ap.add_argument("--m", type=int, default=131072)
    ap.add_argument("--n", type=int, default=131072)
    ap.add_argument("--d", type=int, default=128)
    ap.add_argument("--frames", type=int, default=200)
    ap.add_argument("--ratio", type=float, default=0.98)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    a = ap.parse_args(argv)
    _lib.load()
    rows = []
    if a.what == "attn":
        rows.append(bench_attn(a.lq, a.lk, a.heads, not a.no_bias, a.iters, a.warmup, batch=a.batch))
    elif a.what == "sim":
        rows.append(bench_sim(a.m, a.n, a.d, a.iters, a.warmup))
    elif a.what == "merge":
        rows.append(bench_merge(a.frames, a.ratio, a.iters, a.warmup))
    elif a.what == "pool":
        rows.append(bench_pool(a.frames, a.iters, a.warmup))
    else:
        for n in (4096, 32768, 131072):
            rows.append(bench_sim(n, n, 128, a.iters, a.warmup))
        rows.append(bench_merge(200, 0.98, a.iters, a.warmup))
        for S in (50, 200, 500):
            rows.append(bench_attn(S * P_TOK, merged_len(S), 16, True, a.iters, a.warmup))
    for r in rows:
        print(json.dumps(r), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
