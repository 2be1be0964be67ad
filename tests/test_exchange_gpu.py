"""The merged-block K/V exchange of the frame-sharded forward on 2 GPUs.

Through peer memory (gpa_merge_exchange_p2p over CUDA IPC, one kernel per rank)
and through NCCL (all-to-all, merge, all-gather: merge_exchange), every rank's
merged rows must equal, bit for bit, merge_kv of all tokens on one GPU (the
reference's merge.heads, merging/merge.py:234-250), for bf16 and fp32 rows, at
merge ratios 0.98 and 0.2 and with a hub dst.  A plan holding a token outside
every rank's rows is skipped by the kernel and flagged in the status word (bit
2) instead of faulting; the next exchange on the same GPUs is exact again."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]

S, W, HH, NSP, HEADS, D = 4, 37, 37, 5, 16, 64
P = W * HH + NSP
N = S * P
CASES = [(0.98, torch.bfloat16, False), (0.2, torch.bfloat16, False), (0.98, torch.float32, True)]


def _case(ratio, dtype, hub, dev):
    """Tokens, positions and plan, identical on every rank (CPU generator)."""
    from gpa_vggt_b200 import kernels
    from oracle import gpa_oracle as O
    g = torch.Generator().manual_seed(int(ratio * 100) + (7 if hub else 0))
    rand = torch.randint(4, size=(S - 1, HH // 2, W // 2), generator=g)
    dst, src = O.split_positions(O.dst_mask(S, W, HH, 2, 2, NSP, rand))
    node_max = torch.rand(src.numel(), generator=g)
    node_idx = torch.randint(0, dst.numel(), (src.numel(),), generator=g)
    if hub:
        node_idx[::10] = 7
    k = torch.randn(N, HEADS, D, generator=g).to(dtype)
    v = torch.randn(N, HEADS, D, generator=g).to(dtype)
    plan = kernels.merge_plan(node_max.to(dev), node_idx.int().to(dev), int(N * ratio),
                              dst.int().to(dev), src.int().to(dev))
    return k.to(dev), v.to(dev), plan


def _worker(rank, world, port, outdir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from gpa_vggt_b200 import kernels
    from gpa_vggt_b200.vggt.shard import FrameShard, merge_exchange, merge_exchange_p2p
    dev = torch.device("cuda", rank)
    sh = FrameShard(S)
    dpf = NSP + (HH // 2) * (W // 2)
    d_range = sh.role_ranges(P, dpf)[rank][0]
    lo, hi = sh.f0 * P, sh.f1 * P
    res = {}
    for ratio, dtype, hub in CASES:
        k, v, plan = _case(ratio, dtype, hub, dev)
        want_k = kernels.merge_kv(k.transpose(0, 1), plan).transpose(0, 1)     # [N_m, H, D]
        want_v = kernels.merge_kv(v.transpose(0, 1), plan).transpose(0, 1)
        got = merge_exchange_p2p(sh, k[lo:hi], v[lo:hi], plan, P, d_range, kernels)
        got = got.view(plan.n_out, 2, HEADS, D)
        p2p_ok = bool(torch.equal(got[:, 0], want_k) and torch.equal(got[:, 1], want_v))
        rows = torch.stack((k[lo:hi], v[lo:hi]), 1).reshape(hi - lo, 2 * HEADS * D)
        nccl = merge_exchange(sh, rows, plan, P, kernels).view(plan.n_out, 2, HEADS, D)
        nccl_ok = bool(torch.equal(nccl[:, 0], want_k) and torch.equal(nccl[:, 1], want_v))
        res[f"{ratio}-{dtype}-{hub}"] = (p2p_ok, nccl_ok, plan.n_out)
    # a member token outside every rank's rows: skipped and flagged, no fault
    k, v, plan = _case(0.98, torch.bfloat16, False, dev)
    bad_src = plan.src_pos.clone()
    bad_src[plan.seg_src[0].long()] = N + 5        # a member of dst slot 0 (rank 0's)
    bad = kernels.MergePlan(plan.num_src, plan.num_dst, plan.r, plan.dst_pos, bad_src, plan.unm_src,
                            plan.seg_start, plan.seg_src, plan.counts)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    pb = sh.peer_buffers((hi - lo) * 2 * HEADS * D * 2, N * 2 * HEADS * D * 2, dev)
    rows = pb.rows[: (hi - lo) * 2 * HEADS * D * 2].view(torch.bfloat16).view(hi - lo, 2, HEADS, D)
    torch.stack((k[lo:hi], v[lo:hi]), 1, out=rows)
    sh.device_barrier()
    kernels.merge_exchange_p2p(pb.peer_rows, pb.peer_out, rank, torch.bfloat16, sh.local * P,
                               2 * HEADS * D, bad, d_range[0], d_range[1], status=status)
    sh.device_barrier()
    flags = status.clone()
    dist.all_reduce(flags, op=dist.ReduceOp.MAX)
    res["bad_status"] = int(flags.item())
    got = merge_exchange_p2p(sh, k[lo:hi], v[lo:hi], plan, P, d_range, kernels).view(plan.n_out, 2, HEADS, D)
    want_k = kernels.merge_kv(k.transpose(0, 1), plan).transpose(0, 1)
    res["after_bad"] = bool(torch.equal(got[:, 0], want_k))
    torch.save(res, os.path.join(outdir, f"x{rank}.pt"))
    sh.peer_buffers(0, 0, dev).close()
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_merge_exchange_p2p_bit_identical(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    for r in range(world):
        res = torch.load(tmp_path / f"x{r}.pt")
        print(r, res)
        for key, val in res.items():
            if key == "bad_status":
                assert val & 2, "the out-of-range member was not flagged"
            elif key == "after_bad":
                assert val
            else:
                p2p_ok, nccl_ok, n_out = val
                assert p2p_ok, f"peer-memory exchange differs from one GPU's merge ({key})"
                assert nccl_ok, f"NCCL exchange differs from one GPU's merge ({key})"
