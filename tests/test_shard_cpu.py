"""Query-frame sharding (gpa_vggt_b200/vggt/shard.py), checked on CPU with two
gloo ranks: a small VGGT (dim 128, 4 global blocks covering frame+shared,
merged and core-merged attention, 9x9 patch grid) run with its frames split
over the ranks must give the unsharded run's tokens and camera encoding.  The
kernel entry points are the oracle-backed CPU stand-ins (tests/cpu_kernels.py),
so the check is on the host logic: roles, gathers, plan, ordering."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

S, IMG = 4, 126          # 4 frames of 126x126 -> 9x9 patches
OUT = "shard_out_rank{}.pt"


def _model():
    from gpa_vggt_b200.vggt.model import VGGT, init_weights
    m = VGGT(img_size=518, embed_dim=128, merging=2, merge_end=3, merge_ratio=0.9,
             early_frame_split=1, broadcast_pool=4, core_blocks=(3,), core_merge_ratio=0.3,
             merge_metric_dim=64, enable_depth=False)
    agg = m.aggregator
    agg.depth = 4
    agg.tap_blocks = (0, 1, 2, 3)
    agg.frame_blocks = agg.frame_blocks[:4]
    agg.global_blocks = agg.global_blocks[:4]
    agg.patch_embed.blocks = agg.patch_embed.blocks[:2]
    init_weights(m, seed=1)
    m.eval()
    m.update_patch_dimensions(9, 9)
    return m


def _draws(C=128, dim=64):
    g = torch.Generator().manual_seed(33)
    rand_idx = torch.randint(4, size=(S - 1, 4, 4), generator=g)
    proj = torch.randn(C, dim, generator=torch.Generator().manual_seed(1234))
    return rand_idx, proj


def _run(model, images):
    with torch.no_grad():
        taps, _ = model.aggregator(images)
        pose = model.camera_head(taps, shard=model.aggregator.shard)[-1]
    return taps[-1], pose


class _Patch:
    def __init__(self):
        self.saved = []

    def __call__(self, obj, name, value):
        self.saved.append((obj, name, getattr(obj, name)))
        setattr(obj, name, value)

    def undo(self):
        for obj, name, value in reversed(self.saved):
            setattr(obj, name, value)


def _worker(rank, world, port, tmpdir, overlap=False):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import cpu_kernels
    from gpa_vggt_b200.vggt import layers
    from gpa_vggt_b200.vggt.shard import FrameShard
    cpu_kernels.install(setattr)
    layers.OVERLAP_GATHER = overlap
    model = _model()
    shard = FrameShard(S)
    model.set_shard(shard)
    for blk in model.aggregator.global_blocks:
        blk.attn.rng_override = _draws()
    images = torch.rand(1, S, 3, IMG, IMG, generator=torch.Generator().manual_seed(0))
    tap, pose = _run(model, images[:, shard.f0:shard.f1])
    torch.save({"tap": tap, "pose": pose, "f0": shard.f0, "f1": shard.f1},
               os.path.join(tmpdir, OUT.format(rank)))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("overlap", [False, True])
def test_frame_sharded_forward_matches_unsharded(tmp_path, overlap):
    """overlap: merged blocks attend to own and gathered merged keys as two
    partitions combined by log-sum-exp."""
    import cpu_kernels
    patch = _Patch()
    cpu_kernels.install(patch)
    try:
        model = _model()
        for blk in model.aggregator.global_blocks:
            blk.attn.rng_override = _draws()
        images = torch.rand(1, S, 3, IMG, IMG, generator=torch.Generator().manual_seed(0))
        ref_tap, ref_pose = _run(model, images)
    finally:
        patch.undo()
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), overlap), nprocs=world,
                       start_method="spawn")
    for r in range(world):
        got = torch.load(tmp_path / OUT.format(r))
        want = ref_tap[:, got["f0"]:got["f1"]]
        assert torch.allclose(got["tap"], want, atol=1e-4, rtol=1e-4), \
            float((got["tap"] - want).abs().max())
        assert torch.allclose(got["pose"], ref_pose, atol=1e-4, rtol=1e-4)


def _gather_worker(rank, world, port, tmpdir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from gpa_vggt_b200.vggt.shard import FrameShard
    sh = FrameShard(4)
    assert sh.kv_group is not None
    k = torch.full((3, 2, 4), float(rank), dtype=torch.float32)
    v = torch.full((3, 2, 4), 10.0 + rank, dtype=torch.bfloat16)
    # one exchange of a stacked [N, 2, ...] buffer, and two exchanges of mixed dtypes,
    # in flight together with a gather on the main communicator
    kv, w1 = sh.gather_async(torch.stack((k, v.float()), 1))
    kf, w2 = sh.gather_async(k)
    vf, w3 = sh.gather_async(v)
    small = sh.gather(torch.tensor([rank], dtype=torch.int64))
    for w in (w1, w2, w3):
        w.wait()
    torch.save({"kv": kv, "k": kf, "v": vf, "small": small}, os.path.join(tmpdir, f"g{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_gather_async_on_the_kv_communicator(tmp_path):
    world = 2
    mp.start_processes(_gather_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    for r in range(world):
        got = torch.load(tmp_path / f"g{r}.pt")
        assert got["small"].tolist() == [0, 1]
        assert got["k"].shape == (6, 2, 4) and got["v"].dtype == torch.bfloat16
        assert got["k"][:3].eq(0).all() and got["k"][3:].eq(1).all()
        assert got["v"][:3].float().eq(10).all() and got["v"][3:].float().eq(11).all()
        assert torch.equal(got["kv"][:, 0], got["k"]) and torch.equal(got["kv"][:, 1], got["v"].float())


def _exchange_worker(rank, world, port, tmpdir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import cpu_kernels
    from gpa_vggt_b200.vggt.shard import FrameShard, merge_exchange
    sh = FrameShard(4)
    plan, rows, P = _exchange_case()
    mine = rows[sh.f0 * P:sh.f1 * P]
    merged = merge_exchange(sh, mine, plan, P, cpu_kernels)
    torch.save(merged, os.path.join(tmpdir, f"x{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def _exchange_case(ratio=0.6):
    """A 4-frame 9x9 split, random matches across all frames (many member rows
    sit in other frames than their dst), rows of 16 features."""
    import cpu_kernels
    g = torch.Generator().manual_seed(21)
    P = 9 * 9 + 5
    rand = torch.randint(4, size=(3, 4, 4), generator=g)
    dst, src, _ = cpu_kernels.merge_roles(rand, 4, 9, 9, 2, 2, 5, False, "cpu")
    nm = torch.rand(src.numel(), generator=g)
    ni = torch.randint(0, dst.numel(), (src.numel(),), generator=g)
    plan = cpu_kernels.merge_plan(nm, ni, int(4 * P * ratio), dst, src)
    rows = torch.randn(4 * P, 16, generator=g)
    return plan, rows, P


@pytest.mark.parametrize("world", [2, 4])
def test_merge_exchange_matches_single_merge(tmp_path, world):
    """Every rank gets the merged rows of every slot, equal to merging all
    tokens on one rank (same plan, same summation order)."""
    import cpu_kernels
    plan, rows, P = _exchange_case()
    want = cpu_kernels.merge_kv(rows[None], plan)[0]          # one "head" of 16 features
    mp.start_processes(_exchange_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    for r in range(world):
        got = torch.load(tmp_path / f"x{r}.pt")
        assert got.shape == want.shape
        assert torch.allclose(got, want, atol=1e-6, rtol=1e-6)
