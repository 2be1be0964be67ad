"""Rank failure between steps, on the host (gloo, two CPU ranks).

Rank 1 runs one exchange step of a frame shard (the per-block all-gather the
sharded forward uses), then raises and leaves the process group between
steps.  Rank 0 goes on to the next step's exchange; with the short process-
group timeout the collective ends with an error on rank 0 instead of waiting
for good.  Rank 0 records what it saw and how long it waited.
"""
import datetime
import json
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

TIMEOUT_S = 5


def _worker(rank, world, port, tmpdir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=TIMEOUT_S))
    from gpa_vggt_b200.vggt.shard import FrameShard
    sh = FrameShard(4)
    first = sh.gather(torch.full((2, 3), float(rank)))            # step 1: both ranks
    if rank == 1:
        # fails between steps: no kernel or collective of it is in flight
        with open(os.path.join(tmpdir, "r1.json"), "w") as f:
            json.dump({"step1": first[:, 0].tolist()}, f)
        os._exit(3)
    t0 = time.time()
    err = None
    try:
        sh.gather(torch.full((2, 3), float(rank)))                # step 2: the peer is gone
    except Exception as e:                                        # noqa: BLE001
        err = f"{type(e).__name__}: {e}"
    with open(os.path.join(tmpdir, "r0.json"), "w") as f:
        json.dump({"step1": first[:, 0].tolist(), "error": err, "waited_s": time.time() - t0}, f)
    os._exit(0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_peer_failure_between_steps_surfaces_as_an_error(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert procs[1].exitcode == 3
    r0 = json.loads((tmp_path / "r0.json").read_text())
    r1 = json.loads((tmp_path / "r1.json").read_text())
    assert r0["step1"] == [0.0, 0.0, 1.0, 1.0] and r1["step1"] == r0["step1"]
    assert r0["error"] is not None, "the second step's exchange completed without the peer"
    assert r0["waited_s"] < 10 * TIMEOUT_S
