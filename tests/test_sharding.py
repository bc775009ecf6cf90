"""Multi-rank host logic on CPU with gloo (world size 2): utterance sharding
covers the batch exactly once, and a rank that fails before a collective is
detected by its peer through the process-group timeout instead of hanging.
No GPU is touched (failure is made on the host)."""
import os
import pathlib
import sys
from datetime import timedelta

import pytest
import torch.multiprocessing as mp

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _init(rank, world, port, timeout_s=30):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))
    return dist


def _shard_worker(rank, world, port, q):
    sys.path.insert(0, str(ROOT))
    from __graft_entry__ import load_package

    pkg = load_package()
    import bark3_b200.synthetic as syn

    dist = _init(rank, world, port)
    secs = syn.batch_lengths(5, 256)
    frames = [pkg.frames_for_seconds(s) for s in secs]
    rank_of = pkg.shard_lpt(frames, world)
    mine = [i for i in range(len(frames)) if rank_of[i] == rank]
    got = [None] * world
    dist.all_gather_object(got, mine)
    if rank == 0:
        q.put(got)
    dist.barrier()
    dist.destroy_process_group()


def _failing_worker(rank, world, port, q):
    dist = _init(rank, world, port, timeout_s=3)
    if rank == 1:
        # leaves between steps, before the next collective
        dist.destroy_process_group()
        return
    try:
        import torch

        t = torch.ones(1)
        dist.all_reduce(t)
        q.put("no-error")
    except Exception as e:  # noqa: BLE001 - the peer's failure must surface here
        q.put(type(e).__name__)


def _free_port():
    import socket

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_gloo_shards_cover_batch_once():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    flat = sorted(i for part in got for i in part)
    assert flat == list(range(256))
    assert set(got[0]).isdisjoint(got[1])


@pytest.mark.timeout(120)
def test_peer_failure_is_reported_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outcome = q.get(timeout=100)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert outcome != "no-error"
