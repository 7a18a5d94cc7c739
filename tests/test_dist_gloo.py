"""World-size-2 ``gloo`` runs of the multi-rank bench plumbing on CPU: shards
cover the batch exactly once, the timing reduction is the max over ranks, and
a rank that fails before joining makes the others' collective error out
within the process-group timeout instead of hanging."""

import os
import socket
from datetime import timedelta

import pytest
import torch.multiprocessing as mp

from hackathon_b200 import dist as D


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, mode):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    if mode == "fail" and rank == 1:
        q.put((rank, "raised"))
        raise SystemExit(3)  # never joins the group
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        total, start, count = D.rows_for("strong", 4096, world, rank)
        fake_ms = 10.0 + rank  # per-rank device time
        m = D.reduce_max(fake_ms)
        D.barrier()
        q.put((rank, (total, start, count, m)))
        dist.destroy_process_group()
    except Exception as e:  # the survivor reports instead of hanging
        q.put((rank, f"error:{type(e).__name__}"))


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung past the deadline")
    out = {}
    while not q.empty():
        r, v = q.get()
        out[r] = v
    return out, [p.exitcode for p in procs]


def test_two_rank_shards_and_max_timing():
    out, codes = _run("ok")
    assert codes == [0, 0]
    spans = sorted((v[1], v[1] + v[2]) for v in out.values())
    assert spans == [(0, 2048), (2048, 4096)]
    assert all(v[3] == 11.0 for v in out.values())  # max over ranks


def test_missing_rank_is_detected_not_hung():
    out, codes = _run("fail")
    assert codes[1] == 3
    assert out[0].startswith("error:")


def test_weak_and_uneven_shards():
    assert D.rows_for("weak", 256, 4, 3) == (1024, 768, 256)
    spans = [D.shard(10, 4, r) for r in range(4)]
    assert spans == [(0, 3), (3, 6), (6, 8), (8, 10)]
