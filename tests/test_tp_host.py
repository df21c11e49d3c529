"""Host side of the multi-GPU path on CPU: two gloo ranks exchange the NCCL
unique id the way bench.py and tests/tp_check.py do, and reduce per-rank step
times to their maximum (the bench reports the slowest rank)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from prana_b200 import _ffi
from prana_b200 import build as pbuild


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from prana_b200 import model as pm

        uid = [pm.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        gathered = [None] * world
        dist.all_gather_object(gathered, uid[0])
        t = torch.tensor([1.5 + rank, 10.0 - rank])  # this rank's (step ms, e2e ms)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        q.put((rank, len(uid[0]), all(g == gathered[0] for g in gathered), t.tolist()))
    finally:
        dist.destroy_process_group()


def test_two_ranks_share_one_nccl_id_and_reduce_to_the_slowest():
    if not _ffi.LIB_PATH.exists():
        pbuild.build_all()
    try:
        from prana_b200 import model as pm

        pm.tp_unique_id()
    except Exception as e:  # no libnccl on this host
        pytest.skip(f"NCCL unavailable: {e}")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, n, same, t in out:
        assert n == 128 and same
        assert t == [2.5, 10.0]
