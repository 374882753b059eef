"""A rank that leaves a row-sharded run: the others learn of it through the
process group and end with an error instead of waiting for ever.

Three gloo ranks gather row slices with RowGather (the exchange of the
row-sharded path).  After one good exchange, rank 2 leaves between steps, as a
rank of a GPU run would: no collective of its own is in flight.  Ranks 0 and 1
enter the next exchange; its collective cannot complete, and the process
group's short timeout (or the closed connection) ends it with an exception
that each surviving rank catches and reports.
"""

import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from deepfold.model.kernels.sinkhorn_rowshard import RowGather


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out, took):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    N = 12
    g = RowGather(N)
    x = torch.zeros(2, N)
    x[:, g.r0:g.r1] = rank + 1.0
    g(x)  # one good exchange
    out[rank] = 1 if bool((x > 0).all()) else -1
    if rank == world - 1:
        os._exit(0)  # leaves between steps, without tearing down its process group
    t0 = time.monotonic()
    try:
        g(torch.zeros(2, N))
        out[rank] = 3  # the exchange completed without the departed rank: wrong
    except Exception:  # noqa: BLE001 -- gloo raises RuntimeError (timeout or closed connection)
        out[rank] = 2
    took[rank] = time.monotonic() - t0
    os._exit(0)


@pytest.mark.timeout(120)
def test_departed_rank_ends_the_exchange_with_an_error():
    world = 3
    ctx = mp.get_context("spawn")
    out = ctx.Array("i", [0] * world)
    took = ctx.Array("d", [0.0] * world)
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out, took)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
        assert p.exitcode == 0
    assert list(out) == [2, 2, 1]
    assert max(took[:2]) < 60.0
