"""Host-side logic of the row-sharded path on CPU: row ranges and the
all-gather of row slices, with world_size 2 and 3 over gloo."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from deepfold.model.kernels.sinkhorn_rowshard import RowGather, row_range


def test_row_ranges_cover_every_row_once():
    for N in (1, 7, 64, 1000, 8192):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                r0, r1, n_loc = row_range(N, world, r)
                assert 0 <= r0 <= r1 <= N and r1 - r0 <= n_loc
                seen.extend(range(r0, r1))
            assert seen == list(range(N))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, N, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = RowGather(N)
        full = torch.arange(3 * N * 2, dtype=torch.float32).view(3, N, 2)
        x = torch.full_like(full, -1.0)                 # only this rank's rows are valid
        x[:, g.r0:g.r1] = full[:, g.r0:g.r1]
        g(x)
        v = torch.full((3, N), -1.0)
        v[:, g.r0:g.r1] = full[:, g.r0:g.r1, 0]
        g(v)
        ok = torch.equal(x, full) and torch.equal(v, full[..., 0])
        out[rank] = 1 if ok else 0
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,N", [(2, 10), (3, 10), (2, 64)])
def test_row_gather_gloo(world, N):
    ctx = mp.get_context("spawn")
    out = ctx.Array("i", [0] * world)
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, N, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert list(out) == [1] * world


@pytest.mark.parametrize("N,world", [(8192, 8), (1000, 2), (1000, 3), (129, 2), (128, 4), (300, 8)])
def test_peer_arrivals_match_the_kernel_launch_grid(N, world):
    """The host's expected arrivals per half-update equal the row blocks every
    rank's launch covers (launch grid: P * ceil(rows / 128) blocks per rank)."""
    from deepfold.model.kernels.sinkhorn_rowshard import arrivals_per_half_update, row_range
    P = 5
    blocks = 0
    for r in range(world):
        r0, r1, _ = row_range(N, world, r)
        rows = r1 - r0
        blocks += P * ((rows + 127) // 128 if rows > 0 else 0)
    assert arrivals_per_half_update(P, N, world) == blocks
