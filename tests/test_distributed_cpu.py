"""Host logic of the block-row-sharded solver on CPU: partition, halo maps and
the halo exchange, run as world_size-2 / 3 gloo process groups."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from trnsparse_b200 import distributed as D
from trnsparse_b200 import workloads as w


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_block_row_ranges():
    assert D.block_row_ranges(10, 3) == [(0, 4), (4, 7), (7, 10)]
    assert D.block_row_ranges(2048, 8)[-1] == (1792, 2048)


@pytest.mark.parametrize("world", [1, 2, 3])
def test_shards_reassemble_the_matrix(world):
    A, _ = w.block_pentadiagonal_spd(10, b=8)
    dense = A.to_dense()
    for r in range(world):
        sh = D.shard_bsr(A, r, world)
        loc = sh.local.to_dense()
        rows = slice(sh.r0 * 8, sh.r1 * 8)
        torch.testing.assert_close(loc[:, : sh.n_own], dense[rows, rows])
        for i, c in enumerate(sh.halo_blocks):
            torch.testing.assert_close(loc[:, sh.n_own + i * 8 : sh.n_own + (i + 1) * 8], dense[rows, c * 8 : (c + 1) * 8])
        # pentadiagonal: at most 2 halo block-rows on each side
        assert len(sh.halo_blocks) <= 4


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        A, _ = w.block_pentadiagonal_spd(9, b=4)
        sh = D.shard_bsr(A, rank, world)
        glob = torch.arange(A.shape[0], dtype=torch.float32) * 0.5 + 1.0
        vec = torch.full((sh.n_ext,), -7.0)
        vec[: sh.n_own] = glob[sh.r0 * 4 : sh.r1 * 4]
        D.halo_exchange(sh, vec)
        expect = torch.cat([glob[sh.r0 * 4 : sh.r1 * 4]] + [glob[c * 4 : (c + 1) * 4] for c in sh.halo_blocks])
        out[rank] = bool(torch.equal(vec, expect))
        # the local product over the extended vector equals the global product's rows
        y = sh.local.to_dense() @ vec
        ref = A.to_dense() @ glob
        out[world + rank] = bool(torch.allclose(y, ref[sh.r0 * 4 : sh.r1 * 4], atol=1e-5))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_halo_exchange_gloo(world):
    port = _free_port()
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, port, out), nprocs=world, start_method="spawn", join=True)
    assert all(out[i] for i in range(2 * world)), dict(out)
