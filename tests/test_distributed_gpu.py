"""Block-row-sharded Jacobi-PCG on 2 GPUs (NCCL) against the single-GPU solve.

Runs as two spawned processes, one per GPU; skipped with fewer than 2 GPUs.
Tolerance: 1e-5 relative Frobenius error on the assembled solution.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, cases, out, transport="nccl"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        import trnsparse_b200 as ts
        from trnsparse_b200 import distributed as D, workloads as w

        for ci, (nbr, tol, max_iter) in enumerate(cases):
            A, b = w.block_pentadiagonal_spd(nbr)
            sh = D.shard_bsr(A, rank, world)
            bl = b[sh.r0 * 128 : sh.r1 * 128].cuda()
            cg = D.ShardedCG(sh, bl, tol=tol, max_iter=max_iter, transport=transport, graph=(transport != "nccl"))
            x, it, rel = cg.run()
            x2, it2, rel2 = cg.run()  # a second solve on the same buffers gives the same answer
            assert (torch.linalg.norm(x - x2) / torch.linalg.norm(x)).item() <= 1e-6 and it == it2
            cg.close()
            parts = [torch.zeros(D.shard_bsr(A, q, world).n_own, device="cuda") for q in range(world)]
            dist.all_gather(parts, x)
            if rank == 0:
                xg = torch.cat(parts)
                xr, itr, relr = ts.cg_bsr(A, b.cuda(), tol=tol, max_iter=max_iter, M=ts.jacobi_preconditioner_bsr(A))
                err = (torch.linalg.norm(xg - xr) / torch.linalg.norm(xr)).item()
                out[ci] = (err, it, itr, rel, relr)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["nccl", "peer", "fused", "coop"])
def test_sharded_cg_two_gpus(transport):
    cases = [(64, 0.0, 30), (96, 1e-6, 100)] if transport == "nccl" else [(64, 0.0, 30), (96, 0.0, 40)]
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    mp.start_processes(_worker, args=(2, _free_port(), cases, out, transport), nprocs=2, start_method="spawn",
                       join=True)
    for ci in range(len(cases)):
        err, it, itr, rel, relr = out[ci]
        assert err <= 1e-5, out[ci]
        assert abs(it - itr) <= 1, out[ci]
