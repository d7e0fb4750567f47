"""Block-row-sharded Jacobi-PCG on 1 and 2 GPUs against the single-GPU solve.

Runs as spawned processes, one per GPU; the 2-GPU cases are skipped with
fewer than 2 GPUs.
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
    """A port that binds now, drawn at random from a high range (an ephemeral port the
    OS just handed to the previous test's store can still be in TIME_WAIT)."""
    import random

    for _ in range(100):
        p = random.randint(20000, 60000)
        s = socket.socket()
        try:
            s.bind(("127.0.0.1", p))
            return p
        except OSError:
            continue
        finally:
            s.close()
    raise RuntimeError("no free port")


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
            cg = D.ShardedCG(sh, bl, tol=tol, max_iter=max_iter, transport=transport,
                             graph=(transport != "nccl" and tol <= 0))
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


@pytest.mark.parametrize("world", [1, 2])
@pytest.mark.parametrize("transport", ["nccl", "peer", "fused", "coop", "cgcg"])
def test_sharded_cg(transport, world):
    """world 1 runs the same sharded machinery (own flags, no halo) on one GPU."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cases = [(64, 0.0, 30), (96, 1e-6, 100)] if transport == "nccl" else [(64, 0.0, 30), (96, 0.0, 40)]
    if transport == "cgcg":
        cases.append((80, 1e-6, 100))  # converges before max_iter: the tolerance exit
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), cases, out, transport), nprocs=world,
                       start_method="spawn", join=True)
    for ci in range(len(cases)):
        err, it, itr, rel, relr = out[ci]
        assert err <= 1e-5, out[ci]
        assert abs(it - itr) <= 1, out[ci]


def test_cgcg_peer_timeout_is_reported():
    """A rank whose peer never answers: one process runs the one-reduction solver as
    rank 0 of a world of 2 whose "peer" buffer is its own, so rank 1's flags are never
    raised. The bounded wait gives up (10 s), the solve ends with the peer-timeout
    status and the device error word says why; no GPU fault, the context stays usable."""
    import ctypes

    import trnsparse_b200 as ts
    from trnsparse_b200 import _lib
    from trnsparse_b200 import workloads as w
    from trnsparse_b200.ops import _bsr_geometry

    dev = torch.device("cuda", 0)
    A, b = w.block_pentadiagonal_spd(8)
    n = A.shape[0]
    geo = _bsr_geometry(A, dev)
    ws_bytes = _lib.raw("trnsparse_bsr_cgcg_workspace_size")(n, 5)
    comm_off = (ws_bytes + 255) // 256 * 256
    buf = torch.zeros(comm_off + _lib.raw("trnsparse_peer_comm_bytes")(2), dtype=torch.uint8, device=dev)
    peers = torch.tensor([buf.data_ptr(), buf.data_ptr()], dtype=torch.int64, device=dev)
    sends = torch.zeros(3, dtype=torch.int64, device=dev)
    x = torch.zeros(n, device=dev)
    bd = b.to(dev)
    _lib.device_error()  # start clean
    _lib.call("trnsparse_bsr_cgcg_solve", *geo, bd.data_ptr(), x.data_ptr(), None, 0.0, 5, n, buf.data_ptr(), 0,
              ws_bytes, peers.data_ptr(), 2, 0, comm_off, sends.data_ptr(), 0, _lib.stream_handle(dev))
    torch.cuda.synchronize()
    head = buf[:64].cpu()
    assert head[0:4].view(torch.int32).item() == 1  # done
    assert head[8:12].view(torch.int32).item() == 5  # REASON_PEER_TIMEOUT
    assert _lib.device_error() == 3  # DEVERR_PEER_TIMEOUT (read and cleared)
    # the context is still usable
    y = ts.bsr_spmm(A, bd.unsqueeze(1))
    assert torch.isfinite(y).all()


def _worker_fixed(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        import trnsparse_b200 as ts
        from trnsparse_b200 import distributed as D, workloads as w

        A, b = w.block_pentadiagonal_spd(48)
        sh = D.shard_bsr(A, rank, world)
        bl = b[sh.r0 * 128 : sh.r1 * 128].cuda()
        v0 = torch.randn(A.shape[0], generator=torch.Generator().manual_seed(7))
        res = {}
        for name, run_sh, run_1 in [
            ("cheb", lambda: D.chebyshev_bsr_sharded(sh, bl, 4.0, 16.0, K=20),
             lambda: ts.chebyshev_bsr(A, b.cuda(), 4.0, 16.0, K=20)),
            ("rich", lambda: D.richardson_bsr_sharded(sh, bl, 0.09, K=15),
             lambda: ts.richardson_bsr(A, b.cuda(), 0.09, K=15)),
        ]:
            x, K, rel = run_sh()
            parts = [torch.zeros(D.shard_bsr(A, q, world).n_own, device="cuda") for q in range(world)]
            dist.all_gather(parts, x.contiguous())
            xr, Kr, relr = run_1()
            res[name] = ((torch.linalg.norm(torch.cat(parts) - xr) / torch.linalg.norm(xr)).item(), K, Kr, rel, relr)
        lam, v, it = D.power_iteration_bsr_sharded(sh, v0[sh.r0 * 128 : sh.r1 * 128].cuda(), max_iter=60, tol=1e-6)
        parts = [torch.zeros(D.shard_bsr(A, q, world).n_own, device="cuda") for q in range(world)]
        dist.all_gather(parts, v.contiguous())
        lr, vr, itr = ts.power_iteration_bsr(A, v0.cuda(), max_iter=60, tol=1e-6)
        res["power"] = ((torch.linalg.norm(torch.cat(parts) - vr) / torch.linalg.norm(vr)).item(), it, itr, lam, lr)
        if rank == 0:
            out.update(res)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2])
def test_sharded_chebyshev_richardson_power(world):
    """Block-row-sharded fixed-step solvers and power iteration against the single-GPU
    ones (1e-5 relative on the solution / eigenvector, identical step counts)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    mp.start_processes(_worker_fixed, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    for name in ("cheb", "rich"):
        err, K, Kr, rel, relr = out[name]
        assert err <= 1e-5 and K == Kr and abs(rel - relr) <= 1e-4 * max(relr, 1e-12) + 1e-7, (name, out[name])
    err, it, itr, lam, lr = out["power"]
    assert err <= 1e-4 and abs(it - itr) <= 1 and abs(lam - lr) <= 1e-5 * abs(lr), out["power"]
