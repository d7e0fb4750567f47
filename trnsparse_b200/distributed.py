"""Block-row-sharded BSR conjugate gradient over torch.distributed.

One process per GPU. The matrix's block-rows are split into contiguous,
equal ranges; a rank keeps the blocks of its rows with their column
indices remapped into an extended local index space: its own rows first,
then "halo" copies of the rows of other ranks that its blocks reference,
grouped by owning rank. Per CG iteration (the reference's loop,
trnsparse/iterative.py:53-126):

  1. fused SpMV kernel (p update + A p + partial p.Ap)      -> all_reduce(p.Ap)
  2. vector kernel (x, r update + partial r.r, r.z)         -> all_reduce(r.r, r.z)
  3. halo exchange of r (send/recv of the referenced boundary rows only)

The halo part of the direction p is recomputed locally from the exchanged r,
so one vector crosses the link per iteration. All ranks take the same
decisions (convergence, breakdown) because they see the same reduced scalars.
The host logic here (partition, halo maps, exchange) is device-agnostic and
is tested with the gloo backend on CPU; the kernels need the CUDA library.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from .formats import BSRMatrix


def block_row_ranges(n_block_rows: int, world: int) -> list[tuple[int, int]]:
    """Contiguous, near-equal block-row ranges, one per rank."""
    base, extra = divmod(n_block_rows, world)
    out, s = [], 0
    for r in range(world):
        e = s + base + (1 if r < extra else 0)
        out.append((s, e))
        s = e
    return out


@dataclass
class BSRShard:
    rank: int
    world: int
    block_size: int
    r0: int  # first owned block-row (global)
    r1: int  # one past the last owned block-row
    local: BSRMatrix  # (n_own*b) x (n_ext*b), columns remapped
    halo_blocks: list[int]  # global block index of each halo slot, grouped by owner
    recv_from: dict[int, tuple[int, int]]  # owner -> (first halo slot, count)
    send_to: dict[int, list[int]]  # peer -> owned local block-rows it needs, in its halo order
    _dev: dict = field(default_factory=dict, repr=False)

    @property
    def n_own(self) -> int:
        return (self.r1 - self.r0) * self.block_size

    @property
    def n_ext(self) -> int:
        return (self.r1 - self.r0 + len(self.halo_blocks)) * self.block_size


def _needs(A: BSRMatrix, lo: int, hi: int) -> list[int]:
    """Sorted global block-columns outside [lo, hi) referenced by rows [lo, hi)."""
    rp = A.block_row_ptrs.tolist()
    cols = A.block_col_indices[rp[lo] : rp[hi]].tolist()
    return sorted({c for c in cols if c < lo or c >= hi})


def shard_bsr(A: BSRMatrix, rank: int, world: int) -> BSRShard:
    """The rank's shard of a square BSR matrix (every rank calls this with the same A)."""
    b = A.block_size
    nbr = A.block_row_ptrs.shape[0] - 1
    assert A.shape[0] == A.shape[1] and A.shape[0] == nbr * b, "sharded solve needs a square, block-aligned matrix"
    ranges = block_row_ranges(nbr, world)
    owner = torch.empty(nbr, dtype=torch.long)
    for q, (lo, hi) in enumerate(ranges):
        owner[lo:hi] = q
    lo, hi = ranges[rank]
    need = _needs(A, lo, hi)
    need.sort(key=lambda c: (int(owner[c]), c))  # grouped by owner rank
    slot = {c: (hi - lo) + i for i, c in enumerate(need)}
    recv_from: dict[int, tuple[int, int]] = {}
    for i, c in enumerate(need):
        q = int(owner[c])
        s, n = recv_from.get(q, (i, 0))
        recv_from[q] = (s, n + 1)
    send_to: dict[int, list[int]] = {}
    for q, (qlo, qhi) in enumerate(ranges):
        if q == rank:
            continue
        theirs = [c for c in sorted(_needs(A, qlo, qhi), key=lambda c: (int(owner[c]), c)) if lo <= c < hi]
        if theirs:
            send_to[q] = [c - lo for c in theirs]
    rp = A.block_row_ptrs
    s0, s1 = int(rp[lo]), int(rp[hi])
    cols = A.block_col_indices[s0:s1].tolist()
    local_cols = torch.tensor([c - lo if lo <= c < hi else slot[c] for c in cols], dtype=torch.long)
    local = BSRMatrix(
        blocks=A.blocks[s0:s1],
        block_col_indices=local_cols,
        block_row_ptrs=(rp[lo : hi + 1] - rp[lo]).clone(),
        shape=((hi - lo) * b, (hi - lo + len(need)) * b),
        block_size=b,
    )
    return BSRShard(rank, world, b, lo, hi, local, need, recv_from, send_to)


def halo_exchange(shard: BSRShard, vec: torch.Tensor, group=None) -> None:
    """Fill vec[n_own:n_ext] with the owners' current values of the halo rows.

    ``vec`` is the rank's extended vector (own rows then halo rows, length
    n_ext). Only the referenced boundary block-rows travel.
    """
    b = shard.block_size
    ops = []
    key = ("send_idx", str(vec.device))
    if key not in shard._dev:  # built outside any graph capture: no host->device copies in the loop
        shard._dev[key] = {
            q: (rows[0], len(rows)) if rows == list(range(rows[0], rows[0] + len(rows)))
            else torch.tensor(rows, device=vec.device)
            for q, rows in shard.send_to.items()
        }
    for q, sel in sorted(shard._dev[key].items()):
        if isinstance(sel, tuple):  # consecutive block-rows: send a view, no copy
            buf = vec[sel[0] * b : (sel[0] + sel[1]) * b]
        else:
            buf = vec[: shard.n_own].view(-1, b).index_select(0, sel).reshape(-1).contiguous()
        ops.append(dist.P2POp(dist.isend, buf, q, group))
    for q, (s, n) in sorted(shard.recv_from.items()):
        dst = vec[shard.n_own + s * b : shard.n_own + (s + n) * b]
        ops.append(dist.P2POp(dist.irecv, dst, q, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


def _slot_view(ws: torch.Tensor, offs, k: int, first: int, count: int) -> torch.Tensor:
    o = offs[1] + 32 * k + 8 * first
    return ws[o : o + 8 * count].view(torch.float64)


class _RawDevice:
    """Zero-copy torch view of library-allocated device memory (CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


PEER_TRANSPORTS = ("peer", "fused", "coop", "cgcg")


class ShardedCG:
    """A prepared sharded Jacobi-PCG solve for one shard, right-hand side and
    iteration budget.

    transport="nccl": scalar all-reduces and halo exchanges are NCCL
    collectives / send-recv. transport="fused": the exchanges happen inside
    the two solver kernels of an iteration (see trnsparse_bsr_cg_fused_*);
    transport="coop": the same in one cooperative kernel for the whole solve
    (the peer flags double as the grid barrier between phases).
    transport="cgcg": one cooperative kernel for the whole solve with one
    exchange per iteration (Chronopoulos-Gear recurrences: the reference's
    iterates in exact arithmetic, half the synchronisations).
    transport="peer": the workspace lives in a CUDA
    IPC buffer every rank maps, and one single-CTA kernel per exchange pushes
    the halo rows and partial sums straight into the peers' memory over
    NVLink, raises a flag and waits for the peers' flags (bounded), replacing
    each NCCL call; the ranks must share one NVLink/NVSwitch box.

    ``run()`` performs the solve; with ``graph=True`` (fixed-iteration mode,
    ``tol <= 0``) the whole solve — setup kernels, every iteration's two
    kernels, the scalar all-reduces and the halo exchanges — is captured once
    into a CUDA graph and each ``run()`` is a single graph replay, so the host
    issues nothing per iteration.
    """

    def __init__(self, shard: BSRShard, b_local: torch.Tensor, tol: float = 1e-6, max_iter: int = 1000,
                 jacobi: bool = True, group=None, check_every: int = 16, graph: bool = False,
                 transport: str = "nccl"):
        from . import _lib
        from .iterative import bsr_diagonal
        from .ops import _bsr_geometry

        self._lib = _lib
        self.shard, self.tol, self.max_iter, self.group = shard, float(tol), max_iter, group
        self.check_every = check_every
        dev = b_local.device
        self.dev = dev
        n_own, n_ext = shard.n_own, shard.n_ext
        self.geo = _bsr_geometry(shard.local, dev)
        self.inv_d = None
        if jacobi:
            d = bsr_diagonal(shard.local).to(dev)
            if torch.any(d.abs() < 1e-15):
                raise ValueError("Jacobi preconditioner: diagonal has near-zero entries")
            self.inv_d = torch.zeros(n_ext, dtype=torch.float32, device=dev)
            self.inv_d[:n_own] = 1.0 / d.float()
            halo_exchange(shard, self.inv_d, group)
        self.b = b_local.to(dev, torch.float32).contiguous()
        self.x = torch.zeros(n_own, dtype=torch.float32, device=dev)
        self.transport = transport
        self._peer_ptrs: list[int] = []
        if transport == "cgcg":
            # one layout on every rank: vectors sized for the largest extended shard
            sizes = [None] * dist.get_world_size(group)
            dist.all_gather_object(sizes, n_ext, group=group)
            self.n_alloc = max(sizes)
            self.ws_bytes = _lib.raw("trnsparse_bsr_cgcg_workspace_size")(self.n_alloc, max_iter)
        else:
            self.ws_bytes = _lib.raw("trnsparse_bsr_cg_workspace_size")(n_ext, max_iter)
        if transport in PEER_TRANSPORTS:
            self._setup_peer(max_iter)
        elif transport == "nccl":
            self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)
        else:
            raise ValueError(f"transport must be one of 'nccl', {', '.join(map(repr, PEER_TRANSPORTS))}; "
                             f"got {transport!r}")
        offs = (ctypes.c_size_t * 9)()
        if transport == "cgcg":
            _lib.call("trnsparse_bsr_cgcg_layout", self.n_alloc, max_iter, offs)
        else:
            _lib.call("trnsparse_bsr_cg_layout", n_ext, max_iter, offs)
        self.offs = list(offs)
        self.r_vec = self.ws[offs[2] : offs[2] + 4 * n_ext].view(torch.float32)
        if transport in PEER_TRANSPORTS:
            self._build_sends(element_offsets=transport == "cgcg")
        self.graph = None
        if graph:
            if self.tol > 0:
                raise ValueError("graph mode runs a fixed number of iterations: use tol <= 0")
            torch.cuda.synchronize(dev)
            self._solve(check=False)  # warm-up (NCCL communicators, kernels)
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    self._solve(check=False)
            torch.cuda.synchronize(dev)
            self.graph = g

    # ------------------------------------------------------------ peer transport
    def _setup_peer(self, max_iter: int) -> None:
        lib = self._lib
        g = self.group
        self.world, self.rank = dist.get_world_size(g), dist.get_rank(g)
        mine = (self.ws_bytes + 255) // 256 * 256
        sizes = [None] * self.world
        dist.all_gather_object(sizes, mine, group=g)
        self.comm_off = max(sizes)
        total = self.comm_off + lib.raw("trnsparse_peer_comm_bytes")(self.world)
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        with torch.cuda.device(self.dev):
            lib.call("trnsparse_peer_alloc", total, ctypes.byref(ptr), handle)
        self._own_ptr = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=g)
        ptrs = []
        for q, h in enumerate(handles):
            if q == self.rank:
                ptrs.append(self._own_ptr)
                continue
            p = ctypes.c_void_p()
            hb = (ctypes.c_ubyte * 64).from_buffer_copy(h)
            with torch.cuda.device(self.dev):
                lib.call("trnsparse_peer_open", hb, ctypes.byref(p))
            ptrs.append(p.value)
            self._peer_ptrs.append(p.value)
        self.peers_dev = torch.tensor(ptrs, dtype=torch.int64, device=self.dev)
        self.ws = torch.as_tensor(_RawDevice(self._own_ptr, total), device=self.dev)[: self.ws_bytes]

    def _build_sends(self, element_offsets: bool = False) -> None:
        """Halo rows this rank pushes: (source element, destination rank, destination byte offset
        of the receiver's r) or, with ``element_offsets``, the destination element."""
        sh = self.shard
        info = (sh.n_own, 0 if element_offsets else self.offs[2], dict(sh.recv_from))
        infos = [None] * self.world
        dist.all_gather_object(infos, info, group=self.group)
        b = sh.block_size
        sends = []
        for q, rows in sorted(sh.send_to.items()):
            n_own_q, r_off_q, recv_q = infos[q]
            start, count = recv_q[self.rank]
            assert count == len(rows)
            for i, row in enumerate(rows):
                dst = n_own_q + (start + i) * b
                sends.append((row * b, q, dst if element_offsets else r_off_q + 4 * dst))
        self.n_sends = len(sends)
        self.sends_dev = torch.tensor(sends if sends else [(0, 0, 0)], dtype=torch.int64, device=self.dev)

    def _push(self, a_off: int | None, b_off: int | None, area: int, step: int, halo: bool) -> None:
        lib = self._lib
        base = self.ws.data_ptr()
        lib.call("trnsparse_peer_reduce_push", self.peers_dev.data_ptr(), self.world, self.rank, self.comm_off,
                 None if a_off is None else base + a_off, None if b_off is None else base + b_off, area,
                 2 * self.max_iter + 4, step, self.r_vec.data_ptr(), self.sends_dev.data_ptr(),
                 self.n_sends if halo else 0, self.shard.block_size, lib.stream_handle(self.dev))

    def close(self) -> None:
        """Release the peer mappings and the shared buffer (peer transport)."""
        if self.transport not in PEER_TRANSPORTS or not hasattr(self, "_own_ptr"):
            return
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.dev):
            for p in self._peer_ptrs:
                self._lib.call("trnsparse_peer_close", p)
            self._peer_ptrs = []
        dist.barrier(group=self.group)
        with torch.cuda.device(self.dev):
            self._lib.call("trnsparse_peer_free", self._own_ptr)
        del self._own_ptr

    def _solve(self, check: bool) -> None:
        if self.transport == "peer":
            return self._solve_peer()
        if self.transport in ("fused", "coop"):
            return self._solve_fused(coop=self.transport == "coop")
        if self.transport == "cgcg":
            return self._solve_cgcg()
        lib, sh, ws, offs, g = self._lib, self.shard, self.ws, self.offs, self.group
        s = lib.stream_handle(self.dev)
        n_own, n_ext = sh.n_own, sh.n_ext
        inv = lib.ptr(self.inv_d)
        self.x.zero_()
        lib.call("trnsparse_bsr_cg_dist_start", n_own, n_ext, self.b.data_ptr(), inv, self.max_iter,
                 ws.data_ptr(), self.ws_bytes, s)
        dist.all_reduce(ws[24:32].view(torch.float64), group=g)  # ||b||^2 in the status record
        dist.all_reduce(_slot_view(ws, offs, 0, 1, 1), group=g)  # r0.z0
        halo_exchange(sh, self.r_vec, g)
        for k in range(self.max_iter + 1):
            lib.call("trnsparse_bsr_cg_dist_phase", *self.geo, self.x.data_ptr(), inv, self.tol, self.max_iter, k, 0,
                     ws.data_ptr(), s)
            if k == self.max_iter:
                break
            dist.all_reduce(_slot_view(ws, offs, k, 0, 1), group=g)
            lib.call("trnsparse_bsr_cg_dist_phase", *self.geo, self.x.data_ptr(), inv, self.tol, self.max_iter, k, 1,
                     ws.data_ptr(), s)
            dist.all_reduce(_slot_view(ws, offs, k, 2, 2), group=g)
            halo_exchange(sh, self.r_vec, g)
            if check and self.tol > 0 and (k + 1) % self.check_every == 0 and int(ws[0:4].view(torch.int32).item()):
                break

    def _solve_peer(self) -> None:
        lib, sh, ws, offs = self._lib, self.shard, self.ws, self.offs
        s = lib.stream_handle(self.dev)
        inv = lib.ptr(self.inv_d)
        self.x.zero_()
        lib.call("trnsparse_peer_bump_epoch", self._own_ptr, self.comm_off, self.world, s)
        lib.call("trnsparse_bsr_cg_dist_start", sh.n_own, sh.n_ext, self.b.data_ptr(), inv, self.max_iter,
                 ws.data_ptr(), self.ws_bytes, s)
        slot = offs[1]
        self._push(24, slot + 8, 2, 0, True)  # ||b||^2, r0.z0, halo of r0 (area 2: setup only)
        for k in range(self.max_iter + 1):
            lib.call("trnsparse_bsr_cg_dist_phase", *self.geo, self.x.data_ptr(), inv, self.tol, self.max_iter, k, 0,
                     ws.data_ptr(), s)
            if k == self.max_iter:
                break
            self._push(slot + 32 * k, None, 0, 1 + 2 * k, False)  # p.Ap
            lib.call("trnsparse_bsr_cg_dist_phase", *self.geo, self.x.data_ptr(), inv, self.tol, self.max_iter, k, 1,
                     ws.data_ptr(), s)
            self._push(slot + 32 * k + 16, slot + 32 * k + 24, 1, 2 + 2 * k, True)  # r.r, r.z, halo of r

    def _solve_fused(self, coop: bool = False) -> None:
        lib, sh, ws = self._lib, self.shard, self.ws
        s = lib.stream_handle(self.dev)
        inv = lib.ptr(self.inv_d)
        peer = (self.peers_dev.data_ptr(), self.world, self.rank, self.comm_off, self.sends_dev.data_ptr(),
                self.n_sends)
        self.x.zero_()
        lib.call("trnsparse_bsr_cg_fused_start", sh.n_own, sh.n_ext, sh.block_size, self.b.data_ptr(), inv,
                 self.max_iter, ws.data_ptr(), self.ws_bytes, *peer, s)
        if coop:
            lib.call("trnsparse_bsr_cg_coop_run", *self.geo, self.x.data_ptr(), inv, self.tol, self.max_iter, 0,
                     self.max_iter, ws.data_ptr(), *peer, s)
            return
        for k in range(self.max_iter + 1):
            lib.call("trnsparse_bsr_cg_fused_phase", *self.geo, self.x.data_ptr(), inv, self.tol, self.max_iter, k, 0,
                     ws.data_ptr(), *peer, s)
            if k == self.max_iter:
                break
            lib.call("trnsparse_bsr_cg_fused_phase", *self.geo, self.x.data_ptr(), inv, self.tol, self.max_iter, k, 1,
                     ws.data_ptr(), *peer, s)

    def _solve_cgcg(self) -> None:
        lib, sh = self._lib, self.shard
        lib.call("trnsparse_bsr_cgcg_solve", *self.geo, self.b.data_ptr(), self.x.data_ptr(), lib.ptr(self.inv_d),
                 self.tol, self.max_iter, self.n_alloc, self.ws.data_ptr(), 0, self.ws_bytes,
                 self.peers_dev.data_ptr(), self.world, self.rank, self.comm_off, self.sends_dev.data_ptr(),
                 self.n_sends, lib.stream_handle(self.dev))

    def run(self) -> tuple[torch.Tensor, int, float]:
        self.launch()
        return self.result()

    def launch(self) -> None:
        """Enqueue the solve on this rank's stream (one graph replay when captured; the
        uncaptured transports also poll the device between chunks of iterations)."""
        with torch.cuda.device(self.dev):
            if self.graph is not None:
                self.graph.replay()
            else:
                self._solve(check=True)

    def result(self) -> tuple[torch.Tensor, int, float]:
        """Wait for the solve enqueued by ``launch`` and read its status: this rank's
        slice of x, the iteration count and the relative residual."""
        head = self.ws[:64].cpu()
        if head[8:12].view(torch.int32).item() == 5:
            raise RuntimeError("sharded CG: an exchange with a peer timed out (device error word set)")
        return self.x, head[4:8].view(torch.int32).item(), head[16:24].view(torch.float64).item()

    def executed_iterations(self) -> int:
        """Iterations that did work (the reference's loop may break early on |p.Ap| < 1e-30)."""
        pap = self.ws[self.offs[1] : self.offs[1] + 32 * (self.max_iter + 2)].view(torch.float64).view(-1, 4)[:, 0]
        nz = (pap != 0).nonzero()
        return int(nz[-1].item()) + 1 if nz.numel() else 0


def cg_bsr_sharded(
    shard: BSRShard,
    b_local: torch.Tensor,
    tol: float = 1e-6,
    max_iter: int = 1000,
    jacobi: bool = True,
    group=None,
    check_every: int = 16,
) -> tuple[torch.Tensor, int, float]:
    """Sharded PCG with the reference's control flow; returns this rank's
    slice of x, the iteration count and the relative residual (identical on
    every rank). ``b_local`` is the rank's n_own-long slice of b; the Jacobi
    preconditioner (iterative.py:129-145) is applied when ``jacobi``."""
    return ShardedCG(shard, b_local, tol, max_iter, jacobi, group, check_every).run()


# ---------------------------------------------------------------- fixed-step solvers, power iteration
def _shard_setup(shard: BSRShard, vec: torch.Tensor):
    from . import _lib
    from .ops import _bsr_geometry

    dev = vec.device
    return _lib, _bsr_geometry(shard.local, dev), _lib.stream_handle(dev), dev


def _global_sq(local_sq: torch.Tensor, group) -> float:
    """Sum of a float64 device scalar over the ranks (rank order is NCCL's, so the
    total may differ from a single-GPU sum in the last bit)."""
    dist.all_reduce(local_sq, group=group)
    return float(local_sq.item())


def _fixed_step_sharded(shard: BSRShard, b_local: torch.Tensor, coeffs, K: int, x0_local, group):
    lib, geo, s, dev = _shard_setup(shard, b_local)
    n_own, n_ext = shard.n_own, shard.n_ext
    b = b_local.to(dev, torch.float32).contiguous()
    bb = torch.sum(b.double() * b.double()).reshape(1)
    b_norm = float(torch.tensor(_global_sq(bb, group) ** 0.5, dtype=torch.float32))
    # three extended buffers rotate: x_k (halo refreshed before each step), x_{k-1}, x_{k+1}
    bufs = [torch.zeros(n_ext, dtype=torch.float32, device=dev) for _ in range(3)]
    if x0_local is not None:
        bufs[0][:n_own] = x0_local.to(dev, torch.float32)
    with torch.cuda.device(dev):
        for k in range(K):
            xk, xp, xn = bufs[k % 3], bufs[(k + 2) % 3], bufs[(k + 1) % 3]
            halo_exchange(shard, xk, group)
            a, bc = coeffs(k)
            lib.call("trnsparse_bsr_chebyshev_step", *geo, b.data_ptr(), xk.data_ptr(), xp.data_ptr(), xn.data_ptr(),
                     a, 0.0 if bc is None else bc, 1 if k > 0 and bc is not None else 0, s)
        x = bufs[K % 3]
        halo_exchange(shard, x, group)
        rr = torch.zeros(1, dtype=torch.float64, device=dev)
        lib.call("trnsparse_bsr_residual_sq", *geo, b.data_ptr(), x.data_ptr(), rr.data_ptr(), s)
    r_norm = float(torch.tensor(_global_sq(rr, group) ** 0.5, dtype=torch.float32))
    return x[:n_own].clone(), K, r_norm / max(b_norm, 1e-15)


def chebyshev_bsr_sharded(shard: BSRShard, b_local: torch.Tensor, lam_min: float, lam_max: float, K: int = 50,
                          x0_local: torch.Tensor | None = None, group=None) -> tuple[torch.Tensor, int, float]:
    """K-step Chebyshev semi-iteration (reference: iterative.py:193-253) on a
    block-row shard: per step the halo rows of x are refreshed (NCCL
    send/recv), then one fused SpMV + update launch runs on the own rows; the
    final relative residual is reduced across the ranks. Returns this rank's
    slice of x, K and rel (identical on every rank)."""
    from .iterative import chebyshev_coeffs

    alpha, beta = chebyshev_coeffs(lam_min, lam_max, K)
    al, be = alpha.tolist(), beta.tolist()
    return _fixed_step_sharded(shard, b_local, lambda k: (al[k], be[k] if k > 0 else 0.0), K, x0_local, group)


def richardson_bsr_sharded(shard: BSRShard, b_local: torch.Tensor, omega: float, K: int = 100,
                           x0_local: torch.Tensor | None = None, group=None) -> tuple[torch.Tensor, int, float]:
    """K-step Richardson ``x += omega (b - A x)`` (reference: iterative.py:256-295) on a block-row shard."""
    w = float(omega)
    return _fixed_step_sharded(shard, b_local, lambda k: (w, None), K, x0_local, group)


def power_iteration_bsr_sharded(shard: BSRShard, v0_local: torch.Tensor, max_iter: int = 100, tol: float = 1e-9,
                                group=None) -> tuple[float, torch.Tensor, int]:
    """Dominant eigenpair by power iteration (reference: iterative.py:298-340)
    on a block-row shard. Per iteration: halo refresh of v, one SpMV launch
    that also forms the partial v.Av and ||Av||^2, one all-reduce of the two
    partials, then v = Av / ||Av|| on the device. The host reads the two
    reduced scalars each iteration for the reference's stopping tests.
    Returns (eigenvalue, this rank's slice of v, iterations)."""
    lib, geo, s, dev = _shard_setup(shard, v0_local)
    n_own, n_ext = shard.n_own, shard.n_ext
    v = torch.zeros(n_ext, dtype=torch.float32, device=dev)
    w = torch.zeros(n_own, dtype=torch.float32, device=dev)
    v0 = v0_local.to(dev, torch.float32).contiguous()
    ss = torch.sum(v0.double() * v0.double()).reshape(1)
    dist.all_reduce(ss, group=group)
    dots = torch.zeros(2, dtype=torch.float64, device=dev)
    lam_prev, lam = 0.0, 0.0
    with torch.cuda.device(dev):
        lib.call("trnsparse_vec_div_norm", n_own, v0.data_ptr(), ss.data_ptr(), v.data_ptr(), s)
        for k in range(max_iter):
            halo_exchange(shard, v, group)
            dots.zero_()
            lib.call("trnsparse_bsr_power_step", *geo, v.data_ptr(), w.data_ptr(), dots.data_ptr(), s)
            dist.all_reduce(dots, group=group)
            lam, ww = dots.tolist()
            norm = float(torch.tensor(ww ** 0.5, dtype=torch.float32))
            if norm < 1e-30:
                return 0.0, v[:n_own].clone(), k + 1
            lib.call("trnsparse_vec_div_norm", n_own, w.data_ptr(), dots[1:].data_ptr(), v.data_ptr(), s)
            if abs(lam - lam_prev) < tol:
                return lam, v[:n_own].clone(), k + 1
            lam_prev = lam
    return lam, v[:n_own].clone(), max_iter
