"""Benchmark of the trnsparse_b200 sparse compute path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (one JSON line on rank 0): config 2, CSR spmv ``y = 2.0 * A @ x`` on
the 5-point Poisson Laplacian of a 2048x2048 grid (4,194,304 rows,
20,963,328 nnz, int32 indices, fp32), reported as algorithmic HBM GB/s:
bytes = 4*nnz (values) + 4*nnz (col idx) + 4*(n+1) (row ptr) + 4*n (x) + 4*n (y).
Each timed step is one spmv launch on device-resident inputs. The inputs
(218 MB) exceed L2 (126 MB), so the K timed steps run back to back, captured
in one CUDA graph and timed with CUDA events around its replay (no host gaps
between launches). ``e2e`` times the public
API call ``trnsparse_b200.spmv`` with the dense operand in pinned host
memory: the host->device copy of x, the kernel and the device->host copy of
y are inside the window.

Secondary measurements (bsr_spmm TFLOP/s and the other configurations) are
reported under ``extra``. With N > 1 (torchrun, one process per GPU, NCCL)
every rank runs the headline workload on its own GPU (weak scaling, no
data-path collective); time is the max over ranks.

``--impl reference`` times the reference algorithm on the host CPU instead
(the oracle restatement in ``oracle/``: ATen's CSR SpMV, all host threads),
rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BASELINE = json.loads((ROOT / "BASELINE.json").read_text())

# DRAM bytes per launch measured with ncu (dram__bytes_read.sum + dram__bytes_write.sum,
# one launch of each kernel on the workload its row reports)
NCU_TRAFFIC = {
    "csr_spmv_warp_kernel": 205.3e6,  # config 2 spmv
}
METRIC = BASELINE["metric"]


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- helpers
def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, ws: int) -> float:
    if ws == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class L2Flush:
    """Writes, then reads, a buffer 4x the L2 size: L2 ends up holding only
    clean lines of this buffer, so the timed kernel neither hits its inputs
    in L2 nor pays for write-backs of the flush."""

    def __init__(self, nbytes=512 << 20):
        self.buf = torch.empty(nbytes // 4, dtype=torch.float32, device="cuda")

    def __call__(self):
        self.buf.fill_(1.0)
        self.buf.sum()


def graph_steps(step, steps: int, warmup: int):
    """Captures ``steps`` back-to-back calls of ``step`` in one CUDA graph and
    times its replay with CUDA events (no host gaps between launches); returns
    milliseconds per step. Used for workloads whose inputs exceed L2."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
        with torch.cuda.graph(g, stream=s):
            for _ in range(steps):
                step()
    torch.cuda.synchronize()
    g.replay()  # warm replay
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def timed_steps(step, steps: int, warmup: int, flush: L2Flush | None):
    """Runs warmup + timed steps; returns per-step device milliseconds (kernel window only)."""
    for _ in range(warmup):
        if flush:
            flush()
        step()
    torch.cuda.synchronize()
    evs = []
    for _ in range(steps):
        if flush:
            flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        step()
        b.record()
        evs.append((a, b))
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


# --------------------------------------------------------------------------- workloads
def spmv_bytes(A) -> int:
    n = A.shape[0]
    isz = A.row_ptrs.element_size()
    return 4 * A.nnz + isz * A.nnz + isz * (n + 1) + 4 * n + 4 * n


def run_ours(args, ws, rank, local):
    import trnsparse_b200 as ts
    from trnsparse_b200 import workloads as w

    pk = peaks()
    dev = torch.device("cuda", local)
    A = w.poisson2d_csr(2048)
    x_host = w.poisson_rhs(A.shape[0])
    n = A.shape[0]
    x = x_host.to(dev)
    A.device_layout(dev)
    nbytes = spmv_bytes(A)
    flush = L2Flush()

    def step():
        return ts.spmv(A, x, alpha=2.0)

    barrier(ws)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ms_local = graph_steps(step, args.steps, args.warmup)
    barrier(ws)
    ms_per_step = max_over_ranks(ms_local, ws)
    value = ws * nbytes / (ms_per_step * 1e-3) / 1e9

    # e2e through the public API with host buffers
    x_pin = x_host.pin_memory()

    def e2e_step():
        return ts.spmv(A, x_pin, alpha=2.0)

    e2e_ms = timed_steps(e2e_step, args.steps, args.warmup, flush)
    e2e_ms = max_over_ranks(sum(e2e_ms), ws) / args.steps
    e2e_val = ws * nbytes / (e2e_ms * 1e-3) / 1e9

    ach = nbytes / (ms_local * 1e-3) / 1e9
    line = {
        "metric": METRIC,
        "headline": "csr_spmv (config 2) algorithmic HBM GB/s",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded 5-point Poisson, x ~ N(0,1) seed 1)",
        "config": {"workload": "config2_csr_spmv_poisson2048_alpha2", "rows": n, "nnz": A.nnz, "index": "int32",
                   "bytes_per_step": nbytes,
                   "l2": "inputs (218 MB) exceed L2 (126 MB); steps back to back in one CUDA graph",
                   "parallelism": f"replica x{ws}"},
        "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "ms_per_step": round(e2e_ms, 5),
                "h2d_bytes_per_step": 4 * n, "d2h_bytes_per_step": 4 * n},
        "gpu_launches": args.steps,
        "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(ach / pk["hbm_gbs"], 4), "peak_source": pk["source"] + " (burst copy)",
                     "frac_of_nominal_8tbs": round(ach / 8000.0, 4),
                     "traffic": NCU_TRAFFIC["csr_spmv_warp_kernel"],
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch on this "
                     "workload (L2 flushed before it)", "kernel": "csr_spmv_warp_kernel<int,float,2,384>"},
        "clocks": clk.summary(),
    }
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_spmv(A, x_host)
    if rank == 0 and ws == 1 and not args.no_extra:
        line["extra"] = run_extras(pk, flush, reps=args.reps)
    if ws > 1 and not args.no_extra:
        sharded = run_sharded_cg(ws, rank, local, pk)
        if rank == 0:
            line["extra_sharded"] = sharded
    elif not args.no_extra:
        # the same sharded solvers on one rank: the N = 1 point of their scaling curve
        import socket

        import torch.distributed as dist

        sock = socket.socket()
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
        sock.close()
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                                device_id=torch.device("cuda", local))
        try:
            line["extra_sharded"] = run_sharded_cg(1, 0, local, pk, transports=("cgcg", "coop"))
        finally:
            dist.destroy_process_group()
    return line


def _gather_x(x_local: torch.Tensor, ws: int) -> torch.Tensor | None:
    """The full solution on rank 0 (shards are contiguous block-row ranges in rank order)."""
    if ws == 1:
        return x_local
    import torch.distributed as dist

    n = torch.tensor([x_local.numel()], dtype=torch.int64, device=x_local.device)
    sizes = [torch.zeros_like(n) for _ in range(ws)]
    dist.all_gather(sizes, n)
    cap = int(max(int(t.item()) for t in sizes))
    buf = torch.zeros(cap, dtype=x_local.dtype, device=x_local.device)
    buf[: x_local.numel()] = x_local
    parts = [torch.empty_like(buf) for _ in range(ws)]
    dist.all_gather(parts, buf)
    return torch.cat([p[: int(t.item())] for p, t in zip(parts, sizes)])


def run_sharded_cg(ws: int, rank: int, local: int, pk: dict,
                   transports: tuple = ("cgcg", "coop", "fused", "peer", "nccl")) -> dict:
    """Config 5 on ws GPUs: block-row-sharded Jacobi-PCG (strong scaling: the
    2048-block-row matrix is split across the ranks), each transport (cgcg:
    one reduction per iteration in one cooperative launch; coop / fused /
    peer / nccl: the reference's two reductions), whole solve captured in one
    CUDA graph, ``iters`` iterations with tol 0. ``us_per_iteration`` is the
    device time of the graph replay (CUDA events on the solve's stream around
    ``launch()``), max over ranks; ``us_per_iteration_with_readback`` also
    holds the host read of the status words (``result()``).

    Every row carries its own correctness check and speed-up: the sharded x
    is gathered to rank 0 and compared (relative 2-norm error) with the
    unsharded single-GPU ``cg_bsr`` solve of the same matrix, right-hand side
    and iteration count, which rank 0 also times in the same run
    (``us_per_iteration_single_gpu``: the faster of the public ``cg_bsr`` call
    and the one-rank cgcg solve in a CUDA graph timed like the sharded one,
    named in ``single_gpu_solver``);
    ``speedup_vs_1gpu`` = that time per iteration / sharded time per iteration."""
    import torch.distributed as dist

    import trnsparse_b200 as ts
    from trnsparse_b200 import distributed as D
    from trnsparse_b200 import workloads as w

    A, b = w.block_pentadiagonal_spd()
    iters = 30
    # the single-GPU reference solve (rank 0): the library's own cg_bsr with Jacobi
    single = {}
    if rank == 0:
        M = ts.jacobi_preconditioner_bsr(A)
        bd = b.cuda()
        ts.cg_bsr(A, bd, tol=0.0, max_iter=iters, M=M)
        torch.cuda.synchronize()
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        x1, it1, rel1 = ts.cg_bsr(A, bd, tol=0.0, max_iter=iters, M=M)
        e.record()
        torch.cuda.synchronize()
        single = {"x": x1.clone(), "ms": a.elapsed_time(e), "rel": rel1}
        del M, bd
    # the best single-GPU solve of the same problem: the one-rank cgcg solve captured in a
    # CUDA graph like the sharded ones (every rank takes part in creating the group)
    one = dist.new_group([0])
    if rank == 0:
        try:
            sh1 = D.shard_bsr(A, 0, 1)
            cg1 = D.ShardedCG(sh1, b.cuda(), tol=0.0, max_iter=iters, graph=True, transport="cgcg", group=one)
            cg1.run()
            torch.cuda.synchronize()
            a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            cg1.launch()
            e.record()
            cg1.result()
            single["ms_cgcg1"] = a.elapsed_time(e)
            single["exec_cgcg1"] = cg1.executed_iterations()
            cg1.close()
        except Exception as exc:  # keep the cg_bsr baseline if the one-rank solve cannot run
            single["cgcg1_error"] = f"{type(exc).__name__}: {exc}"[:120]
    dist.barrier()
    sh = D.shard_bsr(A, rank, ws)
    bl = b[sh.r0 * 128 : sh.r1 * 128].cuda()
    devs = [None] * ws
    dist.all_gather_object(devs, str(torch.cuda.get_device_properties(local).uuid))
    out = {}
    for transport in transports:
        try:
            cg = D.ShardedCG(sh, bl, tol=0.0, max_iter=iters, graph=True, transport=transport)
            cg.run()
            torch.cuda.synchronize()
            dist.barrier()
            a, e, f = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            a.record()
            cg.launch()
            e.record()
            x, it, rel = cg.result()
            f.record()
            torch.cuda.synchronize()
            ms = max_over_ranks(a.elapsed_time(e), ws)
            ms_rb = max_over_ranks(a.elapsed_time(f), ws)
            executed = cg.executed_iterations()
            xg = _gather_x(x, ws)
            cg.close()
        except Exception as exc:  # one transport failing must not lose the others' numbers
            out[f"config5_cg_sharded_{transport}"] = {"error": f"{type(exc).__name__}: {exc}"[:200]}
            continue
        nb = A.n_blocks * 128 * 128 * 4
        row = {"us_per_iteration": round(ms / max(executed, 1) * 1e3, 2),
               "us_per_iteration_with_readback": round(ms_rb / max(executed, 1) * 1e3, 2),
               "executed_iterations": executed,
               "max_iter": iters, "ranks": ws, "gpus_active": len(set(devs)),
               "matrix_GB/s_aggregate": round(nb * executed / (ms * 1e-3) / 1e9, 1),
               "scaling": "strong", "rel_residual": rel}
        if rank == 0:
            err = float((xg.double() - single["x"].double()).norm() / single["x"].double().norm())
            us_api = single["ms"] / max(executed, 1) * 1e3
            us1, src = us_api, "cg_bsr"
            if "ms_cgcg1" in single:
                us_g = single["ms_cgcg1"] / max(single["exec_cgcg1"], 1) * 1e3
                if us_g < us1:
                    us1, src = us_g, "one-rank cgcg, CUDA graph"
            row.update({"rel_err_vs_single_gpu": err, "us_per_iteration_single_gpu": round(us1, 2),
                        "single_gpu_solver": src, "us_per_iteration_cg_bsr_api": round(us_api, 2),
                        "speedup_vs_1gpu": round(us1 / (ms / max(executed, 1) * 1e3), 3)})
        out[f"config5_cg_sharded_{transport}"] = row
    return out


def time_call(f, reps: int, flush: L2Flush | None) -> float:
    """Median device milliseconds of one call of ``f`` replayed from a CUDA
    graph; with ``flush`` the L2 is flushed (outside the timed window) before
    every replay, for workloads whose inputs fit in L2."""
    for _ in range(3):
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        f()
        with torch.cuda.graph(g, stream=s):
            f()
    torch.cuda.synchronize()
    out = []
    for _ in range(reps):
        if flush:
            flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        out.append(a.elapsed_time(b))
    out.sort()
    return out[len(out) // 2]


def graph_k(f, k: int) -> float:
    """Milliseconds per call of ``f`` over ``k`` back-to-back calls captured in
    one CUDA graph (launch overhead amortised; inputs that fit in L2 stay warm)."""
    for _ in range(3):
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        f()
        with torch.cuda.graph(g, stream=s):
            for _ in range(k):
                f()
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / k


def row_bsr_spmm(pk: dict, flush: L2Flush, reps: int, cases: tuple = ("config1", "grid128"),
                 dtypes: tuple = ("f32", "bf16")) -> dict:
    """Config 1 and a scaled variant (128 x 128 block grid, k = 512, same
    distribution), fp32 (3xTF32) and bf16. Nonzero-block FLOPs
    2*128*128*k per stored block. ``ms`` = one call replayed from a graph
    after an L2 flush (cold); ``ms_back_to_back`` = K calls in one graph / K
    (the launch latency amortised; config 1's 7.5 MB of inputs stay in L2)."""
    import trnsparse_b200 as ts
    from trnsparse_b200 import workloads as w

    tf32 = 0.5 * pk["bf16_tflops"]
    ex = {}
    for name, grid, k in [("config1_bsr_spmm", 16, 256), ("bsr_spmm_grid128_k512", 128, 512)]:
        if name.split("_")[0] not in cases and name.split("_")[2] not in cases:
            continue
        for dt, tag in [(torch.float32, "f32_3xtf32"), (torch.bfloat16, "bf16")]:
            if tag.split("_")[0] not in dtypes:
                continue
            A, B = w.bsr_random_grid(grid=grid, k=k, dtype=dt)
            Bd = B.cuda()
            small = grid == 16
            f = lambda: ts.bsr_spmm(A, Bd)  # noqa: E731
            ms = time_call(f, reps, flush if small else None)
            ms_k = graph_k(f, 20 if small else 5)
            flop = 2 * 128 * 128 * k * A.n_blocks
            tfl = flop / (ms * 1e-3) / 1e12
            tfl_k = flop / (ms_k * 1e-3) / 1e12
            peak = pk["bf16_tflops"] if dt == torch.bfloat16 else tf32 / 3
            ex[f"{name}_{tag}"] = {
                "TFLOP/s": round(tfl, 1), "ms": round(ms, 4), "ms_back_to_back": round(ms_k, 4),
                "n_blocks": A.n_blocks, "frac_of_peak": round(tfl / peak, 3),
                "roofline": {"bound": "tensor", "achieved": round(tfl_k, 1), "peak": round(peak, 1),
                             "unit": "TFLOP/s", "frac": round(tfl_k / peak, 3),
                             "peak_source": ("bf16 measured (burst)" if dt == torch.bfloat16 else
                                             "tf32 = 0.5 x measured bf16, / 3 passes"),
                             "time": "back to back"},
                "l2": "flushed before the single call" if small else "inputs exceed L2",
                "includes": "every kernel of the call (B split for fp32, C clearing when a block-row is split)"}
            del A, B, Bd
    return ex


def row_csr_spmm(pk: dict, flush: L2Flush, reps: int) -> dict:
    """Config 2b: CSR spmm, k = 32 (inputs exceed L2)."""
    import trnsparse_b200 as ts
    from trnsparse_b200 import workloads as w

    A = w.poisson2d_csr(2048)
    Bm = w.poisson_rhs(A.shape[0], 32).cuda()
    n = A.shape[0]
    ms = time_call(lambda: ts.spmm(A, Bm), reps, None)
    nb = 8 * A.nnz + 4 * (n + 1) + 4 * n * 32 * 2
    return {"config2b_csr_spmm_k32": {"GB/s": round(nb / (ms * 1e-3) / 1e9, 1), "ms": round(ms, 4),
                                      "frac_of_hbm": round(nb / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 3)}}


def row_screened(pk: dict, flush: L2Flush, reps: int) -> dict:
    """Config 3: screened_spmm with 2-D pair bounds."""
    import trnsparse_b200 as ts
    from trnsparse_b200 import workloads as w

    tf32 = 0.5 * pk["bf16_tflops"]
    Af, Qf, Bf, _, thr = w.fock_like()
    Ad, Qd, Bd = Af.cuda(), Qf.cuda(), Bf.cuda()
    del Af, Qf, Bf
    ms = time_call(lambda: ts.screened_spmm(Ad, Qd, Bd, thr), reps, None)
    fl = 2 * 8192 * 8192 * 512  # every 128x128 block has a surviving pair (unsorted centres)
    return {"config3_screened_spmm": {"TFLOP/s": round(fl / (ms * 1e-3) / 1e12, 1), "ms": round(ms, 4),
                                      "frac_of_peak": round(fl / (ms * 1e-3) / 1e12 / (tf32 / 3), 3),
                                      "peak": "tf32 derived / 3 passes"}}


def row_attention(pk: dict, flush: L2Flush, reps: int) -> dict:
    """Config 4: block-sparse attention forward and backward (bf16)."""
    import trnsparse_b200 as ts
    from trnsparse_b200 import workloads as w
    from trnsparse_b200.ops import _attn_backward, _attn_forward

    ex = {}
    mask = w.sliding_window_mask()
    Qa, Ka, Va = (t.cuda() for t in w.attention_inputs())
    ms = time_call(lambda: ts.block_sparse_attention_tiled(Qa, Ka, Va, mask), max(3, reps // 2), None)
    fl = 4 * 128 ** 3 * mask.n_blocks * 16
    ex["config4_block_sparse_attention_bf16"] = {
        "TFLOP/s": round(fl / (ms * 1e-3) / 1e12, 1), "ms": round(ms, 4), "blocks_per_head": mask.n_blocks,
        "frac_of_peak": round(fl / (ms * 1e-3) / 1e12 / pk["bf16_tflops"], 3), "peak": "bf16 measured",
        "note": "FLOPs counted once per block (QK^T + PV); one pass with an online softmax"}
    # backward: dQ, dK, dV on the tensor cores, with the forward's saved log-sum-exp (as autograd runs it)
    Oa, lse = _attn_forward(Qa, Ka, Va, mask, 128 ** -0.5, want_lse=True)
    dOa = torch.randn(Oa.shape, generator=torch.Generator().manual_seed(5)).to(Oa.dtype).cuda()
    ms = time_call(lambda: _attn_backward(Qa, Ka, Va, Oa, dOa, mask, 128 ** -0.5, lse=lse), max(3, reps // 3), None)
    flb = 10 * 128 ** 3 * mask.n_blocks * 16
    ex["config4_attention_backward_bf16"] = {
        "TFLOP/s": round(flb / (ms * 1e-3) / 1e12, 1), "ms": round(ms, 3),
        "frac_of_peak": round(flb / (ms * 1e-3) / 1e12 / pk["bf16_tflops"], 3), "peak": "bf16 measured",
        "note": "tcgen05 kernels (dQ row-first, dK/dV column-first); FLOPs = S, dP, dQ, dK, dV per block "
                "(10*128^3)"}
    return ex


def row_cg(pk: dict, flush: L2Flush, reps: int) -> dict:
    """Config 5: Jacobi-PCG, tol 0, max_iter 200, and the config-5 BSR SpMV."""
    import trnsparse_b200 as ts
    from trnsparse_b200 import workloads as w
    from trnsparse_b200.iterative import _cg_bsr_device

    ex = {}
    A5, b5 = w.block_pentadiagonal_spd()
    M5 = ts.jacobi_preconditioner_bsr(A5)
    bd = b5.cuda()
    _cg_bsr_device(A5, bd, None, 0.0, 5, M5)
    torch.cuda.synchronize()
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    x, it, rel, executed = _cg_bsr_device(A5, bd, None, 0.0, 200, M5)
    e.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(e)
    ex["config5_cg_bsr_jacobi_200"] = {
        "ms_total": round(ms, 3), "iters_reported": it, "executed_iterations": executed,
        "us_per_executed_iteration": round(ms / max(executed, 1) * 1e3, 2), "rel_residual": rel,
        "note": "tol 0, max_iter 200 with the reference's control flow: the loop breaks when |p.Ap| < 1e-30 "
                "(iters_reported stays max_iter, as the reference returns); the whole solve is one cooperative "
                "launch that returns at the break, so ms_total covers the executed iterations only"}
    xv = bd.unsqueeze(1)
    ms = time_call(lambda: ts.bsr_spmm(A5, xv), reps, None)
    nb = A5.n_blocks * 128 * 128 * 4 + 4 * A5.n_blocks + 4 * 2049 + 8 * A5.shape[0]
    ex["config5_bsr_spmv"] = {"GB/s": round(nb / (ms * 1e-3) / 1e9, 1), "ms": round(ms, 4),
                              "frac_of_hbm": round(nb / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 3)}
    return ex


def row_formats(pk: dict, flush: L2Flush, reps: int) -> dict:
    return run_format_extras(pk)


ROWS = {"bsr_spmm": row_bsr_spmm,
        # single bsr_spmm cases, for profiling one kernel configuration
        "bsr_spmm_config1_f32": lambda pk, fl, r: row_bsr_spmm(pk, fl, r, ("config1",), ("f32",)),
        "bsr_spmm_config1_bf16": lambda pk, fl, r: row_bsr_spmm(pk, fl, r, ("config1",), ("bf16",)),
        "bsr_spmm_grid128_f32": lambda pk, fl, r: row_bsr_spmm(pk, fl, r, ("grid128",), ("f32",)),
        "bsr_spmm_grid128_bf16": lambda pk, fl, r: row_bsr_spmm(pk, fl, r, ("grid128",), ("bf16",)), "csr_spmm": row_csr_spmm, "screened": row_screened,
        "attention": row_attention, "cg": row_cg, "formats": row_formats}


DEFAULT_ROWS = ("bsr_spmm", "csr_spmm", "screened", "attention", "cg", "formats")


def run_extras(pk: dict, flush: L2Flush, only: list[str] | None = None, reps: int = 10) -> dict:
    """Secondary rows: the other benchmark configurations (``only`` selects row groups)."""
    ex = {}
    for name, fn in ROWS.items():
        if (only is None and name in DEFAULT_ROWS) or (only is not None and name in only):
            ex.update(fn(pk, flush, reps))
    return ex


def time_eager(f, reps: int) -> float:
    """Median device milliseconds of ``f`` run eagerly (for calls that read a count back
    to the host mid-way and so cannot be captured in a graph)."""
    for _ in range(3):
        f()
    torch.cuda.synchronize()
    out = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        f()
        b.record()
        torch.cuda.synchronize()
        out.append(a.elapsed_time(b))
    out.sort()
    return out[len(out) // 2]


def run_format_extras(pk: dict) -> dict:
    """Device-side format construction (csrc/formats.cu): algorithmic bytes = the dense
    input read once + the sparse output written (COO: indices and values read, sorted
    output written); inputs exceed L2."""
    import trnsparse_b200 as ts
    from trnsparse_b200 import workloads as w

    ex = {}
    g = torch.Generator().manual_seed(0)
    n, b = 16384, 128
    keep = torch.rand(n // b, n // b, generator=g) < 0.25
    A = torch.randn(n, n, generator=g)
    A.mul_(keep.repeat_interleave(b, 0).repeat_interleave(b, 1))
    Ad = A.cuda()
    del A
    bsr = ts.BSRMatrix.from_dense(Ad, block_size=b)
    ms = time_eager(lambda: ts.BSRMatrix.from_dense(Ad, block_size=b), 5)
    nb = Ad.numel() * 4 + bsr.n_blocks * (b * b * 4 + 8) + 8 * (n // b + 1)
    ex["formats_bsr_from_dense_16384_p025"] = {
        "ms": round(ms, 3), "GB/s": round(nb / (ms * 1e-3) / 1e9, 1), "n_blocks": bsr.n_blocks,
        "frac_of_hbm": round(nb / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 3),
        "note": "screen pass reads A; fill pass re-reads the kept blocks (not counted); one host read of the count"}
    del bsr
    Ad = torch.randn(8192, 8192, generator=g).cuda()
    Ad[torch.rand(8192, 8192, device="cuda") < 0.983] = 0.0
    csr = ts.from_dense(Ad)
    ms = time_eager(lambda: ts.from_dense(Ad), 5)
    nb = Ad.numel() * 4 + csr.nnz * 12 + 8 * 8193
    ex["formats_csr_from_dense_8192_d0017"] = {
        "ms": round(ms, 3), "GB/s": round(nb / (ms * 1e-3) / 1e9, 1), "nnz": csr.nnz,
        "frac_of_hbm": round(nb / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 3),
        "note": "the count pass reads A and writes a kept-entry bit mask; the fill gathers the kept values "
                "through it (its reads not counted); one host read of nnz"}
    del Ad, csr
    A2 = w.poisson2d_csr(2048)
    counts = (A2.row_ptrs[1:] - A2.row_ptrs[:-1]).long()
    rows = torch.repeat_interleave(torch.arange(A2.shape[0]), counts)
    perm = torch.randperm(rows.numel(), generator=g)
    coo = ts.COOMatrix(values=A2.values[perm].cuda(), row_indices=rows[perm].cuda(),
                       col_indices=A2.col_indices[perm].long().cuda(), shape=A2.shape)
    ms = time_eager(lambda: coo.to_csr(), 5)
    nnz = coo.nnz
    nb = nnz * (8 + 8 + 4) + nnz * (8 + 4) + 8 * (A2.shape[0] + 1)
    ex["formats_coo_to_csr_config2_shuffled"] = {
        "ms": round(ms, 3), "GB/s": round(nb / (ms * 1e-3) / 1e9, 1), "nnz": nnz,
        "frac_of_hbm": round(nb / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 3),
        "note": "config-2 Poisson entries in random order; includes the index check read-back"}
    return ex


def cpu_baseline_spmv(A, x_host, budget_s: float = 3.0) -> dict:
    import oracle

    nbytes = spmv_bytes(A)
    oracle.csr_spmv(A.row_ptrs, A.col_indices, A.values, A.shape, x_host, 2.0)
    t0 = time.perf_counter()
    reps = 0
    while time.perf_counter() - t0 < budget_s or reps < 3:
        oracle.csr_spmv(A.row_ptrs, A.col_indices, A.values, A.shape, x_host, 2.0)
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"full config-2 spmv x{reps} (ATen CSR SpMV, as the reference's ops.py:30-48)",
            "ms_per_call": round(dt * 1e3, 3)}


def run_reference(args, ws, rank):
    from trnsparse_b200 import workloads as w

    if rank != 0:
        return None
    A = w.poisson2d_csr(2048)
    x = w.poisson_rhs(A.shape[0])
    import oracle

    nbytes = spmv_bytes(A)
    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(args.warmup):
        oracle.csr_spmv(A.row_ptrs, A.col_indices, A.values, A.shape, x, 2.0)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.csr_spmv(A.row_ptrs, A.col_indices, A.values, A.shape, x, 2.0)
    dt = (time.perf_counter() - t0) / args.steps
    val = nbytes / dt / 1e9
    return {
        "metric": METRIC, "impl": "reference", "value": round(val, 3), "unit": "GB/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded 5-point Poisson)",
        "config": {"workload": "config2_csr_spmv_poisson2048_alpha2", "rows": A.shape[0], "nnz": A.nnz,
                   "index": "int32", "bytes_per_step": nbytes},
        "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": "full config-2 spmv per step (oracle restatement of ops.py:30-48, ATen CSR SpMV)"},
        "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the secondary configurations")
    ap.add_argument("--only", default=None,
                    help="comma-separated row groups (" + ",".join(ROWS) + "): run only these secondary rows, "
                         "no headline (for profiling)")
    ap.add_argument("--reps", type=int, default=10, help="timed calls per secondary row")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = run_reference(args, ws, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    ws, rank, local = dist_setup()
    if args.only:
        line = {"only": args.only.split(","),
                "extra": run_extras(peaks(), L2Flush(), args.only.split(","), args.reps)}
        if rank == 0:
            print(json.dumps(line), flush=True)
        return
    line = run_ours(args, ws, rank, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
