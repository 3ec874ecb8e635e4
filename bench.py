"""Benchmark of the B200 sparse-product path (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl b200|reference] [--no-extras]

Headline workload (default ``spmm_f32``): BASELINE config 2, CSR SpMM of a
2^20 x 2^20 matrix with exactly 16 nonzeros per row times a dense 2^20 x 64
fp32 RHS. ``value`` is GB/s of the metric's algorithmic bytes
(nnz*(4+4) + 4(n+1) + 2*n*64*4 = 675.3 MB per product) over device time;
with N GPUs (torchrun) rows are split by balanced nnz, the RHS is replicated,
each rank times its share and the slowest rank sets the time (strong scaling).
Other workloads (``--workload``): spmm_bf16, spmv_lap2d, spmv_powerlaw,
pcg_poisson3d, spgemm. At N=1 the line also carries ``workloads`` with the
other configs measured the same way (skip with ``--no-extras``).

Timing: W warm-up steps, then K steps, each bracketed by CUDA events on the
launching stream; the L2 is flushed (a 512 MiB write) before every step and
outside its events. ``e2e`` repeats the product through the public API from
pinned host buffers, with the host->device copy of the inputs and the
device->host copy of the result inside the timed region. ``cpu_baseline`` times
the CPU oracle (a restatement of the reference's CPU loops) on a bounded
sample. ``--impl reference`` times that CPU implementation alone (all host
threads) on the same workload and prints its own line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, os.path.join(ROOT, "mlx-sparse_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

import workloads as wl  # noqa: E402

METRIC = "SpMV/SpMM HBM GB/s (% of B200 peak); CG iters/s at 1/2/4/8 B200 vs host CPU"


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# clocks sampling
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return None
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [s.strip() for s in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for name, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
def _shard_rows(indptr: np.ndarray, rank: int, world: int):
    """nnz-balanced contiguous row range of this rank (the reference's weighted
    ranges idea, cpu_parallel.cpp:202-253, applied to GPUs)."""
    n = indptr.shape[0] - 1
    nnz = int(indptr[-1])
    targets = [(nnz * r) // world for r in range(world + 1)]
    bounds = [int(np.searchsorted(indptr, t, side="left")) for t in targets]
    bounds[0], bounds[-1] = 0, n
    return bounds[rank], bounds[rank + 1]


def _slice_rows(d, i, p, r0, r1):
    k0, k1 = int(p[r0]), int(p[r1])
    return d[k0:k1], i[k0:k1], (p[r0:r1 + 1] - p[r0]).astype(p.dtype)


class Workload:
    name = ""
    unit = "GB/s"
    higher_is_better = True
    dtype = "f32"
    scaling = "strong"

    def setup(self, rank, world, device):
        raise NotImplementedError

    def step(self):
        raise NotImplementedError

    def e2e_step(self):
        raise NotImplementedError


class SpmmWorkload(Workload):
    def __init__(self, bf16=False, n=1 << 20, k=64, per_row=16, seed=2):
        self.bf16, self.n, self.k, self.per_row, self.seed = bf16, n, k, per_row, seed
        self.name = f"spmm_{'bf16' if bf16 else 'f32'}"
        self.dtype = "bf16 values/RHS, f32 accumulate" if bf16 else "f32"
        s = 2 if bf16 else 4
        nnz = n * per_row
        self.problem_bytes = nnz * (s + 4) + 4 * (n + 1) + 2 * n * k * s
        self.world = 1

    def config(self):
        return {"workload": self.name, "matrix": f"{self.n}x{self.n} csr, {self.per_row} nnz/row uniform cols",
                "rhs": f"{self.n}x{self.k} row-major", "index": "int32",
                "l2": "flushed before every step (512 MiB write)"}

    def setup_host(self):
        (d, i, p), shape = wl.random_k_per_row(self.n, self.n, self.per_row, self.seed)
        B = np.random.default_rng(self.seed + 100).uniform(-1, 1, (self.n, self.k)).astype(np.float32)
        self.full = (d, i, p, B)

    def setup(self, rank, world, device):
        import torch
        import mlx_sparse as ms

        self.setup_host()
        d, i, p, B = self.full
        r0, r1 = _shard_rows(p, rank, world)
        self.world, self.r0, self.r1 = world, r0, r1
        d, i, p = _slice_rows(d, i, p, r0, r1)
        self.host = (d, i, p, B)
        self.rows = r1 - r0
        tdt = torch.bfloat16 if self.bf16 else torch.float32
        self.tdt = tdt
        self.A = ms.csr_array((torch.from_numpy(d).to(device).to(tdt), torch.from_numpy(i).to(device),
                               torch.from_numpy(p).to(device)), shape=(self.rows, self.n), canonical=True)
        self.B = torch.from_numpy(B).to(device).to(tdt)
        self.out = torch.empty((self.rows, self.k), dtype=tdt, device=device)
        s = 2 if self.bf16 else 4
        self.dev = device
        self.launches_per_step = 1
        self.h_d = torch.from_numpy(d).to(tdt).pin_memory()
        self.h_p = torch.from_numpy(p).pin_memory()
        self.h_out = torch.empty((self.rows, self.k), dtype=tdt).pin_memory()
        if world == 1:
            # pinned host copies for the end-to-end leg
            self.h_i = torch.from_numpy(i).pin_memory()
            self.h_B = torch.from_numpy(B).to(tdt).pin_memory()
            self.h_A = ms.CSRArray(self.h_d, self.h_i, self.h_p, (self.rows, self.n), has_canonical_format=True)
            self.h2d_bytes = d.size * s + i.nbytes + p.nbytes + B.size * s
        else:
            # end to end at N > 1: each rank uploads its slab of A and only its
            # own rows of B; the rows of B are then all-gathered over NVLink
            # (NCCL), so no rank copies the whole B over PCIe
            from mlx_sparse.distributed import OperandExchange

            fd, fi, fp, _ = self.full
            self.exch = OperandExchange(fd, fi, fp, self.n, rank, world, device, mode="allgather")
            self.h_i = torch.from_numpy(np.ascontiguousarray(self.exch.local_indices)).pin_memory()
            self.h_B = torch.from_numpy(B[r0:r1]).to(tdt).pin_memory()
            self.n_local_cols = self.exch.n_local_cols
            self.h2d_bytes = d.size * s + i.nbytes + p.nbytes + (r1 - r0) * self.k * s
        self.d2h_bytes = self.rows * self.k * s

    def step(self):
        from mlx_sparse import _native

        _native.csr_matmul(self.A.data, self.A.indices, self.A.indptr, self.B, self.A.shape, out=self.out)

    def e2e_step(self):
        import mlx_sparse as ms

        dev = self.dev
        if self.world == 1:
            # host operands through the public streamed entry point: uploads,
            # row-block products and downloads overlap on three streams
            ms.csr_matmul_streamed(self.h_A, self.h_B, device=dev, out=self.h_out)
            return
        else:
            A = ms.csr_array((self.h_d.to(dev, non_blocking=True), self.h_i.to(dev, non_blocking=True),
                              self.h_p.to(dev, non_blocking=True)), shape=(self.rows, self.n_local_cols),
                             canonical=True)
            Y = A @ self.exch.exchange(self.h_B.to(dev, non_blocking=True))
        self.h_out.copy_(Y, non_blocking=True)

    def cpu_sample(self, workers, budget_s=10.0):
        from oracle import oracle

        d, i, p, B = self.full
        rows = self.n
        if self.bf16:
            dd, Bc = oracle.f32_to_bf16_bits(d), oracle.f32_to_bf16_bits(B)
        else:
            dd, Bc = d, B
        s = 2 if self.bf16 else 4
        sample_bytes = int(p[-1]) * (s + 4) + 4 * (rows + 1) + 2 * rows * self.k * s
        times = []
        t_end = time.perf_counter() + budget_s
        while time.perf_counter() < t_end or len(times) < 2:
            t0 = time.perf_counter()
            oracle.csr_matmul(dd, i, p, Bc, rows, bf16=self.bf16, workers=workers)
            times.append(time.perf_counter() - t0)
            if len(times) >= 200:
                break
        med = statistics.median(times)
        return sample_bytes / med / 1e9, f"full matrix ({rows} rows), median of {len(times)} runs"


class SpmvWorkload(Workload):
    """BASELINE configs 1 and 3. ``sharded=False``: at N > 1 every rank holds
    all of x (replicated input placement) and its nnz-balanced row slab;
    ``sharded=True``: x is sharded like the rows and each step first
    exchanges the entries a rank reads (NCCL: halo all-to-all for the
    Laplacian, all-gather for random power-law columns) - the exchange is
    inside the timed step."""

    def __init__(self, kind="lap2d", sharded=False):
        self.kind, self.sharded = kind, sharded
        self.name = f"spmv_{kind}" + ("_xsharded" if sharded else "")
        if kind == "lap2d":
            self.make = lambda: wl.lap2d(1024, np.int32)
            self.x_seed, self.it_bytes, self.dtype = 0, 4, "f32"
        else:
            self.make = lambda: wl.power_law(1 << 22, 3, np.int64)
            self.x_seed, self.it_bytes, self.dtype = 5, 8, "f32 values, int64 indices"

    def config(self):
        x = {"x": "row-sharded, exchanged each step" if self.sharded else "replicated on every GPU"}
        if self.kind == "lap2d":
            return {"workload": self.name, "matrix": "2D 5-point Laplacian 1024x1024 grid (n=1,048,576)",
                    "index": "int32", "l2": "flushed before every step (512 MiB write)", **x}
        return {"workload": self.name, "matrix": "power-law rows n=4,194,304 (Lomax alpha 2.1, mean ~20)",
                "index": "int64", "l2": "flushed before every step (512 MiB write)", **x}

    def setup_host(self):
        (d, i, p), shape = self.make()
        x = wl.uniform_vector(shape[1], self.x_seed)
        ib = self.it_bytes
        self.full = (d, i, p, x)
        self.shape = shape
        # metric bytes of the whole product: (4+ib) per nnz, indptr, x once, y
        self.problem_bytes = d.size * (4 + ib) + ib * (shape[0] + 1) + 4 * shape[1] + 4 * shape[0]

    def setup(self, rank, world, device):
        import torch
        import mlx_sparse as ms

        self.setup_host()
        d, i, p, x = self.full
        shape = self.shape
        ib = self.it_bytes
        self.world, self.rank, self.dev = world, rank, device
        r0, r1 = _shard_rows(p, rank, world)
        self.r0, self.r1 = r0, r1
        self.rows, self.n = r1 - r0, shape[1]
        if self.sharded and world > 1:
            from mlx_sparse.distributed import DistProduct

            self.P = DistProduct(d, i, p, shape[0], rank, world, device,
                                 mode="halo" if self.kind == "lap2d" else "allgather")
            self.x_own = torch.from_numpy(x[r0:r1].copy()).to(device)
            self.A = self.P.A
            self.plan = self.A.spmv_plan()
            sd, si, sp_ = self.P.slab.data, self.P.local_indices, self.P.slab.indptr
            self.h_x = torch.from_numpy(x[r0:r1].copy()).pin_memory()
            self.h2d_bytes = sd.nbytes + si.nbytes + sp_.nbytes + 4 * (r1 - r0)
        else:
            sd, si, sp_ = _slice_rows(d, i, p, r0, r1)
            self.A = ms.csr_array((torch.from_numpy(sd).to(device), torch.from_numpy(si).to(device),
                                   torch.from_numpy(sp_).to(device)), shape=(self.rows, self.n), canonical=True)
            self.plan = self.A.spmv_plan()
            self.x = torch.from_numpy(x).to(device)
            self.h_x = torch.from_numpy(x).pin_memory()
            self.h2d_bytes = sd.nbytes + si.nbytes + sp_.nbytes + x.nbytes
        self.host = (sd, si, sp_, x)
        self.y = torch.empty(self.rows, dtype=torch.float32, device=device)
        self.h_d, self.h_i, self.h_p = (torch.from_numpy(np.ascontiguousarray(a)).pin_memory() for a in (sd, si, sp_))
        self.h_y = torch.empty(self.rows, dtype=torch.float32).pin_memory()
        self.launches_per_step = 1 + (1 if self.plan.n_long > 0 else 0) + (2 if self.sharded and world > 1 else 0)
        self.d2h_bytes = self.rows * 4
        self.local_bytes = sd.size * (4 + ib) + ib * (self.rows + 1) + 4 * self.n + 4 * self.rows

    def step(self):
        from mlx_sparse import _native

        if self.sharded and self.world > 1:
            xl = self.P.exchange(self.x_own)
        else:
            xl = self.x
        _native.csr_matvec(self.A.data, self.A.indices, self.A.indptr, xl, self.A.shape, plan=self.plan,
                           out=self.y)

    def e2e_step(self):
        import mlx_sparse as ms

        dev = self.dev
        A = ms.csr_array((self.h_d.to(dev, non_blocking=True), self.h_i.to(dev, non_blocking=True),
                          self.h_p.to(dev, non_blocking=True)), shape=self.A.shape, canonical=True)
        xd = self.h_x.to(dev, non_blocking=True)
        if self.sharded and self.world > 1:
            xd = self.P.exchange(xd)
        y = A @ xd
        self.h_y.copy_(y, non_blocking=True)

    def parity(self):
        """N > 1: the row-sharded product gathered on rank 0 against the
        single-GPU product of the whole matrix (per row 1e-5)."""
        import torch
        import torch.distributed as dist

        self.step()
        ys = [None] * self.world
        dist.all_gather_object(ys, (self.r0, self.y.cpu().numpy()))
        if self.rank != 0:
            return None
        import mlx_sparse as ms

        d, i, p, x = self.full
        A = ms.csr_array((torch.from_numpy(d).to(self.dev), torch.from_numpy(i).to(self.dev),
                          torch.from_numpy(p).to(self.dev)), shape=self.shape, canonical=True)
        xd = torch.from_numpy(x).to(self.dev)
        y1 = (A @ xd).cpu().numpy()
        scale = (ms.csr_array((A.data.abs(), A.indices, A.indptr), shape=self.shape, canonical=True)
                 @ xd.abs()).cpu().numpy()
        yg = np.zeros_like(y1)
        for r0, yl in ys:
            yg[r0:r0 + yl.size] = yl
        err = float(np.max(np.abs(yg - y1) / np.maximum(np.maximum(np.abs(y1), scale), 1e-30)))
        del A
        return {"status": "ok" if err <= 1e-5 else "FAIL", "check": "gathered y vs 1-GPU product of the whole matrix",
                "max_rel_row_err": err}

    def cpu_sample(self, workers, budget_s=10.0):
        from oracle import oracle

        d, i, p, x = self.full
        times = []
        t_end = time.perf_counter() + budget_s
        while time.perf_counter() < t_end or len(times) < 3:
            t0 = time.perf_counter()
            oracle.csr_matvec(d, i, p, x, self.shape[0], workers=workers)
            times.append(time.perf_counter() - t0)
            if len(times) >= 500:
                break
        med = statistics.median(times)
        return self.problem_bytes / med / 1e9, f"full matrix, median of {len(times)} runs"


class PcgWorkload(Workload):
    """Jacobi-PCG on the 3D 7-point Poisson matrix (256^3),
    b = A x* with x* ~ U(-1, 1) from seed 1, x0 = 0, rtol 1e-6, maxiter 2000.
    A step is one full solve; value = iterations per second."""

    unit = "iters/s"
    unit_scale = 1.0
    dtype = "f32"
    scaling = "strong"

    def __init__(self, m=256):
        self.m = m
        self.name = "pcg_poisson3d"
        self.bytes_per_iter = None

    def config(self):
        return {"workload": self.name, "matrix": f"3D 7-point Poisson {self.m}^3 (n={self.m ** 3})",
                "solver": "Jacobi PCG, rtol 1e-6, maxiter 2000, x0 = 0", "index": "int32",
                "l2": "inputs (1.2 GB) exceed L2"}

    def setup_host(self):
        (d, i, p), (n, _) = wl.poisson3d(self.m)
        xs = wl.uniform_vector(n, 1)
        self.n, self.nnz = n, d.size
        self.bytes_per_iter = 8 * d.size + 4 * (n + 1) + 52 * n
        self.host = (d, i, p, xs)

    def setup(self, rank, world, device):
        import torch
        import mlx_sparse as ms

        self.setup_host()
        d, i, p, xs = self.host
        n = self.n
        self.world, self.dev, self.rank = world, device, rank
        if world == 1:
            self.A = ms.csr_array((torch.from_numpy(d).to(device), torch.from_numpy(i).to(device),
                                   torch.from_numpy(p).to(device)), shape=(n, n), canonical=True)
            self.b = self.A @ torch.from_numpy(xs).to(device)
            self.M = ms.linalg.preconditioners.jacobi(self.A)
            self.h_d, self.h_i, self.h_p = (torch.from_numpy(a).pin_memory() for a in (d, i, p))
            self.h_b = self.b.cpu().pin_memory()
            self.h_x = torch.empty(n, dtype=torch.float32).pin_memory()
            self.h2d_bytes = d.nbytes + i.nbytes + p.nbytes + 4 * n
            self.d2h_bytes = 4 * n
        else:
            from mlx_sparse import distributed as dd
            from mlx_sparse import _native

            slab = dd.build_slab(d, i, p, n, rank, world)
            self.r0 = slab.r0
            self.slab = dd.DeviceSlab(slab, device)
            xl = np.concatenate([xs[slab.r0:slab.r1], xs[slab.halo_cols]]).astype(np.float32)
            self.b = _native.csr_matvec(self.slab.data, self.slab.indices, self.slab.indptr,
                                        torch.from_numpy(xl).to(device), (slab.n_owned, xl.size))
            rows = np.repeat(np.arange(slab.n_owned), np.diff(slab.indptr.astype(np.int64)))
            diag = np.zeros(slab.n_owned, np.float32)
            own = slab.indices.astype(np.int64) == rows
            np.add.at(diag, rows[own], slab.data[own])
            self.inv = torch.from_numpy((np.float32(1.0) / diag).astype(np.float32)).to(device)
            self.mode = os.environ.get("MSX_DIST_COMM", "p2p")
            self.solver = dd.DistCG(self.slab, preconditioned=True, comm=self.mode)
            self.h_b = self.b.cpu().pin_memory()
            self.h_x = torch.empty(slab.n_owned, dtype=torch.float32).pin_memory()
            self.h2d_bytes = 4 * slab.n_owned
            self.d2h_bytes = 4 * slab.n_owned
        self.step()  # warm up and learn the (deterministic) iteration count
        self.units_per_step = float(self.iterations)
        self.local_bytes = self.bytes_per_iter * self.iterations / world
        # per iteration: SpMV(+dots), update, direction update; peer memory
        # fuses the scalar all-reduces and the halo push into those and adds
        # the halo unpack; NCCL adds the halo pack and two decision kernels
        # (NCCL's own kernels are not counted)
        per_it = 3 if world == 1 else (4 if self.mode == "p2p" else 6)
        self.launches_per_step = per_it * self.iterations + 6

    def step(self):
        import mlx_sparse as ms

        if self.world == 1:
            _, info = ms.linalg.cg(self.A, self.b, M=self.M, rtol=1e-6, maxiter=2000, return_info=True)
            self.iterations, self.info = info.iterations, info.status
        else:
            _, info, _, its = self.solver.solve(self.b, inv_diag_local=self.inv, rtol=1e-6, maxiter=2000)
            self.iterations, self.info = its, info

    def parity(self):
        """N > 1: the sharded solve against the same system solved on rank 0's
        GPU alone (status, iterations +-2, max |x - x_1|), and against the
        oracle's committed 256^3 result (tests/golden/pcg_poisson3d.json:
        status 0, 147 iterations, the first entries of x)."""
        import torch
        import torch.distributed as dist

        x, info, _, its = self.solver.solve(self.b, inv_diag_local=self.inv, rtol=1e-6, maxiter=2000)
        parts = [None] * self.world
        dist.all_gather_object(parts, (self.r0, x.cpu().numpy(), info, its))
        if self.rank != 0:
            return None
        import mlx_sparse as ms

        d, i, p, xs = self.host
        n = self.n
        xg = np.zeros(n, np.float32)
        for r0, xl, _, _ in parts:
            xg[r0:r0 + xl.size] = xl
        A = ms.csr_array((torch.from_numpy(d).to(self.dev), torch.from_numpy(i).to(self.dev),
                          torch.from_numpy(p).to(self.dev)), shape=(n, n), canonical=True)
        b = A @ torch.from_numpy(xs).to(self.dev)
        x1, inf1 = ms.linalg.cg(A, b, M=ms.linalg.preconditioners.jacobi(A), rtol=1e-6, maxiter=2000,
                                return_info=True)
        diff = float(np.max(np.abs(xg - x1.cpu().numpy())))
        out = {"check": "gathered x vs 1-GPU solve on rank 0, and vs the oracle's 256^3 fixture",
               "iterations": its, "iterations_1gpu": inf1.iterations, "info": info,
               "ranks_agree": all(pp[2:] == parts[0][2:] for pp in parts), "max_abs_dx_vs_1gpu": diff}
        ok = out["ranks_agree"] and info == inf1.status == 0 and abs(its - inf1.iterations) <= 2 and diff <= 1e-3
        gpath = os.path.join(ROOT, "tests", "golden", "pcg_poisson3d.json")
        if self.m == 256 and os.path.exists(gpath):
            with open(gpath) as f:
                g = json.load(f)["256"]
            head = float(np.max(np.abs(xg[:8] - np.asarray(g["x_head"], np.float32))))
            out.update(golden_iterations=g["iterations"], max_abs_dx_head_vs_golden=head)
            ok = ok and abs(its - g["iterations"]) <= 2 and head <= 1e-3
        del A
        out["status"] = "ok" if ok else "FAIL"
        return out

    def e2e_step(self):
        import mlx_sparse as ms

        if self.world > 1:
            # the matrix slabs stay resident in the persistent solver; each
            # step uploads this rank's b and reads back its x
            x, *_ = self.solver.solve(self.h_b.to(self.dev, non_blocking=True), inv_diag_local=self.inv,
                                      rtol=1e-6, maxiter=2000)
            self.h_x.copy_(x, non_blocking=True)
            return
        A = ms.csr_array((self.h_d.to(self.dev, non_blocking=True), self.h_i.to(self.dev, non_blocking=True),
                          self.h_p.to(self.dev, non_blocking=True)), shape=(self.n, self.n), canonical=True)
        x, _ = ms.linalg.cg(A, self.h_b.to(self.dev, non_blocking=True), M=ms.linalg.preconditioners.jacobi(A),
                            rtol=1e-6, maxiter=2000)
        self.h_x.copy_(x, non_blocking=True)

    def cpu_sample(self, workers, budget_s=10.0):
        from oracle import oracle

        d, i, p, xs = self.host
        b = oracle.csr_matvec(d, i, p, xs, self.n, workers=workers)
        inv = np.full(self.n, np.float32(1.0) / np.float32(6.0), np.float32)
        x0 = np.zeros(self.n, np.float32)
        t0 = time.perf_counter()
        oracle.csr_pcg_jacobi(d, i, p, b, x0, inv, rtol=1e-6, atol=0.0, maxiter=2000, stop_after=1)
        t1 = time.perf_counter() - t0
        k = int(max(2, min(2000, budget_s / max(t1, 1e-6))))
        t0 = time.perf_counter()
        _, _, _, its = oracle.csr_pcg_jacobi(d, i, p, b, x0, inv, rtol=1e-6, atol=0.0, maxiter=2000, stop_after=k)
        dt = time.perf_counter() - t0
        return its / dt, f"first {its} PCG iterations of the solve (serial loop, as the reference's)"


class SpgemmWorkload(Workload):
    """C = A @ A, A 2^18 x 2^18 with 8 uniform nonzeros per
    row; value = GB/s of compulsory bytes (A read as both operands, C written)."""

    unit = "GB/s"
    dtype = "f32"

    def __init__(self, n=1 << 18, per_row=8, seed=4):
        self.n, self.per_row, self.seed = n, per_row, seed
        self.name = "spgemm"
        self.local_bytes = None

    def config(self):
        return {"workload": self.name, "matrix": f"{self.n}x{self.n}, {self.per_row} nnz/row uniform",
                "output": "canonical CSR, exact zeros pruned", "index": "int32"}

    def setup_host(self):
        (d, i, p), _ = wl.random_k_per_row(self.n, self.n, self.per_row, self.seed)
        self.host = (d, i, p)
        self.products = int(np.sum(np.diff(p)[i]))

    def setup(self, rank, world, device):
        import torch
        import mlx_sparse as ms

        self.setup_host()
        d, i, p = self.host
        self.A = ms.csr_array((torch.from_numpy(d).to(device), torch.from_numpy(i).to(device),
                               torch.from_numpy(p).to(device)), shape=(self.n, self.n), canonical=True)
        C = self.A @ self.A
        nnz_a = d.size
        self.products = int(np.sum(np.diff(p)[i]))
        self.local_bytes = 2 * (8 * nnz_a + 4 * (self.n + 1)) + 8 * C.nnz + 4 * (self.n + 1)
        self.problem_bytes = self.local_bytes
        self.launches_per_step = 12
        self.h2d_bytes = d.nbytes + i.nbytes + p.nbytes
        self.d2h_bytes = 8 * C.nnz + 4 * (self.n + 1)
        self.dev = device

    def step(self):
        self.C = self.A @ self.A

    def e2e_step(self):
        import mlx_sparse as ms
        import torch

        d, i, p = self.host
        A = ms.csr_array((torch.from_numpy(d).to(self.dev), torch.from_numpy(i).to(self.dev),
                          torch.from_numpy(p).to(self.dev)), shape=(self.n, self.n), canonical=True)
        C = A @ A
        C.data.cpu(), C.indices.cpu(), C.indptr.cpu()

    def cpu_sample(self, workers, budget_s=10.0):
        from oracle import oracle

        d, i, p = self.host
        times = []
        t_end = time.perf_counter() + budget_s
        while time.perf_counter() < t_end or len(times) < 2:
            t0 = time.perf_counter()
            c = oracle.csr_matmat((d, i, p), (d, i, p), (self.n, self.n), (self.n, self.n))
            self.c_nnz = int(c[0].size)
            times.append(time.perf_counter() - t0)
        if self.local_bytes is None:  # reference arm: compulsory bytes from the oracle's own output
            self.local_bytes = 2 * (8 * d.size + 4 * (self.n + 1)) + 8 * self.c_nnz + 4 * (self.n + 1)
        return self.local_bytes / statistics.median(times) / 1e9, f"full product, median of {len(times)} runs, 1 thread"


WORKLOADS = {
    "spmm_f32": lambda: SpmmWorkload(bf16=False),
    "spmm_bf16": lambda: SpmmWorkload(bf16=True),
    "spmv_lap2d": lambda: SpmvWorkload("lap2d"),
    "spmv_powerlaw": lambda: SpmvWorkload("powerlaw"),
    "spmv_lap2d_xsharded": lambda: SpmvWorkload("lap2d", sharded=True),
    "spmv_powerlaw_xsharded": lambda: SpmvWorkload("powerlaw", sharded=True),
    "pcg_poisson3d": lambda: PcgWorkload(),
    "spgemm": lambda: SpgemmWorkload(),
}


# ---------------------------------------------------------------------------
# measurement
# ---------------------------------------------------------------------------
def _measure(wk, steps, warmup, device):
    import torch

    flush = torch.empty(512 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    for _ in range(warmup):
        flush.fill_(1)
        wk.step()
    torch.cuda.synchronize(device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for s in range(steps):
        flush.fill_(s & 0xFF)
        # keep the GPU busy while the host enqueues the step, so host-side
        # call overhead never shows up between the events
        torch.cuda._sleep(200000)
        starts[s].record(stream)
        wk.step()
        ends[s].record(stream)
    torch.cuda.synchronize(device)
    times = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    del flush
    return times


class _CopyStep:
    def __init__(self, nbytes, device):
        import torch

        half = max(16, nbytes // 2) // 16 * 16
        self.src = torch.ones(half, dtype=torch.uint8, device=device)
        self.dst = torch.empty_like(self.src)
        self.nbytes = 2 * half

    def step(self):
        self.dst.copy_(self.src)


def _copy_gbs(nbytes, steps, device):
    cs = _CopyStep(nbytes, device)
    t = _measure(cs, max(3, steps), 3, device)
    return cs.nbytes / (sum(t) / len(t) * 1e-3) / 1e9


def _measure_e2e(wk, steps, warmup, device):
    import torch

    stream = torch.cuda.current_stream(device)
    for _ in range(max(1, warmup)):
        wk.e2e_step()
    torch.cuda.synchronize(device)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        wk.e2e_step()
    b.record(stream)
    torch.cuda.synchronize(device)
    return a.elapsed_time(b) / steps


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_b200(args):
    import torch
    import torch.distributed as dist

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device)
    peak, peak_kind = _peaks()

    wk = WORKLOADS[args.workload]()
    wk.setup(rank, world, device)

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clocks:
        times = _measure(wk, args.steps, args.warmup, device)
    clock = clocks.summary()
    ms_step = sum(times) / len(times)
    t = torch.tensor([ms_step], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step_max = float(t.item())
    e2e_ms = _measure_e2e(wk, max(3, args.steps // 2), args.warmup, device)
    te = torch.tensor([e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item())

    problem_units = _units(wk)
    scale = getattr(wk, "unit_scale", 1e9)
    value = problem_units / (ms_step_max * 1e-3) / scale
    # roofline of the dominant kernel on this rank: its local algorithmic bytes
    local_bytes = getattr(wk, "local_bytes", None) or _local_bytes(wk)
    achieved = local_bytes / (ms_step * 1e-3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": wk.unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step_max, 5),
        "higher_is_better": True,
        "scaling": wk.scaling,
        "vs_baseline": None,
        "dtype": wk.dtype,
        "data": "synthetic (seeded numpy default_rng, BASELINE config shapes)",
        "config": dict(wk.config(), parallelism=f"row-shard x{world}, nnz-balanced" if world > 1 else "1 GPU"),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": _traffic(wk.name),
                     "peak_kind": peak_kind + " (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else peak_kind},
        "e2e": {"value": round(problem_units / (e2e_ms * 1e-3) / scale, 3), "unit": wk.unit,
                "h2d_bytes_per_step": int(wk.h2d_bytes), "d2h_bytes_per_step": int(wk.d2h_bytes),
                "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": int(wk.launches_per_step * args.steps),
        "clocks": clock,
    }
    if world > 1 and hasattr(wk, "parity"):
        line["parity"] = wk.parity()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        workers = len(os.sched_getaffinity(0))
        v, sample = wk.cpu_sample(workers, budget_s=args.cpu_budget)
        # the reference's auto worker count and, beside it, one worker
        v1, _ = wk.cpu_sample(1, budget_s=min(3.0, args.cpu_budget))
        line["cpu_baseline"] = {"value": round(v, 3), "unit": wk.unit, "cores": workers, "kind": "port",
                                "sample": sample + "; oracle/oracle.cpp restatement of the reference CPU loop",
                                "value_1_worker": round(v1, 3), "cpu_model": _cpu_model()}
    if not args.no_extras:
        # every rank takes part in the multi-GPU extras; rank 0 reports
        names = (["spmv_lap2d", "spmv_powerlaw", "spmm_bf16", "spmm_f32", "pcg_poisson3d", "spgemm"]
                 if world == 1 else ["pcg_poisson3d", "spmv_powerlaw", "spmv_powerlaw_xsharded",
                                     "spmv_lap2d_xsharded"])
        extras = {}
        for name in names:
            if name == args.workload:
                continue
            try:
                extras[name] = _extra(name, args, device, peak, rank, world)
            except Exception as exc:  # report, do not hide
                extras[name] = {"error": f"{type(exc).__name__}: {exc}"}
        line["workloads"] = extras
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _units(wk):
    """Metric units one step processes: bytes, or solver iterations."""
    return getattr(wk, "units_per_step", None) or wk.problem_bytes


def _local_bytes(wk):
    if isinstance(wk, SpmmWorkload):
        s = 2 if wk.bf16 else 4
        d = wk.host[0]
        return d.size * (s + 4) + 4 * (wk.rows + 1) + wk.n * wk.k * s + wk.rows * wk.k * s
    return wk.local_bytes


_TRAFFIC = {}


def _traffic(name):
    """DRAM bytes per launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not _TRAFFIC and os.path.exists(path):
        with open(path) as f:
            _TRAFFIC.update(json.load(f))
    return _TRAFFIC.get(name)


def _extra(name, args, device, peak, rank=0, world=1):
    import torch
    import torch.distributed as dist

    wk = WORKLOADS[name]()
    wk.setup(rank, world, device)
    steps = max(3, args.steps) if not isinstance(wk, PcgWorkload) else 3
    times = _measure(wk, steps, min(args.warmup, 3), device)
    ms_step = sum(times) / len(times)
    t = torch.tensor([ms_step], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    b = _local_bytes(wk)
    scale = getattr(wk, "unit_scale", 1e9)
    out = {"value": round(_units(wk) / (ms_max * 1e-3) / scale, 2), "unit": wk.unit,
           "ms_per_step": round(ms_max, 5), "n_gpus": world,
           "hbm_gbs_per_gpu": round(b / (ms_step * 1e-3) / 1e9, 1),
           "frac_of_peak": round(b / (ms_step * 1e-3) / 1e9 / peak, 4), "algorithmic_bytes_per_gpu": int(b),
           "config": wk.config(), "dtype": wk.dtype}
    if isinstance(wk, PcgWorkload):
        out.update({"iterations": wk.iterations, "info": wk.info, "bytes_per_iteration": int(wk.bytes_per_iter)})
    if world == 1 and b < (1 << 30) and not isinstance(wk, (PcgWorkload, SpgemmWorkload)):
        # small problems are bound by launch and round-trip latency as much
        # as by bandwidth: the same byte count as one device-to-device copy
        # (half read, half written), timed the same way, is the reachable
        # figure at this size
        cg = _copy_gbs(int(b), steps, device)
        out["copy_same_bytes"] = {"gbs": round(cg, 1), "frac_of_peak": round(cg / peak, 4),
                                  "kernel_frac_of_copy": round(b / (ms_step * 1e-3) / 1e9 / cg, 4)}
    if isinstance(wk, SpgemmWorkload):
        out["products_per_s"] = round(wk.products / (ms_max * 1e-3), 1)
    if world > 1 and hasattr(wk, "parity"):
        out["parity"] = wk.parity()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        workers = len(os.sched_getaffinity(0))
        v, sample = wk.cpu_sample(workers, budget_s=args.cpu_budget / 2)
        out["cpu_baseline"] = {"value": round(v, 3), "unit": wk.unit, "cores": workers, "kind": "port",
                               "sample": sample + "; oracle/oracle.cpp restatement of the reference CPU loop"}
        if not isinstance(wk, (PcgWorkload, SpgemmWorkload)):  # those are serial by construction
            v1, _ = wk.cpu_sample(1, budget_s=2.0)
            out["cpu_baseline"]["value_1_worker"] = round(v1, 3)
        else:
            out["cpu_baseline"]["cores"] = 1
    del wk
    torch.cuda.empty_cache()
    return out


def run_reference(args):
    world, rank, _ = _dist()
    if world > 1 and rank != 0:
        return
    wk = WORKLOADS[args.workload]()
    _setup_host_only(wk)
    workers = len(os.sched_getaffinity(0))
    vals = []
    sample = ""
    for _ in range(args.warmup):
        wk.cpu_sample(workers, budget_s=0.0)
    for _ in range(args.steps):
        v, sample = wk.cpu_sample(workers, budget_s=0.0)
        vals.append(v)
    v = statistics.median(vals)
    if isinstance(wk, (PcgWorkload, SpgemmWorkload)):
        workers = 1  # the reference's solver loop and the oracle's SpGEMM run on one thread
    line = {"metric": METRIC, "value": round(v, 3), "unit": wk.unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": wk.scaling, "vs_baseline": None,
            "dtype": wk.dtype, "data": "synthetic (seeded numpy default_rng, BASELINE config shapes)",
            "config": wk.config(), "impl": "reference",
            "cpu_baseline": {"value": round(v, 3), "unit": wk.unit, "cores": workers, "kind": "port",
                             "sample": sample + "; oracle/oracle.cpp restatement of the reference CPU loop "
                                                "(the reference itself needs MLX, absent here)",
                             "cpu_model": _cpu_model()},
            "e2e": {"value": round(v, 3), "unit": wk.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _setup_host_only(wk):
    wk.setup_host()
    if isinstance(wk, SpmmWorkload):
        wk.rows = wk.n


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="spmm_f32", choices=sorted(WORKLOADS))
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
