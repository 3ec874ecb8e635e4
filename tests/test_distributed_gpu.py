"""Multi-GPU CG / Jacobi PCG (row slabs, NCCL halo exchange + all-reduce) vs
the CPU oracle: same status, iterations within +-2, solution within 1e-3.
Runs one process per GPU on 2 GPUs; skipped when fewer are visible."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import workloads as wl

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, q, mode="stateless"):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "mlx-sparse_b200"), os.path.join(root, "tests")]
    import torch.distributed as dist

    from mlx_sparse import distributed as dd

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kind, precond = case
        (d, i, p), (n, _) = wl.poisson3d(20) if kind == "p3d" else wl.lap2d(40)
        xs = wl.uniform_vector(n, 1)
        from oracle import oracle

        b = oracle.csr_matvec(d, i, p, xs, n)
        slab = dd.build_slab(d, i, p, n, rank, world)
        A = dd.DeviceSlab(slab, dev)
        comm = dd.Communicator(rank, world, dev)
        inv = None
        if precond:
            inv = torch.full((slab.n_owned,), 1.0 / float(d.max()), dtype=torch.float32, device=dev)
        bl = torch.from_numpy(b[slab.r0:slab.r1].copy())
        if mode == "stateless":
            x, info, res, its = dd.dist_cg(comm, A, bl, inv_diag_local=inv, rtol=1e-6, maxiter=2000)
        else:
            solver = dd.DistCG(A, preconditioned=precond, comm=mode,
                               communicator=comm if mode == "nccl" else None)
            # two solves through one context: the second must repeat the first
            first = solver.solve(bl.to(dev), inv_diag_local=inv, rtol=1e-6, maxiter=2000)
            x, info, res, its = solver.solve(bl.to(dev), inv_diag_local=inv, rtol=1e-6, maxiter=2000)
            assert torch.equal(first[0], x) and first[1:] == (info, res, its)
            solver.ctx = None
            torch.cuda.synchronize()
        parts = [None] * world
        dist.all_gather_object(parts, (slab.r0, x.cpu().numpy(), info, res, its))
        comm.close()
        if rank == 0:
            xg = np.zeros(n, np.float32)
            for r0, xl, *_ in parts:
                xg[r0:r0 + xl.size] = xl
            x0 = np.zeros(n, np.float32)
            if precond:
                ref = oracle.csr_pcg_jacobi(d, i, p, b, x0, np.full(n, 1.0 / float(d.max()), np.float32),
                                            rtol=1e-6, atol=0.0, maxiter=2000)
            else:
                ref = oracle.csr_cg(d, i, p, b, x0, rtol=1e-6, atol=0.0, maxiter=2000)
            same = all(pp[2:] == parts[0][2:] for pp in parts)
            q.put((same, info, its, ref[1], ref[3], float(np.max(np.abs(xg - ref[0])))))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["stateless", "nccl", "p2p"])
@pytest.mark.parametrize("case", [("p3d", True), ("p3d", False), ("lap2d", True)])
def test_dist_cg_matches_oracle(case, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.spawn(_worker, args=(2, _free_port(), case, q, mode), nprocs=2, join=True)
    same, info, its, info_r, its_r, err = q.get(timeout=120)
    assert same, "ranks disagree on the scalars"
    assert info == info_r
    assert abs(its - its_r) <= 2
    assert err <= 1e-3


def _product_worker(rank, world, port, kind, mode, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "mlx-sparse_b200"), os.path.join(root, "tests")]
    import torch.distributed as dist

    from mlx_sparse.distributed import DistProduct
    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        (d, i, p), (n, _) = wl.lap2d(96) if kind == "lap2d" else wl.power_law(30000, 3, np.int64)
        x = wl.uniform_vector(n, 2)
        B = wl.uniform_matrix(n, 16, 3)
        P = DistProduct(d, i, p, n, rank, world, dev, mode=mode)
        y = P.matvec(torch.from_numpy(x[P.r0:P.r1].copy()).to(dev)).cpu().numpy()
        Y = P.matmul(torch.from_numpy(B[P.r0:P.r1].copy()).to(dev)).cpu().numpy()
        parts = [None] * world
        dist.all_gather_object(parts, (P.r0, y, Y))
        if rank == 0:
            yg = np.zeros(n, np.float32)
            Yg = np.zeros((n, 16), np.float32)
            for r0, yl, Yl in parts:
                yg[r0:r0 + yl.size] = yl
                Yg[r0:r0 + yl.size] = Yl
            y_ref = oracle.csr_matvec(d, i, p, x, n)
            Y_ref = oracle.csr_matmul(d, i, p, B, n)
            scale = oracle.csr_matvec(np.abs(d), i, p, np.abs(x), n) + 1e-30
            q.put((float(np.max(np.abs(yg - y_ref) / np.maximum(np.abs(y_ref), scale))),
                   bool(np.array_equal(Yg, Y_ref))))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("kind,mode", [("lap2d", "halo"), ("powerlaw", "allgather"), ("lap2d", "auto")])
def test_dist_product_matches_oracle(kind, mode):
    """Row-sharded SpMV / SpMM with x and B sharded too (NCCL exchange):
    the gathered y within 1e-5 per row, Y bit-exact, against the oracle."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.spawn(_product_worker, args=(2, _free_port(), kind, mode, q), nprocs=2, join=True)
    err, spmm_exact = q.get(timeout=120)
    assert err <= 1e-5
    assert spmm_exact
