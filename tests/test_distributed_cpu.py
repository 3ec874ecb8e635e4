"""Host logic of the row-sharded solver, on CPU with gloo ranks.

Each rank cuts its slab (mlx_sparse.distributed.build_slab), exchanges halo
entries of x with its peers by send/recv exactly as the device solve does
(send list order -> halo order), computes its local SpMV with the CPU oracle,
and rank 0 checks the gathered result against the global product.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import workloads as wl


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _make(kind):
    if kind == "poisson":
        return wl.poisson3d(10)
    if kind == "ragged":
        (d, i, p), s = wl.ragged_csr(900, 900, 5, 20)
        return (d, i, p), s
    return wl.random_k_per_row(700, 700, 9, 4)


def _worker(rank, world, port, kind, results):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "mlx-sparse_b200"), os.path.join(root, "tests")]
    from mlx_sparse.distributed import build_slab, partition_rows
    from oracle import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        (d, i, p), (n, _) = _make(kind)
        x = wl.uniform_vector(n, 7)
        ranges = partition_rows(p, world)
        slab = build_slab(d, i, p, n, rank, world, ranges)
        own = x[slab.r0:slab.r1]
        # halo exchange: send owned[send_idx] per peer, receive into halo order
        halo = np.zeros(slab.n_halo, np.float32)
        reqs, bufs, so, ro = [], [], 0, 0
        for q, sc, rc in zip(slab.peers, slab.send_counts, slab.recv_counts):
            if sc:
                t = torch.from_numpy(own[slab.send_idx[so:so + sc]].copy())
                reqs.append(dist.isend(t, int(q)))
            if rc:
                buf = torch.zeros(int(rc))
                bufs.append((ro, buf))
                reqs.append(dist.irecv(buf, int(q)))
            so += int(sc)
            ro += int(rc)
        for r in reqs:
            r.wait()
        for off, buf in bufs:
            halo[off:off + buf.numel()] = buf.numpy()
        xl = np.concatenate([own, halo]).astype(np.float32)
        assert np.array_equal(halo, x[slab.halo_cols])
        y_local = oracle.csr_matvec(slab.data, slab.indices, slab.indptr, xl, slab.n_owned)
        gathered = [None] * world
        dist.all_gather_object(gathered, (slab.r0, y_local))
        if rank == 0:
            y = np.zeros(n, np.float32)
            for r0, yl in gathered:
                y[r0:r0 + yl.size] = yl
            ref = oracle.csr_matvec(d, i, p, x, n)
            results.put(bool(np.array_equal(y, ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("kind", ["poisson", "ragged", "random"])
def test_halo_exchange_reproduces_global_spmv(world, kind):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.spawn(_worker, args=(world, _free_port(), kind, q), nprocs=world, join=True)
    assert q.get(timeout=60) is True


def test_partition_balances_nnz():
    from mlx_sparse.distributed import partition_rows

    (d, i, p), (n, _) = wl.power_law(20000, 3)
    for world in (1, 2, 4, 8):
        ranges = partition_rows(p, world)
        assert ranges[0][0] == 0 and ranges[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        loads = [int(p[b] - p[a]) for a, b in ranges]
        assert max(loads) <= int(p[-1]) / world + int(np.diff(p).max()) + 1


@pytest.mark.parametrize("world", [2, 3, 5])
@pytest.mark.parametrize("kind", ["poisson", "ragged", "random"])
def test_landing_offsets_match_peer_halo_order(world, kind):
    """Peer-memory halo push: rank r's entries, written at dst_offset in peer
    q's local vector, must land exactly on q's halo slots for those columns."""
    from mlx_sparse.distributed import build_slab, partition_rows

    (d, i, p), (n, _) = _make(kind)
    ranges = partition_rows(p, world)
    slabs = [build_slab(d, i, p, n, r, world, ranges) for r in range(world)]
    for s in slabs:
        so = 0
        for q, sc, off in zip(s.peers, s.send_counts, s.dst_offset):
            t = slabs[int(q)]
            cols = s.r0 + s.send_idx[so:so + sc].astype(np.int64)
            h0 = int(off) - t.n_owned
            assert h0 >= 0
            assert np.array_equal(t.halo_cols[h0:h0 + sc], cols)
            so += int(sc)


def _exchange_worker(rank, world, port, kind, mode, results):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "mlx-sparse_b200"), os.path.join(root, "tests")]
    from mlx_sparse.distributed import OperandExchange
    from oracle import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        (d, i, p), (n, _) = _make(kind)
        x = wl.uniform_vector(n, 7)
        B = wl.uniform_matrix(n, 3, 8)
        ex = OperandExchange(d, i, p, n, rank, world, torch.device("cpu"), mode=mode)
        s = ex.slab
        xl = ex.exchange(torch.from_numpy(x[s.r0:s.r1].copy())).numpy().copy()
        y_local = oracle.csr_matvec(s.data, ex.local_indices, s.indptr, xl, s.n_owned)
        Bl = ex.exchange(torch.from_numpy(B[s.r0:s.r1].copy())).numpy()
        Y_local = oracle.csr_matmul(s.data, ex.local_indices, s.indptr, Bl, s.n_owned)
        gathered = [None] * world
        dist.all_gather_object(gathered, (s.r0, y_local, Y_local, ex.mode))
        if rank == 0:
            y = np.zeros(n, np.float32)
            Y = np.zeros((n, 3), np.float32)
            for r0, yl, Yl, _ in gathered:
                y[r0:r0 + yl.size] = yl
                Y[r0:r0 + yl.size] = Yl
            ok = (np.array_equal(y, oracle.csr_matvec(d, i, p, x, n))
                  and np.array_equal(Y, oracle.csr_matmul(d, i, p, B, n))
                  and all(g[3] == (mode if mode != "auto" else g[3]) for g in gathered))
            results.put(ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("mode", ["halo", "allgather", "auto"])
@pytest.mark.parametrize("kind", ["poisson", "random"])
def test_sharded_operand_exchange_reproduces_global_products(world, mode, kind):
    """DistProduct's operand exchange (x and B rows sharded like A's rows):
    after the exchange, each rank's local SpMV / SpMM with the renumbered
    columns equals its rows of the global product, bit for bit."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.spawn(_exchange_worker, args=(world, _free_port(), kind, mode, q), nprocs=world, join=True)
    assert q.get(timeout=60) is True
