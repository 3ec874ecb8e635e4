"""Row-sharded products and CG across the GPUs of one node.

The reference scales only across CPU threads, by contiguous nnz-weighted row
ranges (``src/common/cpu_parallel.cpp:202-253``). Here the same partition is
applied to GPUs: rank ``r`` owns a contiguous slab of rows with about
``nnz / world`` nonzeros. Its local matrix keeps the owned columns first
(renumbered ``c - r0``) and appends the "halo" columns it reads from other
ranks, sorted by global column (hence grouped by owner).

The row-sharded CG (``DistCG``) keeps the reference's recurrence and status
codes; every rank takes identical scalar decisions. Two exchange modes:

- peer memory (default, one node): each rank maps its peers' halo arrays and
  mailboxes (CUDA IPC handles exchanged once through ``torch.distributed``);
  the direction update stores the entries peers read straight into their halo
  arrays as flagged words, the SpMV reads and checks them in place, and the
  reductions' last CTAs all-reduce the CG scalars through the mailboxes;
- NCCL: grouped send/recv of the halo and an all-reduce of the fp64 partial
  sums per reduction (also ``dist_cg``, the stateless form).

Host-side logic (partition, halo lists, landing offsets) is plain numpy and is
tested on CPU with ``gloo`` ranks; the solve itself runs in the CUDA library
(``msx_cg_context_*`` and ``msx_dist_*`` in ``include/msx_sparse.h``).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np


def partition_rows(indptr: np.ndarray, world: int) -> list[tuple[int, int]]:
    """Contiguous row ranges with about nnz / world nonzeros each."""
    indptr = np.asarray(indptr)
    n = indptr.shape[0] - 1
    nnz = int(indptr[-1])
    bounds = [0]
    for r in range(1, world):
        target = (nnz * r) // world
        b = int(np.searchsorted(indptr, target, side="left"))
        bounds.append(min(max(b, bounds[-1]), n))
    bounds.append(n)
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


@dataclass
class RowSlab:
    """One rank's rows of a square CSR matrix with local column numbering."""

    rank: int
    world: int
    r0: int
    r1: int
    data: np.ndarray
    indices: np.ndarray      # local columns: owned [0, n_owned), halo [n_owned, n_owned + n_halo)
    indptr: np.ndarray
    halo_cols: np.ndarray    # global column of each halo slot
    peers: np.ndarray        # ranks this rank exchanges with (ascending)
    send_counts: np.ndarray  # per peer: owned entries sent to it
    recv_counts: np.ndarray  # per peer: halo entries received from it (in halo order)
    send_idx: np.ndarray     # concatenated per peer: local owned indices to send
    dst_offset: np.ndarray   # per peer: where this rank's entries start in that peer's local vector

    @property
    def n_owned(self) -> int:
        return self.r1 - self.r0

    @property
    def n_halo(self) -> int:
        return int(self.halo_cols.shape[0])


def _cols_needed(indices, indptr, a0, a1, lo, hi):
    """Sorted unique columns in [lo, hi) referenced by rows [a0, a1)."""
    c = indices[int(indptr[a0]):int(indptr[a1])]
    c = c[(c >= lo) & (c < hi)]
    return np.unique(c)


def build_slab(data, indices, indptr, n: int, rank: int, world: int, ranges=None) -> RowSlab:
    """Cuts rank ``rank``'s slab out of the global (host) CSR arrays."""
    indptr = np.asarray(indptr)
    indices = np.asarray(indices)
    ranges = ranges or partition_rows(indptr, world)
    r0, r1 = ranges[rank]
    k0, k1 = int(indptr[r0]), int(indptr[r1])
    cols = indices[k0:k1].astype(np.int64)
    owned = (cols >= r0) & (cols < r1)
    halo_cols = np.unique(cols[~owned])
    local = np.empty(cols.shape[0], dtype=np.int64)
    local[owned] = cols[owned] - r0
    local[~owned] = (r1 - r0) + np.searchsorted(halo_cols, cols[~owned])
    peers, send_counts, recv_counts, send_idx, dst_offset = [], [], [], [], []
    for q in range(world):
        if q == rank:
            continue
        q0, q1 = ranges[q]
        lo, hi = np.searchsorted(halo_cols, q0), np.searchsorted(halo_cols, q1)
        n_recv = int(hi - lo)
        needed = _cols_needed(indices, indptr, q0, q1, r0, r1)
        if n_recv == 0 and needed.size == 0:
            continue
        peers.append(q)
        recv_counts.append(n_recv)
        send_counts.append(int(needed.size))
        send_idx.append((needed - r0).astype(np.int32))
        # Peer q's halo is sorted by global column, so this rank's entries
        # sit after q's owned rows and its halo columns below r0.
        qc = np.unique(indices[int(indptr[q0]):int(indptr[q1])])
        below = int(np.count_nonzero((qc < r0) & ((qc < q0) | (qc >= q1))))
        dst_offset.append((q1 - q0) + below)
    it = indices.dtype
    return RowSlab(
        rank=rank, world=world, r0=r0, r1=r1,
        data=np.ascontiguousarray(np.asarray(data)[k0:k1]),
        indices=local.astype(it),
        indptr=(indptr[r0:r1 + 1] - indptr[r0]).astype(it),
        halo_cols=halo_cols,
        peers=np.asarray(peers, dtype=np.int32),
        send_counts=np.asarray(send_counts, dtype=np.int64),
        recv_counts=np.asarray(recv_counts, dtype=np.int64),
        send_idx=np.concatenate(send_idx) if send_idx else np.zeros(0, np.int32),
        dst_offset=np.asarray(dst_offset, dtype=np.int64),
    )


# ---------------------------------------------------------------------------
# NCCL communicator and the distributed solve (GPU)
# ---------------------------------------------------------------------------
class Communicator:
    """An NCCL communicator owned by the CUDA library, one per rank.

    Created collectively: rank 0 draws the NCCL unique id and every rank
    receives it through the already initialised ``torch.distributed`` group
    (any backend), then joins with ``ncclCommInitRank`` on its current device.
    """

    def __init__(self, rank: int, world: int, device):
        import torch
        import torch.distributed as dist

        from mlx_sparse import _native

        L = _native.extension()
        buf = ctypes.create_string_buffer(128)
        if rank == 0:
            _native.check(L.msx_dist_unique_id(buf, 128))
        obj = [bytes(buf.raw) if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        uid = ctypes.create_string_buffer(obj[0], 128)
        h = ctypes.c_void_p()
        with torch.cuda.device(device):
            _native.check(L.msx_dist_comm_create(uid, world, rank, ctypes.byref(h)))
        self.handle, self.rank, self.world, self.device = h, rank, world, device

    def close(self):
        if self.handle:
            from mlx_sparse import _native

            _native.extension().msx_dist_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DeviceSlab:
    """A RowSlab uploaded to one GPU."""

    def __init__(self, slab: RowSlab, device, dtype=None):
        import torch

        self.slab = slab
        self.device = device
        self.data = torch.from_numpy(np.ascontiguousarray(slab.data)).to(device)
        if dtype is not None:
            self.data = self.data.to(dtype)
        self.indices = torch.from_numpy(np.ascontiguousarray(slab.indices)).to(device)
        self.indptr = torch.from_numpy(np.ascontiguousarray(slab.indptr)).to(device)
        self.send_idx = torch.from_numpy(np.ascontiguousarray(slab.send_idx, dtype=np.int32)).to(device)


class DistCG:
    """A persistent row-sharded CG / Jacobi PCG solver, one per rank.

    ``comm="p2p"`` (default on one node): every rank maps its peers' search
    direction and mailbox into its own address space (CUDA IPC handles,
    exchanged once through ``torch.distributed``); each iteration pushes the
    halo entries straight into the peers' vectors and reduces the CG scalars
    through the mailboxes, inside one captured CUDA graph with no host round
    trip. ``comm="nccl"`` does the same exchange with NCCL send/recv and
    all-reduce. Plan, buffers and the graph are built once; ``solve`` only
    runs iterations. Created collectively by all ranks.
    """

    def __init__(self, A: "DeviceSlab", *, preconditioned: bool, comm: str = "p2p", communicator=None):
        import torch.distributed as dist

        from mlx_sparse import _native

        s = A.slab
        if comm not in ("p2p", "nccl"):
            raise ValueError("comm must be 'p2p' or 'nccl'")
        if comm == "p2p" and s.world > 8:
            raise ValueError("peer-memory mode supports at most 8 ranks")
        if comm == "p2p":
            # ranks spin on each other's flags: each must own a distinct GPU
            import torch

            uuids = [None] * s.world
            dist.all_gather_object(uuids, str(torch.cuda.get_device_properties(A.device).uuid))
            if len(set(uuids)) != s.world:
                raise ValueError("peer-memory mode needs one GPU per rank; use comm='nccl'")
        self.A = A
        self.n_global = None
        mode = _native.CgContext.COMM_P2P if comm == "p2p" else _native.CgContext.COMM_NCCL
        if comm == "nccl" and communicator is None:
            communicator = Communicator(s.rank, s.world, A.device)
        self.communicator = communicator
        self.ctx = _native.CgContext(
            A.data, A.indices, A.indptr, s.n_owned, s.n_halo, preconditioned, comm=mode, rank=s.rank,
            world=s.world, nccl_comm=communicator.handle if communicator is not None else None, peers=s.peers,
            send_counts=s.send_counts, recv_counts=s.recv_counts, send_idx=A.send_idx, dst_offset=s.dst_offset)
        if comm == "p2p":
            handles = [None] * s.world
            dist.all_gather_object(handles, self.ctx.ipc_handles())
            self.ctx.connect(handles)
            dist.barrier()

    def solve(self, b_local, *, x0_local=None, inv_diag_local=None, rtol=1e-5, atol=0.0, maxiter=None):
        import torch

        n = self.A.slab.n_owned
        dev = self.A.device
        if maxiter is None:
            if self.n_global is None:
                import torch.distributed as dist

                t = torch.tensor([n], dtype=torch.int64)
                dist.all_reduce(t)
                self.n_global = int(t.item())
            maxiter = 10 * self.n_global
        x0 = torch.zeros(n, dtype=torch.float32, device=dev) if x0_local is None else x0_local
        return self.ctx.solve(b_local, x0, inv_diag_local, rtol=rtol, atol=atol, maxiter=maxiter)

    def close(self):
        self.ctx = None
        if self.communicator is not None:
            self.communicator.close()
            self.communicator = None


def dist_cg(comm: Communicator, A: DeviceSlab, b_local, *, x0_local=None, inv_diag_local=None, rtol=1e-5,
            atol=0.0, maxiter=None):
    """CG (or Jacobi PCG when ``inv_diag_local`` is given) over row slabs.

    Every rank passes its slab and its owned entries of b / x0 / inv_diag and
    gets back its owned entries of x plus the (identical) status, residual and
    iteration count.
    """
    import torch

    from mlx_sparse import _native

    L = _native.extension()
    s = A.slab
    n = s.n_owned
    dev = A.device
    b = b_local.to(dev, torch.float32).contiguous()
    x0 = (torch.zeros(n, dtype=torch.float32, device=dev) if x0_local is None
          else x0_local.to(dev, torch.float32).contiguous())
    inv = None if inv_diag_local is None else inv_diag_local.to(dev, torch.float32).contiguous()
    if maxiter is None:
        n_global = torch.tensor([n], dtype=torch.int64)
        import torch.distributed as dist

        dist.all_reduce(n_global)
        maxiter = 10 * int(n_global.item())
    x = torch.empty(n, dtype=torch.float32, device=dev)
    info, res, its = ctypes.c_int32(), ctypes.c_float(), ctypes.c_int32()
    peers = np.ascontiguousarray(s.peers, dtype=np.int32)
    sc = np.ascontiguousarray(s.send_counts, dtype=np.int64)
    rc = np.ascontiguousarray(s.recv_counts, dtype=np.int64)
    with torch.cuda.device(dev):
        _native.check(L.msx_dist_pcg(
            comm.handle, _native.INDEX_CODES[A.indices.dtype], A.data.data_ptr(), A.indices.data_ptr(),
            A.indptr.data_ptr(), A.data.numel(), n, s.n_halo, b.data_ptr(), x0.data_ptr(),
            inv.data_ptr() if inv is not None else None, x.data_ptr(), float(rtol), float(atol), int(maxiter),
            int(peers.shape[0]), peers.ctypes.data, sc.ctypes.data, rc.ctypes.data, A.send_idx.data_ptr(),
            ctypes.addressof(info), ctypes.addressof(res), ctypes.addressof(its), _native.stream_ptr(dev)))
    return x, info.value, res.value, its.value


# ---------------------------------------------------------------------------
# Row-sharded SpMV / SpMM with the dense operand sharded too (GPU, NCCL)
# ---------------------------------------------------------------------------
def allgather_layout(indices, indptr, ranges, r0: int, r1: int):
    """Column renumbering of rows [r0, r1) for the all-gather exchange.

    Every rank contributes its owned block of x padded to ``max_rows`` =
    the longest row range, so after ``all_gather_into_tensor`` global column
    ``c`` owned by rank ``q`` sits at ``q * max_rows + (c - start_q)``.
    Returns the renumbered indices of the slab (same dtype) and ``max_rows``.
    """
    indptr = np.asarray(indptr)
    starts = np.asarray([a for a, _ in ranges], dtype=np.int64)
    max_rows = max(b - a for a, b in ranges) if ranges else 0
    cols = np.asarray(indices[int(indptr[r0]):int(indptr[r1])]).astype(np.int64)
    owner = np.searchsorted(starts, cols, side="right") - 1
    local = owner * max_rows + (cols - starts[owner])
    return local.astype(np.asarray(indices).dtype), int(max_rows)


class OperandExchange:
    """Gathers, for one rank's row slab, the entries of a row-sharded dense
    operand (x, or the rows of B) that the slab's columns read.

    Each rank owns rows ``r0:r1`` of A and the same entries of x. Two
    exchanges over ``torch.distributed`` (NCCL on GPUs; gloo works for CPU
    tensors):

    - ``"halo"``: one ``all_to_all_single`` carrying exactly the entries each
      peer reads (the slab's send lists, landing in halo order); suits banded
      matrices (stencils), where a rank reads a few planes of its neighbours;
    - ``"allgather"``: ``all_gather_into_tensor`` of the owned blocks padded
      to the longest row range; suits random columns, which read almost all
      of x anyway;
    - ``"auto"``: halo when the halo is under a quarter of the global vector.

    ``local_indices`` is the slab's column numbering into the buffer that
    ``exchange`` fills. Created collectively by all ranks.
    """

    def __init__(self, data, indices, indptr, n: int, rank: int, world: int, device, *, mode: str = "auto",
                 ranges=None):
        import torch
        import torch.distributed as dist

        if mode not in ("auto", "halo", "allgather"):
            raise ValueError("mode must be 'auto', 'halo' or 'allgather'")
        indptr = np.asarray(indptr)
        self.ranges = ranges or partition_rows(indptr, world)
        self.rank, self.world, self.device, self.n = rank, world, device, n
        self.r0, self.r1 = self.ranges[rank]
        slab = build_slab(data, indices, indptr, n, rank, world, self.ranges)
        halo_total = torch.tensor([slab.n_halo], dtype=torch.int64, device=device)
        dist.all_reduce(halo_total)
        if mode == "auto":
            mode = "halo" if int(halo_total.item()) * 4 < n else "allgather"
        self.mode = mode
        self.slab = slab
        if mode == "halo":
            self.local_indices = slab.indices
            self.n_local_cols = slab.n_owned + slab.n_halo
            send = np.zeros(world, np.int64)
            recv = np.zeros(world, np.int64)
            send[slab.peers] = slab.send_counts
            recv[slab.peers] = slab.recv_counts
            self.send_splits, self.recv_splits = send.tolist(), recv.tolist()
            self.send_idx = torch.from_numpy(slab.send_idx.astype(np.int64)).to(device)
        else:
            self.local_indices, self.max_rows = allgather_layout(indices, indptr, self.ranges, self.r0, self.r1)
            self.n_local_cols = self.max_rows * world
        self._buf = {}

    def _get(self, key, shape, dtype):
        import torch

        if key not in self._buf:
            self._buf[key] = torch.zeros(shape, dtype=dtype, device=self.device)
        return self._buf[key]

    def exchange(self, x_owned):
        """Returns the local operand for x_owned (rows r0:r1 of x or B): owned
        entries and those read from other ranks, in ``local_indices``
        numbering. The buffer is reused by the next call."""
        import torch.distributed as dist

        tail = tuple(x_owned.shape[1:])
        buf = self._get(("buf", tail, x_owned.dtype), (self.n_local_cols,) + tail, x_owned.dtype)
        n_own = self.r1 - self.r0
        if self.mode == "halo":
            buf[:n_own].copy_(x_owned)
            send = x_owned.index_select(0, self.send_idx)
            dist.all_to_all_single(buf[n_own:], send, self.recv_splits, self.send_splits)
        else:
            mine = self._get(("own", tail, x_owned.dtype), (self.max_rows,) + tail, x_owned.dtype)
            mine[:n_own].copy_(x_owned)  # the padding is never read
            dist.all_gather_into_tensor(buf, mine)
        return buf


class DistProduct(OperandExchange):
    """``y = A @ x`` and ``Y = A @ B`` over row slabs with x (or the rows of B)
    sharded by the same row ranges as A: the distributed form of the
    reference's ``csr_matvec`` / ``csr_matmul`` (``src/sparse/csr_matvec/
    csr_matvec.cpp:79-168``, ``src/sparse/csr_matmul/csr_matmul.cpp:83-222``),
    whose CPU path splits rows by the same nnz-weighted ranges across threads
    (``src/common/cpu_parallel.cpp:202-253``).

    Each rank passes its owned entries of x and gets its owned entries of y.
    The operand exchange (``OperandExchange``) runs over NCCL; the local
    product is the library's SpMV (with a cached row-bin plan) or SpMM.
    """

    def __init__(self, data, indices, indptr, n: int, rank: int, world: int, device, *, mode: str = "auto",
                 ranges=None, dtype=None):
        import torch

        import mlx_sparse as ms

        super().__init__(data, indices, indptr, n, rank, world, device, mode=mode, ranges=ranges)
        slab = self.slab
        vals = torch.from_numpy(np.ascontiguousarray(slab.data)).to(device)
        if dtype is not None:
            vals = vals.to(dtype)
        idx = torch.from_numpy(np.ascontiguousarray(self.local_indices)).to(device)
        ip = torch.from_numpy(np.ascontiguousarray(slab.indptr)).to(device)
        self.A = ms.csr_array((vals, idx, ip), shape=(slab.n_owned, self.n_local_cols), canonical=True)
        if slab.n_owned > 0:
            self.A.spmv_plan()

    def matvec(self, x_owned):
        return self.A @ self.exchange(x_owned)

    def matmul(self, b_owned):
        return self.A @ self.exchange(b_owned)
