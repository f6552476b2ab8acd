"""N-sharding of a GEMM over the ranks of one node (one process per GPU).

Rank r of g owns rows [r*N/g, (r+1)*N/g) of B (the weights) and computes the column block
C[:, shard] = A . B[shard]^T with its own kernel launch: no data moves between GPUs during the
GEMM. Where every rank needs the whole C, `gather_columns` collects the blocks with one
all-gather (NCCL over NVLink on GPUs) and re-lays them out as row-major [M, N]; `SharedC` (CUDA IPC
peer mappings, one TMA store per peer) and `MulticastC` (an NVSwitch multicast object, one
multimem store for all GPUs) let the GEMM's own epilogue deliver the tiles instead.
"""

from __future__ import annotations


def shard_range(n: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """[lo, hi) of the N dimension owned by `rank`. Boundaries are multiples of `align` (the last
    shard takes the remainder); with align = 1 shards differ in size by at most one row."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")

    def bound(r):
        if r >= world:
            return n
        return min(n, (n * r // world + align // 2) // align * align)

    return bound(rank), bound(rank + 1)


def max_over_ranks(x: float, dist=None, device=None) -> float:
    """The maximum of a per-rank float over the process group (the job is as slow as its slowest rank)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    import torch

    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_columns(c_shard, n: int, dist, align: int = 1, out=None, work=None):
    """All-gather the column blocks C[:, shard_r] of every rank into the full row-major C[M, N].

    Shards may differ in width by one column, so each is padded to the widest before the
    collective and cut back afterwards. `out` ([M, N]) and `work` ([world, M, widest shard], NCCL
    only) are optional preallocated buffers: a loop that passes them allocates nothing per call, and
    equal shards are re-laid out with one strided copy."""
    import torch

    world = dist.get_world_size()
    m = c_shard.shape[0]
    widths = [shard_range(n, world, r, align)[1] - shard_range(n, world, r, align)[0] for r in range(world)]
    wmax = max(widths)
    if c_shard.shape[1] != wmax:
        padded = torch.zeros((m, wmax), dtype=c_shard.dtype, device=c_shard.device)
        padded[:, : c_shard.shape[1]] = c_shard
    else:
        padded = c_shard.contiguous()
    if dist.get_backend() == "nccl":
        gathered = work if work is not None else torch.empty((world, m, wmax), dtype=c_shard.dtype,
                                                             device=c_shard.device)
        dist.all_gather_into_tensor(gathered, padded)
        if out is not None and all(w == wmax for w in widths):
            out.view(m, world, wmax).copy_(gathered.permute(1, 0, 2))
            return out
        parts = list(gathered.unbind(0))
    else:
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded)
    full = torch.cat([p[:, :w] for p, w in zip(parts, widths)], dim=1)
    if out is not None:
        out.copy_(full)
        return out
    return full


class SharedC:
    """A full C [M, N] on every rank, each one writable by every other rank's GEMM epilogue.

    Every rank allocates its own C and shares a CUDA IPC handle of it (all_gather_object over the
    process group); each rank maps the others' buffers. `peer_ptrs(lo)` gives, for column lo, the
    address of that column in every other rank's C: what kl_gemm_gather writes the tiles of the
    rank's shard to. Ranks must be processes on GPUs of one node with NVLink peer access."""

    def __init__(self, m: int, n: int, dtype, device, dist):
        import torch

        import maia_b200 as kl

        self.kl = kl
        self.world = dist.get_world_size()
        self.rank = dist.get_rank()
        self.full = torch.empty((m, n), dtype=dtype, device=device)
        handles = [None] * self.world
        dist.all_gather_object(handles, kl.ipc_handle(self.full.data_ptr()))
        # Peers in the order rank + 1, rank + 2, ... (mod g): the epilogue stores to them in this
        # order, so at any moment the ranks are sending to different GPUs rather than all to one.
        order = [(self.rank + i) % self.world for i in range(1, self.world)]
        self.bases = [kl.ipc_open(handles[r][0]) for r in order]
        self.peers = [base + handles[r][1] for base, r in zip(self.bases, order)]
        self.elem = self.full.element_size()

    def peer_ptrs(self, col0: int) -> list[int]:
        return [p + col0 * self.elem for p in self.peers]

    def close(self) -> None:
        for p in self.bases:
            self.kl.ipc_close(p)
        self.bases = []
        self.peers = []


class MulticastC:
    """A full C [M, N] on every rank, bound to one NVLink multicast object (torch's symmetric
    memory, which allocates it with the CUDA virtual-memory API, exchanges the handles over the
    process group and binds every GPU's copy). A multimem store to `mc_ptr(col)` + offsets lands in
    every rank's C at once: what kl_gemm_gather_multicast writes the tiles of a rank's shard to.

    `available` is False (and `reason` says why) where the GPUs or the driver offer no multicast;
    then nothing is bound. Every rank must call `close()` (collectively) before the process group
    ends: a process must not exit while its memory is still bound to the multicast object."""

    def __init__(self, m: int, n: int, dtype, device, dist):
        import torch

        self.dist = dist
        self.full = None
        self._hdl = None
        self.available = False
        self.reason = None
        try:
            import torch.distributed._symmetric_memory as symm_mem

            group = dist.group.WORLD
            if not symm_mem.is_symm_mem_enabled_for_group(group.group_name):
                symm_mem.enable_symm_mem_for_group(group.group_name)
            self.full = symm_mem.empty((m, n), dtype=dtype, device=device)
            self._hdl = symm_mem.rendezvous(self.full, group.group_name)
        except Exception as e:  # no symmetric memory on this platform
            self.reason = f"symmetric memory: {type(e).__name__}: {e}"
        ok = self._hdl is not None and int(self._hdl.multicast_ptr) != 0
        if self._hdl is not None and not ok:
            self.reason = "no multicast object (the GPUs or the driver offer no NVLink multicast)"
        if ok and self.full.data_ptr() != int(self._hdl.buffer_ptrs[dist.get_rank()]):
            # The multicast address is that of the allocation's start; use only a tensor that starts
            # there, so that tensor offsets and multicast offsets agree.
            ok = False
            self.reason = "the symmetric tensor does not start its allocation"
        # Every rank must agree before anyone uses the multicast path.
        flag = torch.tensor([1.0 if ok else 0.0], device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        self.available = bool(flag.item() == 1.0)
        if ok and not self.available:
            self.reason = "another rank has no multicast object"
        if self.available:
            rank = dist.get_rank()
            base = int(self._hdl.buffer_ptrs[rank])
            self._offset = self.full.data_ptr() - base
            nbytes = self.full.numel() * self.full.element_size()
            if self._offset < 0 or self._offset + nbytes > int(self._hdl.buffer_size):
                raise RuntimeError("symmetric buffer does not contain the tensor")
            self._mc = int(self._hdl.multicast_ptr) + self._offset
            self.elem = self.full.element_size()
            self.n = n

    def mc_ptr(self, col0: int) -> int:
        """Multicast address of element (0, col0) of C."""
        if not self.available:
            raise RuntimeError(f"no multicast C: {self.reason}")
        return self._mc + col0 * self.elem

    def close(self) -> None:
        import gc

        import torch

        if self.full is None and self._hdl is None:
            return
        torch.cuda.synchronize()
        self.dist.barrier()
        self._hdl = None
        self.full = None
        gc.collect()
        torch.cuda.synchronize()
        self.dist.barrier()


class HostShardedGemm:
    """End-to-end N-sharded GEMM from host memory, the operands crossing PCIe once per job.

    Rank r of g holds (pinned host buffers) rows [r M_pad / g, (r + 1) M_pad / g) of A, its column
    shard of B and its column block of C. Each call, on the device: the rank's slab of A is copied in
    and all-gathered into the whole A over NVLink (NCCL, on a side stream), while the shard of B
    streams in over PCIe in column blocks and each block's GEMM and copy of C back out follow
    (kl_gemm_host_b; the GEMMs wait for the gathered A). So A moves over PCIe once in total instead
    of once per GPU. The caller's stream waits for C to be on the host."""

    def __init__(self, m: int, n_shard: int, k: int, ab_dtype, c_dtype, device, dist):
        import torch

        self.dist = dist
        self.world = dist.get_world_size() if dist is not None else 1
        self.rank = dist.get_rank() if dist is not None else 0
        self.m, self.k = m, k
        self.m_pad = -(-m // self.world) * self.world
        self.rows = self.m_pad // self.world
        self.device = device
        self.a_full = torch.empty((self.m_pad, k), dtype=ab_dtype, device=device)
        self.b_dev = torch.empty((n_shard, k), dtype=ab_dtype, device=device)
        self.c_dev = torch.empty((m, n_shard), dtype=c_dtype, device=device)
        self.side = torch.cuda.Stream(device)
        self.a_ready = torch.cuda.Event()

    def slab_rows(self) -> tuple[int, int]:
        """[lo, hi) rows of A this rank brings from its host (hi <= M)."""
        lo = self.rank * self.rows
        return lo, min(self.m, lo + self.rows)

    def __call__(self, a_slab_host, b_host, c_host, **kw):
        import torch

        import maia_b200 as kl

        lo, hi = self.slab_rows()
        if tuple(a_slab_host.shape) != (hi - lo, self.k):
            raise ValueError(f"A slab must be [{hi - lo}, {self.k}], got {tuple(a_slab_host.shape)}")
        main = torch.cuda.current_stream(self.device)
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            mine = self.a_full[self.rank * self.rows:(self.rank + 1) * self.rows]
            if hi > lo:
                mine[: hi - lo].copy_(a_slab_host, non_blocking=True)
            if self.world > 1:
                self.dist.all_gather_into_tensor(self.a_full, mine)
            self.a_ready.record(self.side)
        kl.gemm_host_b(self.a_full[: self.m], b_host, c_host, self.b_dev, self.c_dev, a_ready=self.a_ready,
                       stream=main.cuda_stream, **kw)
        return c_host


class RankLost(RuntimeError):
    """A rank of the group did not check in for a step in time (it raised, exited or never joined)."""

    def __init__(self, step: int, missing: list[int], left: list[int]):
        why = []
        if left:
            why.append(f"rank(s) {left} left")
        if missing:
            why.append(f"rank(s) {missing} did not check in")
        super().__init__(f"step {step}: " + "; ".join(why))
        self.step = step
        self.missing = missing
        self.left = left


class StepGuard:
    """Failure detection on the host, between steps: before launching step s, every rank checks in
    on the process group's key-value store and waits (at most `timeout_s`) until every rank has
    checked in for s. A rank that raised, exited or never joined is noticed there, with nothing of
    step s launched on any GPU, as RankLost. A rank that leaves on purpose calls `leave()`, which the
    others see at once instead of at the deadline. The store lives in rank 0's process (torch's
    TCPStore), so rank 0 is the one rank that cannot leave early."""

    def __init__(self, dist, timeout_s: float = 10.0, prefix: str = "kl/guard", store=None):
        self.world = dist.get_world_size()
        self.rank = dist.get_rank()
        self.timeout_s = timeout_s
        self.prefix = prefix
        if store is None:
            from torch.distributed import distributed_c10d as c10d

            store = c10d._get_default_store()
        self.store = store

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/step{step}/{rank}"

    def _left_key(self, rank: int) -> str:
        return f"{self.prefix}/left/{rank}"

    def leave(self) -> None:
        self.store.set(self._left_key(self.rank), "1")

    def check(self, step: int) -> None:
        import time

        self.store.set(self._key(step, self.rank), "1")
        pending = [r for r in range(self.world) if r != self.rank]
        deadline = time.monotonic() + self.timeout_s
        while pending:
            left = [r for r in pending if self.store.check([self._left_key(r)])]
            if left:
                raise RankLost(step, [r for r in pending if r not in left], left)
            pending = [r for r in pending if not self.store.check([self._key(step, r)])]
            if pending and time.monotonic() >= deadline:
                raise RankLost(step, pending, [])
            if pending:
                time.sleep(0.005)


class Comm:
    """kl_comm: an NCCL communicator whose waits are bounded (the C ABI's kl_comm_*). Rank 0 makes
    the unique id and the process group carries it to the others. `wait` returns normally, or
    raises KlError with KL_ERR_TIMEOUT / KL_ERR_NCCL after aborting the communicator."""

    def __init__(self, dist, device, timeout_ms: int = 30000):
        import ctypes

        import maia_b200 as kl

        self.kl = kl
        self.device = device
        rank, world = dist.get_rank(), dist.get_world_size()
        buf = ctypes.create_string_buffer(128)
        if rank == 0:
            kl.check(kl.lib().kl_comm_get_unique_id(buf))
        obj = [buf.raw if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        buf = ctypes.create_string_buffer(obj[0], 128)
        self._h = ctypes.c_void_p()
        kl.check(kl.lib().kl_comm_init(buf, world, rank, int(timeout_ms), ctypes.byref(self._h)))
        self.world, self.rank = world, rank

    def _stream(self, stream):
        import torch

        return stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream

    def all_gather(self, send, recv, stream=None) -> None:
        """recv = the world's `send` tensors in rank order (recv holds world x send's bytes)."""
        import ctypes

        nbytes = send.numel() * send.element_size()
        if recv.numel() * recv.element_size() != nbytes * self.world:
            raise ValueError("recv must hold world x send's bytes")
        self.kl.check(self.kl.lib().kl_comm_all_gather(self._h, ctypes.c_void_p(send.data_ptr()),
                                                       ctypes.c_void_p(recv.data_ptr()), nbytes,
                                                       ctypes.c_void_p(self._stream(stream))))

    def wait(self, timeout_ms: int, stream=None) -> None:
        import ctypes

        self.kl.check(self.kl.lib().kl_comm_wait(self._h, ctypes.c_void_p(self._stream(stream)), int(timeout_ms)))

    @property
    def aborted(self) -> bool:
        return bool(self.kl.lib().kl_comm_is_aborted(self._h))

    def close(self, timeout_ms: int = 30000) -> None:
        if self._h:
            h, self._h = self._h, None
            self.kl.check(self.kl.lib().kl_comm_destroy(h, int(timeout_ms)))
