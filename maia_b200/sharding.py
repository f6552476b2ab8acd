"""N-sharding of a GEMM over the ranks of one node (one process per GPU).

Rank r of g owns rows [r*N/g, (r+1)*N/g) of B (the weights) and computes the column block
C[:, shard] = A . B[shard]^T with its own kernel launch: no data moves between GPUs during the
GEMM. Where every rank needs the whole C, `gather_columns` collects the blocks with one
all-gather (NCCL over NVLink on GPUs) and re-lays them out as row-major [M, N].
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


def gather_columns(c_shard, n: int, dist, align: int = 1):
    """All-gather the column blocks C[:, shard_r] of every rank into the full row-major C[M, N].

    Shards may differ in width by one column, so each is padded to the widest before the
    collective and cut back afterwards."""
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
        gathered = torch.empty((world, m, wmax), dtype=c_shard.dtype, device=c_shard.device)
        dist.all_gather_into_tensor(gathered, padded)
        parts = list(gathered.unbind(0))
    else:
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded)
    return torch.cat([p[:, :w] for p, w in zip(parts, widths)], dim=1)


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
        self.bases = [kl.ipc_open(h) for r, (h, _) in enumerate(handles) if r != self.rank]
        self.peers = [base + off for base, (r, (_, off)) in
                      zip(self.bases, [(r, x) for r, x in enumerate(handles) if r != self.rank])]
        self.elem = self.full.element_size()

    def peer_ptrs(self, col0: int) -> list[int]:
        return [p + col0 * self.elem for p in self.peers]

    def close(self) -> None:
        for p in self.bases:
            self.kl.ipc_close(p)
        self.bases = []
        self.peers = []
