"""N-sharding of a GEMM over the ranks of one node (one process per GPU).

Rank r of g owns rows [r*N/g, (r+1)*N/g) of B (the weights) and computes the column block
C[:, shard] = A . B[shard]^T with its own kernel launch: no data moves between GPUs during the
GEMM. Where every rank needs the whole C, `gather_columns` collects the blocks with one
all-gather (NCCL over NVLink on GPUs) and re-lays them out as row-major [M, N].
"""

from __future__ import annotations


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of the N dimension owned by `rank`; shards differ in size by at most one row."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return n * rank // world, n * (rank + 1) // world


def max_over_ranks(x: float, dist=None, device=None) -> float:
    """The maximum of a per-rank float over the process group (the job is as slow as its slowest rank)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    import torch

    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_columns(c_shard, n: int, dist):
    """All-gather the column blocks C[:, shard_r] of every rank into the full row-major C[M, N].

    Shards may differ in width by one column, so each is padded to the widest before the
    collective and cut back afterwards."""
    import torch

    world = dist.get_world_size()
    m = c_shard.shape[0]
    widths = [shard_range(n, world, r)[1] - shard_range(n, world, r)[0] for r in range(world)]
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
