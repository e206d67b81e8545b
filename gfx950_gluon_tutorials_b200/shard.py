"""N-sharding of C = A @ B^T across the GPUs of one node.

Each rank holds all of A and a contiguous slab of B's rows (C's columns) and
computes its slab of C with no collective in the loop. An optional NCCL
all-gather then lands every slab in every GPU's own memory as a [world][M][n]
buffer (`gather_slabs`), and `assemble` permutes it to row-major M x N.

The reference has no multi-GPU code; this follows the build target's plan for
its large MXFP4 configuration (16384 x 53248 x 16384 split over 2, 4, 8 GPUs).
"""

from __future__ import annotations

import torch


def shard_range(n: int, world: int, rank: int, align: int = 256) -> tuple[int, int]:
    """[start, stop) of rank's columns: equal slabs rounded to `align` columns
    (whole output tiles), the remainder going to the last ranks' slabs."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    units = -(-n // align)                    # tiles along N
    base, extra = divmod(units, world)
    first = rank * base + max(0, rank - (world - extra))
    count = base + (1 if rank >= world - extra else 0)
    start = min(n, first * align)
    stop = min(n, (first + count) * align)
    return start, stop


def gather_slabs(c_local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather equal-shaped C slabs into a [world][M][n] tensor on every rank."""
    world = torch.distributed.get_world_size(group)
    m, n = c_local.shape
    flat = torch.empty((world * m, n), dtype=c_local.dtype, device=c_local.device)
    torch.distributed.all_gather_into_tensor(flat, c_local.contiguous(), group=group)
    return flat.view(world, m, n)


def assemble(slabs: torch.Tensor) -> torch.Tensor:
    """[world][M][n] -> M x (world * n) row-major (rank r owns columns r*n ..)."""
    world, m, n = slabs.shape
    return slabs.permute(1, 0, 2).reshape(m, world * n)
