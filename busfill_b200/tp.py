"""Column split of one quantized weight across a process group.

Rank r of g owns weight rows [start, stop) of the N output columns (a
contiguous slice of the packed [N, ...] buffers, for Q4_0 planes and Q4_K
blocks alike), computes C_r[M, stop-start] = A @ deq(W_r)^T with the local
GEMM, and an all-gather over the group (NCCL over NVLink on B200 nodes)
assembles C[M, N]. Every rank needs the full activations A. This is the only
exchange on the path: no reduction, since the K dimension is never split
across ranks.

Shards are whole 128-row tiles (the GEMM's tile height); when N does not
divide evenly the last ranks get fewer rows and every rank pads its slice to
the largest shard for the gather.
"""
from __future__ import annotations

from typing import Callable, Optional

TILE_ROWS = 128


def shard_rows(n: int, world: int, rank: int, align: int = TILE_ROWS) -> tuple[int, int]:
    """Rows [start, stop) of an n-row weight that `rank` of `world` owns.

    Tiles of `align` rows are dealt out as evenly as possible; the extra
    tiles go to the last ranks, which also hold the partial last tile, so
    shards differ by less than one tile. A rank can own zero rows when there
    are fewer tiles than ranks.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n < 0 or align < 1:
        raise ValueError(f"n={n}, align={align}")
    tiles = (n + align - 1) // align
    base, extra = divmod(tiles, world)
    first_big = world - extra          # ranks >= first_big take base + 1 tiles
    t0 = rank * base + max(0, rank - first_big)
    t1 = t0 + base + (1 if rank >= first_big else 0)
    return min(t0 * align, n), min(t1 * align, n)


def max_shard_rows(n: int, world: int, align: int = TILE_ROWS) -> int:
    """Rows of the largest shard (the padded gather width)."""
    return max(stop - start for start, stop in (shard_rows(n, world, r, align) for r in range(world)))


def gather_columns(c_local, n: int, group=None, out=None):
    """All-gather column slices C_r[M, rows_r] (rank order) into C[M, n].

    `c_local` is this rank's slice; slices are padded to the largest shard so
    that one all_gather_into_tensor moves them all.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    m = c_local.shape[0]
    width = max_shard_rows(n, world)
    start, stop = shard_rows(n, world, rank)
    if c_local.shape != (m, stop - start):
        raise ValueError(f"local slice {tuple(c_local.shape)} != ({m}, {stop - start})")
    if stop - start == width and c_local.is_contiguous():
        send = c_local
    else:
        send = torch.zeros((m, width), dtype=c_local.dtype, device=c_local.device)
        send[:, : stop - start] = c_local
    recv = torch.empty((world, m, width), dtype=c_local.dtype, device=c_local.device)
    dist.all_gather_into_tensor(recv.view(world * m, width), send, group=group)
    if out is None:
        out = torch.empty((m, n), dtype=c_local.dtype, device=c_local.device)
    if n == world * width:
        out.view(m, world, width).copy_(recv.permute(1, 0, 2))
    else:
        for r in range(world):
            s0, s1 = shard_rows(n, world, r)
            out[:, s0:s1] = recv[r, :, : s1 - s0]
    return out


def gemm_q4k_tp(blocks_local, a, n: int, group=None, out=None, local_out=None,
                local_gemm: Optional[Callable] = None):
    """C[M, n] = A @ deq(W)^T with W's rows split over `group`.

    `blocks_local` holds this rank's rows of the llama.cpp block_q4_K weight
    (shard_rows(n, world, rank)). `local_gemm(blocks, a) -> C_local` defaults
    to busfill_b200.gemm_q4k (the C ABI on this rank's GPU), writing into
    `local_out` when given.
    """
    from . import gemm_q4k

    if blocks_local.shape[0] == 0:
        c_local = _empty_slice(a)
    elif local_gemm is not None:
        c_local = local_gemm(blocks_local, a)
    else:
        c_local = gemm_q4k(blocks_local, a, out=local_out)
    return gather_columns(c_local, n, group=group, out=out)


def gemm_q4_0_tp(wq_local, ws_local, a, n: int, group=None, out=None, local_out=None,
                 local_gemm: Optional[Callable] = None):
    """As gemm_q4k_tp for the split-plane Q4_0 layout (wq [rows, K/2], ws [rows, K/32])."""
    from . import gemm_q4_0

    if wq_local.shape[0] == 0:
        c_local = _empty_slice(a)
    elif local_gemm is not None:
        c_local = local_gemm(wq_local, ws_local, a)
    else:
        c_local = gemm_q4_0(wq_local, ws_local, a, out=local_out)
    return gather_columns(c_local, n, group=group, out=out)


def _empty_slice(a):
    """The slice of a rank that owns no rows (fewer tiles than ranks)."""
    import torch

    return torch.empty((a.shape[0], 0), dtype=torch.float16, device=a.device)
