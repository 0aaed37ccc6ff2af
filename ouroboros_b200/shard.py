"""Host side of the row-sharded matmul (one process per GPU of one node).

The C ABI (ouroq_shard_*) needs a 128-byte group id on every rank. This module
moves it over an existing torch.distributed process group -- any backend, gloo
included -- so a launcher that already has one (torchrun, the bench) can join
the NCCL group of the library in one call:

    ctx = ouroboros_b200.Context(local_rank)
    rank, world = join(ctx)                 # collective over the process group
    w = ctx.upload_shard(TERNARY2, packed_full, M, K, w_scale=s)
    y = ctx.gemm_sharded(w, x)              # y [B][M] on every rank

Row ownership (ouroq_shard_rows): rank r of G holds rows [r*M/G, (r+1)*M/G);
M must divide evenly. The assembled output interleaves the ranks' blocks per
token, y[b][r*R + i] = rank r's y_r[b][i] (`interleave` states it on the host).
"""
from __future__ import annotations

import numpy as np

from . import shard_rows, shard_unique_id


def join(ctx, group=None) -> tuple[int, int]:
    """Join ctx to a shard group spanning `group` (default: the world group)."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    obj = [shard_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group else 0, group=group)
    ctx.shard_init(obj[0], world, rank)
    return rank, world


def interleave(parts: list[np.ndarray]) -> np.ndarray:
    """Full y [B][M] from the per-rank blocks y_r [B][R], in rank order."""
    return np.concatenate([np.asarray(p).reshape(p.shape[0], -1) for p in parts], axis=1)


def rows_of(M: int, world: int, rank: int) -> slice:
    r0, n = shard_rows(M, world, rank)
    return slice(r0, r0 + n)
