"""Host logic of the row-sharded matmul, on CPU with gloo (world size 2).

What is tested here without a GPU: the row partition (ouroq_shard_rows, a
host-only entry point of the library), the group-id exchange over a
torch.distributed process group, and the data flow of one sharded product --
each rank computes its own rows (with the oracle standing in for the kernels),
the blocks are all-gathered and interleaved in rank order -- against the
unsharded oracle result. The GPU tests (test_shard_gpu.py) run the same flow
through ouroq_gemm_sharded with NCCL.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import ouroboros_b200 as oq
from ouroboros_b200 import shard


@pytest.mark.parametrize("M", [28672, 8192, 4096, 96])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_rows_partition_covers_every_row_once(M, world):
    seen = np.zeros(M, np.int32)
    for r in range(world):
        seen[shard.rows_of(M, world, r)] += 1
    assert np.all(seen == 1)


def test_uneven_rows_rejected():
    with pytest.raises(oq.OuroqError) as ei:
        oq.shard_rows(100, 8, 1)
    assert ei.value.status == 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, M, K, B, out_q):
    import torch
    import torch.distributed as dist
    from oracle import pyoracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # group id: made on rank 0, identical bytes on every rank after the exchange
        obj = [oq.shard_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ids = [None] * world
        dist.all_gather_object(ids, obj[0])
        # every rank holds the same full matrix on the host and uploads only its rows
        w = O.ternary(77, M * K).reshape(M, K)
        ws = O.absmean_scale(w, 0.02)
        packed = O.pack_tern2(w)
        x = O.normals(78, B * K).reshape(B, K)
        q, s = O.quantize_act(x)
        rows = shard.rows_of(M, world, rank)
        _, y_local = O.gemm_tern2(packed[rows], rows.stop - rows.start, K, ws, q, s)
        parts = [torch.empty_like(torch.from_numpy(y_local)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(y_local)))
        y = shard.interleave([p.numpy() for p in parts])
        out_q.put((rank, all(i == ids[0] for i in ids), y))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [1, 3])
def test_two_rank_gloo_sharded_product_matches_unsharded(oracle, B):
    M, K, world = 256, 512, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, M, K, B, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    w = oracle.ternary(77, M * K).reshape(M, K)
    qx, sx = oracle.quantize_act(oracle.normals(78, B * K).reshape(B, K))
    _, want = oracle.gemm_tern2(oracle.pack_tern2(w), M, K, oracle.absmean_scale(w, 0.02), qx, sx)
    for rank, same_id, y in results:
        assert same_id
        assert np.array_equal(y, want)
